"""Per-layer weight streaming from pinned host memory into HBM.

The reference streams GGUF weights per layer group from the file into device
slots (GgufPackedBank::load_candidate, native/runtime/streaming/
gguf_packed_bank.cpp:374-517, and GgufWeightPager::{fill,bind,retire},
native/runtime/streaming/gguf_weight_pager.cpp:514-670, with a two-slot
read-ahead worker).  Here the host side does the work that needs no GPU once:
each layer's raw K-quant rows are re-laid into the kernels' panel layout
(tc_relayout_host) in pinned memory.  Each step then moves layer l + 1's
panels into one of two resident weight slots with plain asynchronous copies on
a copy stream (tc_cuda_weight_copy_panels: no kernel, so it overlaps the GEMMs
of layer l, which occupy every SM), and the compute stream waits on a per-slot
event before using the slot.

Usage per step::

    stream.begin(compute)                    # prefetch layers 0 and 1
    for l in range(stream.n_layers):
        w = stream.acquire(l, compute)       # {name: Weight}, ready on `compute`
        ... tc_cuda_qlinear(..., w[name], ...) on `compute` ...
        stream.release(l, compute)           # slot free once `compute` is past here
"""
from __future__ import annotations

import os

import numpy as np

from . import cuda as tcc


class LayerStream:
    """layers: list over layers of {name: (ggml_type, n, k, raw_uint8)} -- raw
    GGUF rows of each weight (or of this rank's N-shard).  Panels are built
    once into pinned host memory; two device slots are cycled."""

    def __init__(self, ctx: tcc.Context, layers, device, threads: int | None = None, pinned_cache: dict | None = None,
                 cancel: tcc.CancelFlag | None = None):
        """cancel: a CancelFlag polled while the panels are built (once per
        panel chunk, tc_relayout_host) and before every layer is prefetched or
        acquired, as the reference's pager and bank poll their cancel flag
        (native/runtime/streaming/gguf_weight_pager.cpp,
        gguf_packed_bank.cpp:393-452); a set flag raises tcc.Cancelled, with
        no copy or compute enqueued for the layer."""
        import torch
        self.ctx, self.device, self.cancel = ctx, device, cancel
        self.n_layers = len(layers)
        threads = threads or os.cpu_count() or 1
        # Pinned panel buffers per layer (layers that share raw bytes share buffers
        # through `pinned_cache`, keyed by the raw array's identity).
        cache = pinned_cache if pinned_cache is not None else {}
        self.host = []
        for spec in layers:
            lay = {}
            for name, (typ, n, k, raw) in spec.items():
                key = (id(raw), typ, n, k)
                if key not in cache:
                    buf = torch.empty(tcc.panel_bytes(typ, n, k), dtype=torch.uint8, pin_memory=True)
                    tcc.relayout_host(typ, raw, n, k, out=buf, threads=threads, cancel=cancel)
                    cache[key] = (raw, buf)   # keep raw alive so its id stays unique
                lay[name] = (typ, n, k, cache[key][1])
            self.host.append(lay)
        self.copy = torch.cuda.Stream(device)
        self.slots = [{}, {}]                  # slot -> {(name, typ, n, k): Weight}
        self.ready = [torch.cuda.Event(), torch.cuda.Event()]
        self.free = [None, None]               # event: compute stream is done with the slot
        self.bytes_per_layer = [sum(b.numel() for *_, b in lay.values()) for lay in self.host]

    def _weight(self, slot: int, name: str, typ: int, n: int, k: int) -> tcc.Weight:
        key = (name, typ, n, k)
        w = self.slots[slot].get(key)
        if w is None:
            w = tcc.Weight.create(self.ctx, typ, n, k)
            self.slots[slot][key] = w
        return w

    def _check_cancel(self):
        if self.cancel is not None and self.cancel.is_set:
            raise tcc.Cancelled("generation cancelled")

    def prefetch(self, layer: int):
        """Enqueue layer's panel copies into slot layer % 2 on the copy stream."""
        self._check_cancel()
        slot = layer % 2
        if self.free[slot] is not None:
            self.copy.wait_event(self.free[slot])
        for name, (typ, n, k, buf) in self.host[layer].items():
            self._weight(slot, name, typ, n, k).copy_panels(buf, stream=self.copy)
        self.ready[slot].record(self.copy)

    def begin(self, compute):
        """Start a pass: the copy stream waits for earlier compute work, then
        prefetches the first two layers."""
        import torch
        ev = torch.cuda.Event()
        ev.record(compute)
        self.copy.wait_event(ev)
        self.free = [None, None]
        for layer in range(min(2, self.n_layers)):
            self.prefetch(layer)

    def acquire(self, layer: int, compute) -> dict:
        self._check_cancel()
        slot = layer % 2
        compute.wait_event(self.ready[slot])
        return {name: self._weight(slot, name, typ, n, k) for name, (typ, n, k, _) in self.host[layer].items()}

    def release(self, layer: int, compute):
        """The compute stream is done with layer's slot; prefetch layer + 2 into it."""
        import torch
        ev = torch.cuda.Event()
        ev.record(compute)
        self.free[layer % 2] = ev
        if layer + 2 < self.n_layers:
            self.prefetch(layer + 2)

    def close(self):
        for slot in self.slots:
            for w in slot.values():
                w.free()
            slot.clear()
