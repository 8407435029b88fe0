"""World-size-2 test of the N>1 host path on CPU (gloo): each rank takes its
row shard of the raw GGUF bytes, computes its slice of Y with the oracle
(there is no GPU here; on a GPU box the slice comes from tc_cuda_qlinear),
the slices are all-gathered with torch.distributed, and the assembled Y must
equal the full oracle result bit for bit.  Uneven N (padding) included."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import kq_cases
from oracle import oracle
from turbocider_b200 import shard


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, typ, n, k, m, raw, xb, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        block = kq_cases.TYPES[typ][1]
        row_bytes = k // 256 * block
        b, c = shard.shard_rows(n, world, rank)
        per = shard.rows_per_rank(n, world)
        local = np.zeros((m, per), dtype=np.float64)
        if c:
            raw_r = raw[b * row_bytes:(b + c) * row_bytes]
            local[:, :c] = oracle.qlinear_ref(xb, raw_r, typ, c, k, "f32")
        # rank-major gather buffer, flat [world * M, per] as both gloo and NCCL take it
        flat = torch.empty(world * m, per, dtype=torch.float64)
        dist.all_gather_into_tensor(flat, torch.from_numpy(local))
        y = shard.assemble(flat.view(world, m, per), n)
        if rank == 0:
            out_q.put(y.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("typ,n", [(12, 512), (14, 384), (12, 300)])
def test_two_rank_shard_and_gather(typ, n):
    k, m, world = 512, 6, 2
    raw = np.frombuffer(__import__("turbocider_b200.cuda", fromlist=["x"]).quantize(
        typ, kq_cases.synthetic_weight(n, k, seed=n)), dtype=np.uint8)
    xb = kq_cases.synthetic_x_bf16(m, k, seed=3)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, typ, n, k, m, raw, xb, q)) for r in range(world)]
    for p in procs:
        p.start()
    y = q.get(timeout=60)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    full = oracle.qlinear_ref(xb, raw, typ, n, k, "f32")
    assert y.shape == full.shape
    assert np.array_equal(y, full)


def test_shard_rows_cover_exactly():
    for n in (1, 7, 256, 3840, 11520, 10241):
        for world in (1, 2, 3, 4, 8):
            spans = [shard.shard_rows(n, world, r) for r in range(world)]
            assert sum(c for _, c in spans) == n
            pos = 0
            for b, c in spans:
                if c:
                    assert b == pos
                pos += c
