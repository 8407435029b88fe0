"""Cancellation of the loader path on the host (no GPU): tc_gguf_read and
tc_relayout_host honour a caller-owned cancel flag and return
TC_CUDA_CANCELLED, as the reference's decoder, bank and read-ahead worker
poll their cancel flag once per block or chunk (native/core/gguf_decode.cpp:
44-47, :344; native/runtime/streaming/read_ahead_worker.hpp:21-70).

Mid-stream cancels are made deterministic without timing: a watcher thread
sets the flag as soon as the call's first output lands in the destination,
so the call must stop with most of the destination still untouched."""
from __future__ import annotations

import threading

import numpy as np
import pytest

import kq_cases
from test_gguf_reader import fixture
from turbocider_b200 import cuda as tcc


def _watch(buf: np.ndarray, flag: tcc.CancelFlag, probe: slice) -> threading.Thread:
    """Set `flag` once buf[probe] holds a nonzero byte."""
    def run():
        for _ in range(20_000_000):
            if buf[probe].any():
                flag.set()
                return
    t = threading.Thread(target=run, daemon=True)
    t.start()
    return t


def test_flag_set_before_the_call():
    flag = tcc.CancelFlag()
    flag.set()
    raw = np.frombuffer(kq_cases.pattern_case(12, 4, 512), dtype=np.uint8)
    with pytest.raises(tcc.Cancelled, match="generation cancelled"):
        tcc.relayout_host(12, raw, 4, 512, cancel=flag)
    flag.clear()
    assert tcc.relayout_host(12, raw, 4, 512, cancel=flag).any()


def test_relayout_cancelled_mid_stream():
    """One worker thread walks the panel chunks in order; the flag is raised
    when the first chunk is written, so the last chunk stays untouched."""
    typ, n, k = 12, 8192, 4096
    raw = np.random.default_rng(1).integers(0, 256, n * (k // 256) * 144, dtype=np.uint8)
    raw.reshape(-1, 144)[:, 0:4] = np.frombuffer(np.float16([0.01, 0.001]).tobytes(), np.uint8)   # finite d, dmin
    out = np.zeros(tcc.panel_bytes(typ, n, k), dtype=np.uint8)
    flag = tcc.CancelFlag()
    chunk = out.size // (n // 128 * (k // 256))
    w = _watch(out, flag, slice(0, chunk))
    with pytest.raises(tcc.Cancelled):
        tcc.relayout_host(typ, raw, n, k, out=out, threads=1, cancel=flag)
    w.join(timeout=10)
    assert flag.is_set and not out[-chunk:].any()


def test_gguf_read_cancelled_mid_stream(tmp_path):
    """tc_gguf_read preads at most 8 MiB at a time and checks the flag before
    each: raised after the first piece lands, the read stops short."""
    rows, k = 2048, 12288                       # Q6_K rows of 10080 bytes: 20.6 MB
    row = k // 256 * 210
    payload = np.random.default_rng(2).integers(1, 256, rows * row, dtype=np.uint8).tobytes()
    path = tmp_path / "big.gguf"
    path.write_bytes(fixture([("w", 14, [k, rows])], payload=payload))
    f = tcc.GGUFFile(path)
    dst = np.zeros(rows * row, dtype=np.uint8)
    flag = tcc.CancelFlag()
    w = _watch(dst, flag, slice(0, 4096))
    with pytest.raises(tcc.Cancelled, match="generation cancelled"):
        f.read("w", out=dst, cancel=flag)
    w.join(timeout=10)
    assert not dst[-(1 << 20):].any()
    flag.clear()
    assert f.read("w", out=dst, cancel=flag).tobytes() == payload
    f.close()
