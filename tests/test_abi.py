"""CPU tests of the C-ABI library: it loads, exports every function declared
in include/*.h, refuses to run without a B200 (no CPU fallback), and its host
quantiser is deterministic and decodable by the reference decoder."""
from __future__ import annotations

import ctypes as C
import hashlib
import re
from pathlib import Path

import numpy as np
import pytest

import kq_cases
from oracle import oracle
from turbocider_b200 import cuda as tcc

ROOT = Path(__file__).resolve().parents[1]


def declared_functions():
    names = []
    for header in sorted((ROOT / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        names += re.findall(r"\b(tc_[a-z0-9_]+)\s*\(", text)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    lib = tcc.lib()
    names = declared_functions()
    assert len(names) >= 15
    for name in names:
        assert hasattr(lib, name), name
        assert name in tcc.EXPORTS, f"{name} has no ctypes signature in turbocider_b200/cuda.py"


def test_abi_version():
    assert tcc.lib().tc_cuda_abi_version() == 2


def test_init_fails_loudly_without_b200():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    h = C.c_void_p()
    assert tcc.lib().tc_cuda_init(0, C.byref(h)) == 1
    assert "no CUDA device" in tcc.lib().tc_cuda_last_error().decode()
    with pytest.raises(tcc.BackendError):
        tcc.Context(0)


def test_null_arguments_rejected_without_device():
    lib = tcc.lib()
    assert lib.tc_cuda_status(None, None, 0) == 1
    assert lib.tc_cuda_dequant(None, None, 0, None, 0, None) == 1
    assert lib.tc_cuda_qlinear(None, None, 0, None, None, 0, None, None, 0, 2, 0, None) == 1
    assert lib.tc_cuda_last_error().decode() == "null argument"


def test_quantiser_pinned_and_decodable(golden):
    w = kq_cases.synthetic_weight(3072, 3072, seed=0)
    raw = tcc.quantize(12, w)
    g = golden["cases"]["config1_q4k"]
    assert hashlib.sha256(raw.tobytes()).hexdigest() == g["raw_sha256"]
    dec = oracle.decode_parallel(raw, 12, 3072, 3072, 0, which="port")
    assert hashlib.sha256(dec.tobytes()).hexdigest() == g["f32_sha256"]
    assert 0.03 < oracle.rel_l2(dec, w) < 0.10


def test_q6k_quantiser_pinned(golden):
    w = kq_cases.synthetic_weight(256, 12288, seed=2)
    raw = tcc.quantize(14, w)
    g = golden["cases"]["q6k_256x12288"]
    assert hashlib.sha256(raw.tobytes()).hexdigest() == g["raw_sha256"]
    dec = oracle.decode_parallel(raw, 14, 256, 12288, 0, which="port")
    assert hashlib.sha256(dec.tobytes()).hexdigest() == g["f32_sha256"]
    assert oracle.rel_l2(dec, w) < 0.03


def test_q5k_quantiser_between_q4k_and_q6k():
    """Q5_K blocks from tc_quantize decode identically through the port and the
    reference decoder, and their error sits between Q4_K's and Q6_K's."""
    w = kq_cases.synthetic_weight(64, 2048, seed=5)
    err = {}
    for typ in (12, 13, 14):
        raw = tcc.quantize(typ, w)
        assert raw.nbytes == 64 * 8 * tcc.BLOCK_BYTES[typ]
        dec = oracle.decode_parallel(raw, typ, 64, 2048, 0, which="port")
        ref = oracle.decode_parallel(raw, typ, 64, 2048, 0, which="ref")
        assert np.array_equal(dec.view(np.uint32), ref.view(np.uint32))
        err[typ] = oracle.rel_l2(dec, w)
    assert err[14] < err[13] < err[12]
    assert err[13] < 0.05


def test_quantiser_threads_do_not_change_bytes():
    w = kq_cases.synthetic_weight(33, 512, seed=7)
    for typ in (12, 13, 14):
        assert np.array_equal(tcc.quantize(typ, w, threads=1), tcc.quantize(typ, w, threads=5))


def test_quantiser_rejects_bad_input():
    with pytest.raises(tcc.BackendError):
        tcc.quantize(12, np.zeros((2, 100), np.float32))
    bad = np.zeros((1, 256), np.float32)
    bad[0, 3] = np.nan
    with pytest.raises(tcc.BackendError):
        tcc.quantize(14, bad)
    with pytest.raises(KeyError):
        tcc.quantize(10, np.zeros((1, 256), np.float32))


@pytest.mark.parametrize("typ", [12, 13, 14])
def test_numpy_quantiser_matches_tc_quantize(typ):
    """oracle/kq_quantize.py (used where the backend library must not be
    loaded: the CPU reference arm of bench.py) produces the same bytes as
    tc_quantize, including all-zero sub-blocks, an all-zero row and large
    and tiny scales."""
    from oracle import kq_quantize
    from turbocider_b200 import cuda as tcc
    rng = np.random.default_rng(typ)
    w = (rng.standard_normal((40, 1024)) * 0.02).astype(np.float32)
    w[3] = 0.0
    w[5, :40] = 0.0
    w[7] *= 3000.0
    w[9] *= 1e-6
    w[11] = np.abs(w[11])
    w[13] = -np.abs(w[13])
    assert np.array_equal(kq_quantize.quantize(typ, w, threads=3), tcc.quantize(typ, w))
    big = kq_cases.synthetic_weight(300, 2048, seed=typ)
    assert np.array_equal(kq_quantize.quantize(typ, big), tcc.quantize(typ, big))
