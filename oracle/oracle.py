"""TEST INFRASTRUCTURE ONLY: CPU checkers of the K-quant linear path.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
legs may import this module, and only as the checker or the timed CPU
baseline; the product (turbocider_b200) never imports it.

Two decoders are available:
  * "port" -- libkqoracle.so, our C restatement of the reference decoder
    (oracle/kq_oracle.c; reference native/core/gguf_decode.cpp);
  * "ref"  -- _ref/libtcref.so, the reference's own decoder compiled from its
    sources by oracle/Makefile (present wherever it was built; the GPU box
    receives the built file).
The GEMM oracle restates the reference's projection probe
(tools/native/qwen21_gguf_import_probe.cpp:57-74: decode_cpu_into(f32) then an
fp32 matmul) with an fp64 matmul so that only the kernel's own rounding shows.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
PORT_SO = HERE / "libkqoracle.so"
REF_SO = HERE / "_ref" / "libtcref.so"
BLOCK_BYTES = {12: 144, 13: 176, 14: 210}
F32, F16, BF16 = 0, 1, 2

_port = None
_ref = None


def build() -> None:
    """Build the port (always) and the reference decoder (when its sources exist)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True, capture_output=True)


def port() -> C.CDLL:
    global _port
    if _port is None:
        if not PORT_SO.exists():
            build()
        lib = C.CDLL(str(PORT_SO))
        lib.kq_last_error.restype = C.c_char_p
        lib.kq_half_to_float.argtypes = [C.c_uint16]
        lib.kq_half_to_float.restype = C.c_float
        lib.kq_float_to_bf16.argtypes = [C.c_float, C.POINTER(C.c_uint16)]
        lib.kq_float_to_half.argtypes = [C.c_float, C.POINTER(C.c_uint16)]
        lib.kq_decode.argtypes = [C.c_uint32, C.c_void_p] + [C.c_uint64] * 7 + [C.c_uint32, C.c_void_p] + [C.c_uint64] * 3
        _port = lib
    return _port


def ref() -> C.CDLL | None:
    """The reference decoder, or None when it was not built here."""
    global _ref
    if _ref is None and REF_SO.exists():
        lib = C.CDLL(str(REF_SO))
        lib.tc_gguf_test_error.restype = C.c_char_p
        lib.tc_gguf_test_half.argtypes = [C.c_uint16]
        lib.tc_gguf_test_half.restype = C.c_float
        lib.tc_gguf_test_round.argtypes = [C.c_uint32, C.c_float, C.POINTER(C.c_uint16)]
        lib.tc_gguf_test_decode.argtypes = ([C.c_uint32, C.c_void_p] + [C.c_uint64] * 7 + [C.c_uint32, C.c_void_p]
                                            + [C.c_uint64] * 3 + [C.POINTER(C.c_uint64), C.c_uint64, C.c_int,
                                                                   C.POINTER(C.c_uint64)])
        _ref = lib
    return _ref


def _as_u8(raw) -> np.ndarray:
    if isinstance(raw, (bytes, bytearray)):
        return np.frombuffer(raw, dtype=np.uint8)
    return np.ascontiguousarray(raw).view(np.uint8).reshape(-1)


def decode(raw, ggml_type: int, rows: int, cols: int, dtype: int = F32, which: str = "port",
           row_begin: int = 0, nrows: int | None = None, col_begin: int = 0, ncols: int | None = None):
    """Decode a slice of a raw K-quant matrix.  Returns (status, array, error):
    array is float32 (dtype F32) or uint16 bit patterns (F16/BF16), shape
    [nrows, ncols]; on failure array is None and error holds the message."""
    src = _as_u8(raw)
    nrows = rows - row_begin if nrows is None else nrows
    ncols = cols - col_begin if ncols is None else ncols
    item = 4 if dtype == F32 else 2
    out = np.zeros((max(nrows, 1), max(ncols, 1)), dtype=np.float32 if dtype == F32 else np.uint16)
    args = (ggml_type, src.ctypes.data, src.nbytes, rows, cols, row_begin, nrows, col_begin, ncols, dtype,
            out.ctypes.data, out.nbytes, ncols * item, item)
    if which == "port":
        lib = port()
        rc = lib.kq_decode(*args)
        err = lib.kq_last_error().decode()
    else:
        lib = ref()
        if lib is None:
            raise RuntimeError("reference decoder not built (oracle/_ref)")
        stats = (C.c_uint64 * 4)()
        rc = lib.tc_gguf_test_decode(*args, None, 0, 0, stats)
        err = lib.tc_gguf_test_error().decode()
    return rc, (out if rc == 0 else None), err


def decode_gather(raw, ggml_type: int, rows: int, cols: int, indices, dtype: int = F32, which: str = "port",
                  col_begin: int = 0, ncols: int | None = None):
    """decode_cpu_gather (gguf_decode.cpp:446-465): row r of the result is
    source row indices[r].  "ref" runs the reference decoder's own gather
    (its probe's gather mode); "port" decodes the rows one by one with the C
    port and applies the reference's index check.  Returns (status, array,
    error) like decode()."""
    src = _as_u8(raw)
    idx = np.ascontiguousarray(indices, dtype=np.uint64)
    ncols = cols - col_begin if ncols is None else ncols
    item = 4 if dtype == F32 else 2
    out = np.zeros((max(len(idx), 1), max(ncols, 1)), dtype=np.float32 if dtype == F32 else np.uint16)
    if which == "ref":
        lib = ref()
        if lib is None:
            raise RuntimeError("reference decoder not built (oracle/_ref)")
        stats = (C.c_uint64 * 4)()
        rc = lib.tc_gguf_test_decode(ggml_type, src.ctypes.data, src.nbytes, rows, cols, 0, 0, col_begin, ncols,
                                     dtype, out.ctypes.data, out.nbytes, ncols * item, item,
                                     idx.ctypes.data_as(C.POINTER(C.c_uint64)), len(idx), 0, stats)
        err = lib.tc_gguf_test_error().decode()
        return rc, (out if rc == 0 else None), err
    if len(idx) == 0:
        return 1, None, "invalid decode slice"
    for r in idx:
        if int(r) >= rows:
            return 1, None, "gather row out of bounds"
    for i, r in enumerate(idx):
        rc, row, err = decode(raw, ggml_type, rows, cols, dtype, "port", row_begin=int(r), nrows=1,
                              col_begin=col_begin, ncols=ncols)
        if rc:
            return rc, None, err
        out[i] = row[0]
    return 0, out, ""


def decode_checked(raw, ggml_type: int, rows: int, cols: int, dtype: int = F32, which: str = "port") -> np.ndarray:
    rc, out, err = decode(raw, ggml_type, rows, cols, dtype, which)
    if rc:
        raise ValueError(err)
    return out


def decode_parallel(raw, ggml_type: int, rows: int, cols: int, dtype: int = F32, which: str = "ref",
                    threads: int | None = None) -> np.ndarray:
    """Row-split decode over host threads (as the reference's RowDecodePool,
    native/runtime/streaming/gguf_packed_bank.cpp:48-100).  ctypes releases the
    GIL during each call, so the threads run in parallel."""
    src = _as_u8(raw)
    threads = threads or os.cpu_count() or 1
    item = 4 if dtype == F32 else 2
    out = np.empty((rows, cols), dtype=np.float32 if dtype == F32 else np.uint16)
    row_bytes = cols // 256 * BLOCK_BYTES[ggml_type]
    step = (rows + threads - 1) // threads

    def work(r0):
        r1 = min(rows, r0 + step)
        if r0 >= r1:
            return 0
        sub = src[r0 * row_bytes:r1 * row_bytes]
        dst = out[r0:r1]
        if which == "port":
            return port().kq_decode(ggml_type, sub.ctypes.data, sub.nbytes, r1 - r0, cols, 0, r1 - r0, 0, cols,
                                    dtype, dst.ctypes.data, dst.nbytes, cols * item, item)
        stats = (C.c_uint64 * 4)()
        return ref().tc_gguf_test_decode(ggml_type, sub.ctypes.data, sub.nbytes, r1 - r0, cols, 0, r1 - r0, 0,
                                         cols, dtype, dst.ctypes.data, dst.nbytes, cols * item, item, None, 0, 0,
                                         stats)

    with ThreadPoolExecutor(threads) as pool:
        codes = list(pool.map(work, range(0, rows, step)))
    if any(codes):
        raise ValueError("decode failed")
    return out


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (finite inputs)."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)


def kquant_fields(raw, ggml_type: int, n: int, k: int):
    """Per-weight fields of a raw K-quant matrix [n, k], restating the block
    layouts of reference native/core/gguf_decode.cpp:48-54 (scale_min), :77-90
    (Q4_K / Q5_K) and :91-105 (Q6_K).  Returns (code, scale, min, sub) as
    [n, k] arrays: code the integer code (Q6_K: 0..63 with its +32 bias),
    scale = fp32 d * sc, min = fp32 dmin * m (0 for Q6_K), sub = the weight's
    sub-block index inside its super-block (Q4_K / Q5_K: 0..7)."""
    b = _as_u8(raw).reshape(n * (k // 256), BLOCK_BYTES[ggml_type])
    nb = b.shape[0]
    half = lambda lo: b[:, lo:lo + 2].copy().view(np.float16).astype(np.float32).reshape(nb)
    if ggml_type in (12, 13):
        d, dmin = half(0), half(2)
        s6 = b[:, 4:16].astype(np.uint32)
        sc = np.empty((nb, 8), np.uint32)
        mn = np.empty((nb, 8), np.uint32)
        for g in range(8):
            if g < 4:
                sc[:, g], mn[:, g] = s6[:, g] & 63, s6[:, g + 4] & 63
            else:
                sc[:, g] = (s6[:, g + 4] & 0xF) | ((s6[:, g - 4] >> 6) << 4)
                mn[:, g] = (s6[:, g + 4] >> 4) | ((s6[:, g] >> 6) << 4)
        qs = b[:, 16:144] if ggml_type == 12 else b[:, 48:176]
        code = np.empty((nb, 8, 32), np.uint32)
        for g in range(8):
            code[:, g, :] = (qs[:, (g // 2) * 32:(g // 2) * 32 + 32] >> (4 * (g & 1))) & 0xF
            if ggml_type == 13:
                code[:, g, :] |= ((b[:, 16:48] >> g) & 1).astype(np.uint32) << 4
        scale = np.repeat(d[:, None] * sc.astype(np.float32), 32, axis=1)
        mins = np.repeat(dmin[:, None] * mn.astype(np.float32), 32, axis=1)
        sub = np.tile(np.repeat(np.arange(8), 32), (nb, 1))
        return (code.reshape(n, k), scale.reshape(n, k), mins.reshape(n, k), sub.reshape(n, k))
    ql, qh = b[:, 0:128].astype(np.uint32), b[:, 128:192].astype(np.uint32)
    sc8 = b[:, 192:208].copy().view(np.int8).astype(np.float32)
    d = half(208)
    code = np.empty((nb, 256), np.uint32)
    scale = np.empty((nb, 256), np.float32)
    for h in range(2):
        for g in range(4):
            j = np.arange(32)
            lo = (ql[:, 64 * h + 32 * (g & 1) + j] >> (4 if g >= 2 else 0)) & 0xF
            code[:, 128 * h + 32 * g + j] = lo | (((qh[:, 32 * h + j] >> (2 * g)) & 3) << 4)
            scale[:, 128 * h + 32 * g + j] = d[:, None] * sc8[:, 8 * h + j // 16 + 2 * g]
    return code.reshape(n, k), scale.reshape(n, k), np.zeros((n, k), np.float32), None


def f16_staged_weight(raw, ggml_type: int, n: int, k: int) -> np.ndarray:
    """The tensor-core GEMMs' fp16 staging (TC_STAGE_F16 / TC_STAGE_F16_X16):
    fp16(code * s_h - m_h) with one rounding of the exact value
    (fma.rn.f16x2), where s_h = fp16(d sc) (Q4_K's odd sub-blocks, high
    nibbles read in place as 16 code: fp16(d sc / 16)) and m_h = fp16(m')
    with the compensated min m' = m + (m / s) (s_h - s) = m s_h / s while s_h
    is a normal fp16 number (plain m otherwise); Q6_K: fp16((code - 32) * s_h).
    The kernel forms 1 / s with an approximate reciprocal, which can move m_h
    by one fp16 step in rare ties.  Widened exactly to float64."""
    code, scale, mins, sub = kquant_fields(raw, ggml_type, n, k)
    if ggml_type == 14:
        v = (code.astype(np.float64) - 32.0) * scale.astype(np.float16).astype(np.float64)
    else:
        q = code.astype(np.float64)
        s32 = scale.astype(np.float32)
        if ggml_type == 12:
            odd = (sub & 1) == 1
            q = np.where(odd, 16.0 * q, q)
            s32 = np.where(odd, s32 * np.float32(0.0625), s32).astype(np.float32)
        sh = s32.astype(np.float16).astype(np.float64)
        s64, m64 = s32.astype(np.float64), mins.astype(np.float64)
        comp = sh >= 2.0 ** -14
        with np.errstate(divide="ignore", invalid="ignore"):
            mc = np.where(comp, m64 + (m64 / np.where(comp, s64, 1.0)) * (sh - s64), m64)
        mh = mc.astype(np.float32).astype(np.float16).astype(np.float64)
        v = q * sh - mh
    return v.astype(np.float16).astype(np.float64)


def staged_weight(raw, ggml_type: int, n: int, k: int, staging: str, which: str = "port") -> np.ndarray:
    """The weight as the kernel sees it: decode to the staging dtype
    (bf16 / f16 / f32: the reference decoder's values) or "f16k" (the
    tensor-core GEMMs' fp16 staging arithmetic), widened exactly to float64."""
    if staging == "f16k":
        return f16_staged_weight(raw, ggml_type, n, k)
    if staging == "f32":
        return decode_checked(raw, ggml_type, n, k, F32, which).astype(np.float64)
    if staging == "bf16":
        return bf16_bits_to_f32(decode_checked(raw, ggml_type, n, k, BF16, which)).astype(np.float64)
    bits = decode_checked(raw, ggml_type, n, k, F16, which)
    return bits.view(np.float16).astype(np.float64)


def qlinear_ref(x_bits: np.ndarray, raw, ggml_type: int, n: int, k: int, staging: str = "f32",
                which: str = "port", x_dtype: str = "bf16") -> np.ndarray:
    """fp64 oracle of Y = X * W^T.  X is given as bf16 bit patterns [M, K]
    (x_dtype "f16": fp16 bit patterns); with staging "f16" a bf16 X is first
    rounded to fp16 (as the kernel's fp16 mode)."""
    if x_dtype == "f16":
        x = np.asarray(x_bits, dtype=np.uint16).view(np.float16)
    else:
        x = bf16_bits_to_f32(x_bits)
        if staging in ("f16", "f16k"):
            x = x.astype(np.float16)
    w = staged_weight(raw, ggml_type, n, k, staging, which)
    return x.astype(np.float64) @ w.T


def epilogue_ref(acc: np.ndarray, bias=None, activation: str | None = None, glu: bool = False,
                 gate=None, residual=None, gate_rows=None) -> np.ndarray:
    """fp64 restatement of the fused epilogue on a product acc [M, rows]:
    bias add (reference native/backends/mlx.cpp:687-688), GELU (tanh or erf
    form), SwiGLU silu(gate) * up over the halves [gate | up] of a gate_up
    product (native/models/qwen21/transformer.cpp:971-976), then the gated
    residual residual + gate[g(m)] * t (transformer.cpp:950, :980).  acc's
    columns are in logical order (gate rows then up rows for glu); gate_rows
    [M] gives each row's gate vector index."""
    from math import erf, pi, sqrt
    t = np.asarray(acc, dtype=np.float64).copy()
    if bias is not None:
        t = t + np.asarray(bias, dtype=np.float64)[None, :]
    if glu:
        f = t.shape[1] // 2
        g, u = t[:, :f], t[:, f:]
        t = g / (1.0 + np.exp(-g)) * u
    elif activation == "gelu_tanh":
        t = 0.5 * t * (1.0 + np.tanh(sqrt(2.0 / pi) * (t + 0.044715 * t ** 3)))
    elif activation == "gelu_erf":
        t = 0.5 * t * (1.0 + np.vectorize(erf)(t / sqrt(2.0)))
    if gate is not None:
        gv = np.asarray(gate, dtype=np.float64)[np.asarray(gate_rows)]
        t = np.asarray(residual, dtype=np.float64) + gv * t
    return t


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))
