"""TEST INFRASTRUCTURE ONLY: numpy restatement of the backend's K-quant
quantiser (turbocider_b200/csrc/quantize.cpp, tc_quantize).

It exists so that a process which must not load the backend library -- the
CPU reference arm of bench.py, which times the reference's own decoder --
can still build the same synthetic GGUF blocks.  The reference ships no
K-quant encoder; the method is the backend's own min/max fit:

  Q4_K / Q5_K  per 32-weight sub-block g: b_g = max(0, -min w),
               a_g = max(0, (max w + b_g) / L) with L = 15 (Q4_K) or 31 (Q5_K);
               d = fp16(max a_g / 63), dmin = fp16(max b_g / 63);
               sc_g = clamp(rint(a_g / d), 0, 63), m_g = clamp(rint(b_g / dmin), 0, 63);
               code = clamp(rint((w + dmin m_g) / (d sc_g)), 0, L).
  Q6_K         per 16-weight sub-block s: c_s = max|w| / 31;
               d = fp16(max c_s / 127); sc_s = clamp(rint(c_s / d), -128, 127);
               code = clamp(rint(w / (d sc_s)), -32, 31) + 32.

Every step is fp32 arithmetic with round-to-nearest-even, as in the C++
version, so the bytes are identical (tests/test_abi.py checks this against
tc_quantize).  Block layouts follow reference native/core/gguf_decode.cpp:77-105.
"""
from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

BLOCK_BYTES = {12: 144, 13: 176, 14: 210}


def _f16_round(v: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """fp32 -> fp16 bits (RNE) and the fp16 value widened back to fp32."""
    h = v.astype(np.float16)
    return h.view(np.uint16), h.astype(np.float32)


def _max0(v: np.ndarray) -> np.ndarray:
    """std::max(0.f, v): +0 unless 0 < v (so -0 becomes +0, as in C++)."""
    return np.where(np.float32(0) < v, v, np.float32(0)).astype(np.float32)


def _safe_div(num: np.ndarray, den: np.ndarray) -> np.ndarray:
    with np.errstate(divide="ignore", invalid="ignore"):
        return np.where(den > 0, num / np.where(den > 0, den, np.float32(1)), np.float32(0)).astype(np.float32)


def _scale_bytes(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """The 12 packed 6-bit (scale, min) bytes of each block (inverse of
    scale_min, gguf_decode.cpp:48-54).  sc, mn: uint32 [B, 8]."""
    s = np.zeros((sc.shape[0], 12), dtype=np.uint32)
    for g in range(4):
        s[:, g] = sc[:, g] | ((sc[:, g + 4] >> 4) << 6)
        s[:, g + 4] = mn[:, g] | ((mn[:, g + 4] >> 4) << 6)
        s[:, g + 8] = (sc[:, g + 4] & 15) | ((mn[:, g + 4] & 15) << 4)
    return s.astype(np.uint8)


def _affine(w: np.ndarray, levels: int):
    """Q4_K / Q5_K fit of blocks w [B, 8, 32]: (d bits, dmin bits, sc, mn, codes)."""
    lo, hi = w.min(axis=2), w.max(axis=2)
    b = _max0(-lo)
    a = _max0((hi + b) / np.float32(levels))
    dh, d = _f16_round(a.max(axis=1) / np.float32(63))
    mh, dmin = _f16_round(b.max(axis=1) / np.float32(63))
    sc = np.clip(np.rint(_safe_div(a, d[:, None])), 0, 63).astype(np.uint32)
    mn = np.clip(np.rint(_safe_div(b, dmin[:, None])), 0, 63).astype(np.uint32)
    A = d[:, None] * sc.astype(np.float32)
    B = dmin[:, None] * mn.astype(np.float32)
    q = np.clip(np.rint(_safe_div(w + B[:, :, None], A[:, :, None])), 0, levels).astype(np.uint32)
    return dh, mh, sc, mn, q


def _q4k(w: np.ndarray) -> np.ndarray:
    nb = w.shape[0]
    dh, mh, sc, mn, q = _affine(w.reshape(nb, 8, 32), 15)
    out = np.zeros((nb, 144), dtype=np.uint8)
    out[:, 0:2] = dh.view(np.uint8).reshape(nb, 2)
    out[:, 2:4] = mh.view(np.uint8).reshape(nb, 2)
    out[:, 4:16] = _scale_bytes(sc, mn)
    qs = (q[:, 0::2, :] | (q[:, 1::2, :] << 4)).astype(np.uint8)   # [B, 4, 32]
    out[:, 16:144] = qs.reshape(nb, 128)
    return out


def _q5k(w: np.ndarray) -> np.ndarray:
    nb = w.shape[0]
    dh, mh, sc, mn, q = _affine(w.reshape(nb, 8, 32), 31)
    out = np.zeros((nb, 176), dtype=np.uint8)
    out[:, 0:2] = dh.view(np.uint8).reshape(nb, 2)
    out[:, 2:4] = mh.view(np.uint8).reshape(nb, 2)
    out[:, 4:16] = _scale_bytes(sc, mn)
    qh = np.zeros((nb, 32), dtype=np.uint32)
    for g in range(8):
        qh |= (q[:, g, :] >> 4) << g
    out[:, 16:48] = qh.astype(np.uint8)
    lo = q & 15
    out[:, 48:176] = (lo[:, 0::2, :] | (lo[:, 1::2, :] << 4)).astype(np.uint8).reshape(nb, 128)
    return out


def _q6k(w: np.ndarray) -> np.ndarray:
    nb = w.shape[0]
    c = np.abs(w.reshape(nb, 16, 16)).max(axis=2) / np.float32(31)
    dh, d = _f16_round(c.max(axis=1) / np.float32(127))
    sc = np.clip(np.rint(_safe_div(c, d[:, None])), -128, 127).astype(np.int32)
    S = np.repeat(d[:, None] * sc.astype(np.float32), 16, axis=1)          # [B, 256]
    q = (np.clip(np.rint(_safe_div(w, S)), -32, 31).astype(np.int32) + 32).astype(np.uint32)
    q = q.reshape(nb, 2, 4, 32)                                              # [B, h, g, j]
    ql = np.zeros((nb, 2, 2, 32), dtype=np.uint32)                           # [B, h, part, j]
    for g in range(4):
        ql[:, :, g & 1, :] |= (q[:, :, g, :] & 15) << (4 if g >= 2 else 0)
    qh = np.zeros((nb, 2, 32), dtype=np.uint32)
    for g in range(4):
        qh |= (q[:, :, g, :] >> 4) << (2 * g)
    out = np.zeros((nb, 210), dtype=np.uint8)
    out[:, 0:128] = ql.astype(np.uint8).reshape(nb, 128)
    out[:, 128:192] = qh.astype(np.uint8).reshape(nb, 64)
    out[:, 192:208] = sc.astype(np.int8).view(np.uint8)
    out[:, 208:210] = dh.view(np.uint8).reshape(nb, 2)
    return out


def quantize(ggml_type: int, w: np.ndarray, threads: int | None = None) -> np.ndarray:
    """Raw GGUF blocks (uint8, row-major, row pitch cols/256 * block bytes) of
    a finite fp32 [rows, cols] matrix, cols % 256 == 0."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, cols = w.shape
    if cols % 256 or ggml_type not in BLOCK_BYTES:
        raise ValueError("quantize: K-quant type and cols % 256 == 0 required")
    if not np.isfinite(w).all():
        raise ValueError("quantize: nonfinite weight")
    fn = {12: _q4k, 13: _q5k, 14: _q6k}[ggml_type]
    blocks = w.reshape(-1, 256)
    out = np.empty((blocks.shape[0], BLOCK_BYTES[ggml_type]), dtype=np.uint8)
    step = 1 << 15
    threads = threads or os.cpu_count() or 1

    def work(b0: int) -> None:
        out[b0:b0 + step] = fn(blocks[b0:b0 + step])

    with ThreadPoolExecutor(threads) as pool:
        list(pool.map(work, range(0, blocks.shape[0], step)))
    return out.reshape(-1)
