"""Deterministic K-quant test inputs, shared by the CPU oracle tests, the GPU
parity tests and tests/golden/make_golden.py.

The random-block cases reproduce the inputs of the reference's own decoder
tests: the same seeds, the same per-block draws (random bytes, then a master
scale d from {0, -0, 2^-24, -0.125, 0.03125, 1.5} and, for Q4_K/Q5_K, a dmin
from {0, -0.5, 0.25, 2^-24}) and the same type order, so the K-type blocks are
the ones those tests decode:
  * seed 6409     -- tests/native/test_gguf_execution.py:318-325
                     (12 blocks per trial, 3 rows x 4 blocks, 32 trials);
  * seed 20260930 -- tests/native/test_gguf_execution.py:268-289
                     (3 rows x 3 blocks, three column slices, stride 8).
The pattern and extreme-scale cases restate tests/native/gguf_k_affine_test.cpp:20-26
and tests/native/gguf_decode_safety_test.cpp:64-79.
"""
from __future__ import annotations

import random
import struct

import numpy as np

# GGML type -> (weights per block, bytes per block), dict order as in the
# reference test module (tests/native/test_gguf_execution.py:21-23).
TYPES = {0: (1, 4), 1: (1, 2), 2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 8: (32, 34),
         12: (256, 144), 13: (256, 176), 14: (256, 210), 30: (1, 2)}
K_TYPES = (12, 13, 14)
D_CHOICES = [0., -0., 2 ** -24, -0.125, 0.03125, 1.5]
DMIN_CHOICES = [0., -0.5, 0.25, 2 ** -24]


def random_block(typ: int, rng: random.Random) -> bytes:
    """One random block, consuming the RNG exactly as the reference test does."""
    _, size = TYPES[typ]
    data = bytearray(rng.randbytes(size))
    if typ == 0:
        return struct.pack("<f", rng.uniform(-3, 3))
    if typ == 1:
        return struct.pack("<e", rng.uniform(-3, 3))
    if typ == 30:
        return struct.pack("<H", struct.unpack("<I", struct.pack("<f", rng.uniform(-3, 3)))[0] >> 16)
    offset = 208 if typ == 14 else 0
    data[offset:offset + 2] = struct.pack("<e", rng.choice(D_CHOICES))
    if typ in (3, 7, 12, 13):
        data[2:4] = struct.pack("<e", rng.choice(DMIN_CHOICES))
    return bytes(data)


def seed6409_cases():
    """Yield (typ, trial, raw, rows, cols) for the block types of the seed-6409
    set (Q4_0, Q4_1, Q5_0, Q5_1, Q8_0 and the K-quants)."""
    rng = random.Random(6409)
    for typ in (2, 3, 6, 7, 8, 12, 13, 14):
        elements, _ = TYPES[typ]
        for trial in range(32):
            raw = b"".join(random_block(typ, rng) for _ in range(12))
            yield typ, trial, raw, 3, elements * 4


def seed20260930_cases():
    """Yield (typ, raw, rows, cols, slices) for every registered type of the
    slice set (the floating-point types with 33 columns)."""
    rng = random.Random(20260930)
    for typ, (elements, _) in TYPES.items():
        columns = max(elements * 3, 33 if elements == 1 else elements * 3)
        raw = b"".join(random_block(typ, rng) for _ in range(3 * columns // elements))
        slices = [(0, columns), (1, columns - 2), (elements - 1, min(elements + 2, columns - elements + 1))]
        yield typ, raw, 3, columns, slices


def f16_bits(value: float) -> int:
    return int(np.array([value], dtype=np.float32).astype(np.float16).view(np.uint16)[0])


def pattern_case(typ: int, rows: int, columns: int) -> bytes:
    """Byte pattern (b*41 + i*17) % 256 with d = fp16(.00031*(b%11+1)) and
    dmin = fp16(.00017) (gguf_k_affine_test.cpp:20-26)."""
    _, size = TYPES[typ]
    blocks = rows * columns // 256
    out = bytearray()
    for b in range(blocks):
        p = bytearray(((b * 41 + i * 17) % 256) for i in range(size))
        d = f16_bits(float(np.float32(0.00031) * np.float32(b % 11 + 1)))
        off = 208 if typ == 14 else 0
        p[off:off + 2] = struct.pack("<H", d)
        if typ != 14:
            p[2:4] = struct.pack("<H", f16_bits(0.00017))
        out += p
    return bytes(out)


EXTREME_SCALES = [0.0, -0.0, 2 ** -24, 0.03125, -0.03125, 65504.0, -65504.0]


def extreme_case(typ: int, scale: float) -> bytes:
    """8 blocks of pattern (i*73 + b*17 + 19) & 255 with master scale `scale`
    and dmin -0.015625 (gguf_decode_safety_test.cpp:69-79); 2 rows x 4 blocks."""
    _, size = TYPES[typ]
    out = bytearray()
    for b in range(8):
        p = bytearray(((i * 73 + b * 17 + 19) & 255) for i in range(size))
        off = 208 if typ == 14 else 0
        p[off:off + 2] = struct.pack("<H", f16_bits(scale))
        if typ in (12, 13):
            p[2:4] = struct.pack("<H", f16_bits(-0.015625))
        out += p
    return bytes(out)


def passthrough_cases():
    """Yield (name, typ, raw, rows, cols) for the non-K types' value rules
    (gguf_decode.cpp:56-76, 110 and the converters :389-405): nonfinite
    inputs and scales, fp16 / bf16 overflow, subnormals and signed zeros."""
    f32 = lambda *v: struct.pack(f"<{len(v)}f", *v)
    f16 = lambda *v: struct.pack(f"<{len(v)}H", *v)
    big = struct.unpack("<f", struct.pack("<I", 0x7F7FFFFF))[0]
    yield "f32_inf", 0, f32(1.0, float("inf"), 2.0, 3.0), 1, 4
    yield "f32_nan", 0, f32(0.5, -1.0, float("nan"), 3.0), 2, 2
    yield "f32_max", 0, f32(big, -big, 1.0, 65504.0), 1, 4
    yield "f32_f16_edge", 0, f32(65519.99, 65520.0, 2 ** -25, -2 ** -24), 1, 4
    yield "f32_subnormal_zero", 0, f32(1e-40, -0.0, 2 ** -133, 7.0), 2, 2
    yield "f16_inf", 1, f16(0x3C00, 0x7C00), 1, 2
    yield "f16_subnormal", 1, f16(0x0001, 0x8000, 0x7BFF, 0x03FF), 2, 2
    yield "bf16_nan", 30, f16(0x3F80, 0x7FC0), 1, 2
    yield "bf16_max", 30, f16(0x7F7F, 0xFF7F, 0x0001, 0x477F), 1, 4
    for typ in (2, 3, 6, 7, 8):
        _, size = TYPES[typ]
        for name, off, bits in (("d_inf", 0, 0x7C00), ("d_nan", 0, 0x7E00), ("m_inf", 2, 0x7C00)):
            if name == "m_inf" and typ not in (3, 7):
                continue
            blk = bytearray(((i * 29 + typ) & 255) for i in range(size))
            blk[0:2] = struct.pack("<H", 0x3C00)
            blk[off:off + 2] = struct.pack("<H", bits)
            yield f"{typ}_{name}", typ, bytes(blk) * 2, 2, 32
        blk = bytearray(((i * 53 + 7 * typ) & 255) for i in range(size))
        blk[0:2] = struct.pack("<H", 0x7BFF)   # d = 65504: products overflow fp16
        if typ in (3, 7):
            blk[2:4] = struct.pack("<H", 0xFBFF)
        yield f"{typ}_d_max", typ, bytes(blk), 1, 32


def synthetic_weight(n: int, k: int, seed: int = 0, std: float = 0.02) -> np.ndarray:
    """W ~ N(0, std) fp32 [n, k] from numpy default_rng(seed)."""
    return (np.random.default_rng(seed).standard_normal((n, k), dtype=np.float32) * np.float32(std))


def synthetic_x_bf16(m: int, k: int, seed: int = 1) -> np.ndarray:
    """X ~ N(0, 1) as bf16 bit patterns [m, k] (round-to-nearest-even)."""
    x = np.random.default_rng(seed).standard_normal((m, k), dtype=np.float32)
    b = x.view(np.uint32)
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)


def synthetic_x_f16(m: int, k: int, seed: int = 1) -> np.ndarray:
    """X ~ N(0, 1) as fp16 bit patterns [m, k] (round-to-nearest-even)."""
    x = np.random.default_rng(seed).standard_normal((m, k), dtype=np.float32)
    return x.astype(np.float16).view(np.uint16)
