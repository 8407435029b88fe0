"""Generate tests/golden/kquant_golden.json from the reference decoder itself.

Run in a container that has the reference sources (they are compiled by
oracle/Makefile into oracle/_ref/libtcref.so):

    make -C oracle && python tests/golden/make_golden.py

For every case in tests/kq_cases.py and every target dtype (f32 / f16 / bf16)
it records the SHA-256 of the reference decoder's output bytes, or the
reference's error message.  While doing so it asserts that our C port
(oracle/libkqoracle.so) produces identical bytes and messages, and that the
independent gguf-py 0.19.0 ``quants.dequantize`` agrees bit for bit on every
finite Q4_K / Q6_K f32 output.  The JSON is small and committed; the tests
regenerate the inputs deterministically and compare digests.
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

from oracle import oracle  # noqa: E402
import kq_cases  # noqa: E402

OUT = Path(__file__).resolve().parent / "kquant_golden.json"


def digest(rc, out, err):
    if rc:
        return "error: " + err
    return hashlib.sha256(np.ascontiguousarray(out).tobytes()).hexdigest()


def both(raw, typ, rows, cols, dtype, **slice_args):
    r = oracle.decode(raw, typ, rows, cols, dtype, which="ref", **slice_args)
    p = oracle.decode(raw, typ, rows, cols, dtype, which="port", **slice_args)
    dr, dp = digest(*r), digest(*p)
    assert dr == dp, (typ, rows, cols, dtype, slice_args, dr, dp)
    return dr


def gguf_py_check(raw, typ, rows, cols):
    try:
        from gguf import GGMLQuantizationType, quants
    except ImportError:
        return False
    rc, out, _ = oracle.decode(raw, typ, rows, cols, 0, which="ref")
    if rc or typ not in (12, 14):
        return False
    qt = GGMLQuantizationType.Q4_K if typ == 12 else GGMLQuantizationType.Q6_K
    arr = np.frombuffer(raw, dtype=np.uint8).reshape(rows, -1)
    other = quants.dequantize(arr, qt).astype(np.float32)
    assert np.array_equal(other.view(np.uint32), out.view(np.uint32)), ("gguf-py mismatch", typ)
    return True


def main():
    if oracle.ref() is None:
        raise SystemExit("oracle/_ref/libtcref.so is missing: run `make -C oracle` where the reference exists")
    golden = {"generator": "tests/golden/make_golden.py", "decoder": "reference decode_cpu_into via "
              "tests/native/gguf_core_probe.cpp tc_gguf_test_decode", "cases": {}}
    cases = golden["cases"]
    gguf_checked = 0

    cases["seed6409"] = {}
    for typ, trial, raw, rows, cols in kq_cases.seed6409_cases():
        cases["seed6409"].setdefault(str(typ), []).append([both(raw, typ, rows, cols, dt) for dt in (0, 1, 2)])
        gguf_checked += gguf_py_check(raw, typ, rows, cols)

    cases["seed20260930"] = {}
    for typ, raw, rows, cols, slices in kq_cases.seed20260930_cases():
        entry = []
        for begin, count in slices:
            entry.append([both(raw, typ, rows, cols, dt, col_begin=begin, ncols=count) for dt in (0, 1, 2)])
        cases["seed20260930"][str(typ)] = entry

    cases["pattern"] = {}
    for typ in kq_cases.K_TYPES:
        for rows in (1, 3, 17):
            for cols in (256, 512, 1024):
                raw = kq_cases.pattern_case(typ, rows, cols)
                cases["pattern"][f"{typ}/{rows}x{cols}"] = [both(raw, typ, rows, cols, dt) for dt in (0, 1, 2)]
                gguf_checked += gguf_py_check(raw, typ, rows, cols)

    cases["extreme"] = {}
    for typ in kq_cases.K_TYPES:
        for scale in kq_cases.EXTREME_SCALES:
            raw = kq_cases.extreme_case(typ, scale)
            cases["extreme"][f"{typ}/{scale!r}"] = [both(raw, typ, 2, 1024, dt) for dt in (0, 1, 2)]

    cases["passthrough"] = {}
    for name, typ, raw, rows, cols in kq_cases.passthrough_cases():
        cases["passthrough"][name] = [both(raw, typ, rows, cols, dt) for dt in (0, 1, 2)]

    cases["nonfinite"] = {}
    for typ in kq_cases.K_TYPES:
        for bits, where in ((0x7C00, "d"), (0x7E00, "d"), (0x7C00, "dmin")):
            if where == "dmin" and typ == 14:
                continue
            raw = bytearray(kq_cases.extreme_case(typ, 1.0))
            off = 208 if typ == 14 else (0 if where == "d" else 2)
            raw[off:off + 2] = bits.to_bytes(2, "little")
            cases["nonfinite"][f"{typ}/{where}/{bits:#06x}"] = [both(bytes(raw), typ, 2, 1024, dt) for dt in (0, 1, 2)]

    # Config-1 weight (Q4_K [3072, 3072], N(0, 0.02), seed 0) through our
    # quantiser: pins the quantiser's determinism and the decode of its blocks.
    sys.path.insert(0, str(ROOT))
    from turbocider_b200 import cuda as tcc
    w = kq_cases.synthetic_weight(3072, 3072, seed=0)
    raw = tcc.quantize(12, w)
    decoded = oracle.decode_parallel(raw, 12, 3072, 3072, 0, which="ref")
    cases["config1_q4k"] = {
        "raw_sha256": hashlib.sha256(raw.tobytes()).hexdigest(),
        "f32_sha256": hashlib.sha256(decoded.tobytes()).hexdigest(),
        "rel_l2_vs_w": oracle.rel_l2(decoded, w),
    }
    w6 = kq_cases.synthetic_weight(256, 12288, seed=2)
    raw6 = tcc.quantize(14, w6)
    dec6 = oracle.decode_parallel(raw6, 14, 256, 12288, 0, which="ref")
    cases["q6k_256x12288"] = {
        "raw_sha256": hashlib.sha256(raw6.tobytes()).hexdigest(),
        "f32_sha256": hashlib.sha256(dec6.tobytes()).hexdigest(),
        "rel_l2_vs_w": oracle.rel_l2(dec6, w6),
    }
    golden["gguf_py_crosschecked_cases"] = gguf_checked
    OUT.write_text(json.dumps(golden, indent=1, sort_keys=True) + "\n")
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes); gguf-py cross-checked {gguf_checked} cases")


if __name__ == "__main__":
    main()
