"""Workload of the bounds-checked library test (run in a subprocess with
TURBOCIDER_CHECKED=1 by test_gpu_checked_build.py): every kernel family on
ragged shapes, each call followed by a status check that must not show
STATUS_BOUNDS (or anything else), and sampled results against the oracle."""
from __future__ import annotations

import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path[:0] = [str(ROOT), str(ROOT / "tests")]

import numpy as np  # noqa: E402
import torch  # noqa: E402

import kq_cases  # noqa: E402
from oracle import oracle  # noqa: E402
from turbocider_b200 import cuda as tcc  # noqa: E402


def main() -> int:
    assert tcc.LIB_PATH.name == "libturbocider_cuda_checked.so", tcc.LIB_PATH
    ctx = tcc.Context(0)
    calls = 0

    def check(label):
        nonlocal calls
        calls += 1
        bits = ctx.status()
        assert bits == 0, f"{label}: status {bits:#x}"

    for typ, n, k in ((12, 1300, 1024), (13, 384, 2048), (14, 200, 768)):
        raw = tcc.quantize(typ, kq_cases.synthetic_weight(n, k, seed=n))
        w = tcc.Weight.upload(ctx, typ, n, k, raw)
        for m, path in ((3, 0), (16, 0), (100, 3), (129, 0), (700, 0), (300, 2)):
            xb = kq_cases.synthetic_x_bf16(m, k, seed=m)
            x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()
            ctx.set_path(path)
            for od in (0, 1, 2):
                y = tcc.qlinear(ctx, w, x, out_dtype=od)
                check(f"type {typ} m {m} path {path} out {od}")
            ctx.set_path(0)
            y = tcc.qlinear(ctx, w, x, out_dtype=0, seg_offsets=[0, m // 3, m], bias=torch.randn(n, device="cuda"),
                            activation="gelu_erf")
            check(f"type {typ} m {m} segments + bias + gelu")
            ref = oracle.epilogue_ref(oracle.qlinear_ref(xb, raw, typ, n, k, "f32" if m <= 16 else "bf16"),
                                      bias=None, activation=None)
            got = tcc.qlinear(ctx, w, x, out_dtype=0).cpu().numpy()
            check("plain f32")
            assert oracle.rel_l2(got, ref) <= (1e-5 if m <= 16 else 1e-4)
        y = tcc.qlinear_small_static(w, torch.randn(4, k, device="cuda").to(torch.bfloat16), out_dtype=tcc.F32)
        assert tcc.small_static_status(0) == 0
        d = tcc.dequant(ctx, w, tcc.BF16)
        check(f"dequant {typ}")
        w.free()
    # SwiGLU and the gated residual through the 2-CTA GEMM (with split-K)
    f, k = 256, 1024
    rg = tcc.quantize(12, kq_cases.synthetic_weight(f, k, seed=1))
    ru = tcc.quantize(12, kq_cases.synthetic_weight(f, k, seed=2))
    wg = tcc.Weight.upload_glu(ctx, 12, f, k, rg, ru)
    x = torch.randn(400, k, device="cuda").to(torch.bfloat16)
    for od in (0, 2):
        tcc.qlinear(ctx, wg, x, out_dtype=od, bias=torch.randn(2 * f, device="cuda"))
        check(f"swiglu out {od}")
    res = torch.randn(400, f, device="cuda")
    tcc.qlinear(ctx, wg, x, out_dtype=0, gate=torch.randn(2, f, device="cuda"), residual=res, seg_offsets=[0, 150, 400],
                seg_gate=[1, 0])
    check("swiglu gated residual")
    # batched GEMV
    ws = [tcc.Weight.upload(ctx, 14, 300, 512, tcc.quantize(14, kq_cases.synthetic_weight(300, 512, seed=i)))
          for i in range(3)]
    tcc.qlinear_batched(ctx, ws, torch.randn(5, 512, device="cuda").to(torch.bfloat16))
    check("batched GEMV")
    # dense weights, odd K
    wd = np.random.default_rng(3).standard_normal((70, 33)).astype(np.float32)
    wt = tcc.Weight.upload(ctx, 0, 70, 33, wd.tobytes())
    tcc.qlinear(ctx, wt, torch.randn(200, 33, device="cuda").to(torch.bfloat16), out_dtype=tcc.F32)
    check("dense")
    # raw decode and gather into exact-size targets
    raw = kq_cases.pattern_case(14, 4, 512)
    src = torch.frombuffer(bytearray(raw), dtype=torch.uint8).cuda()
    tgt = torch.empty(4 * 512 * 4, dtype=torch.uint8, device="cuda")
    tcc.decode(ctx, 14, src, 4, 512, 0, 4, 0, 512, 0, tgt, 2048, 4)
    tcc.decode_gather(ctx, 14, src, 4, 512, torch.tensor([3, 0, 0, 2], device="cuda"), 0, 512, 0, tgt, 2048, 4)
    check("decode / gather")
    ctx.close()
    print(f"checked build: {calls} calls, no bounds violation")
    return 0


if __name__ == "__main__":
    sys.exit(main())
