"""GPU parity of the 2-CTA GEMM's split-K form.

When a call has fewer 256 x 256 tiles than half the GPU's SM pairs, every
tile is computed as ksplit units over equal shares of the K super-blocks;
the units' fp32 partials are added in split order by a reduce kernel that
also applies the fused epilogue.  Checks: against the oracle (weights staged
like the kernel, fp64 matmul) at rel-L2 <= 1e-4 with f32 output, and against
the same call without the split (forced by capping the GEMM to 2 SMs, one
pair, which any tile count fills) at <= 1e-5: only fp32 summation order
differs.
"""
from __future__ import annotations

import numpy as np
import pytest

import kq_cases
from oracle import oracle

pytestmark = pytest.mark.gpu

TIGHT = 1e-4


def _x(m, k, seed):
    import torch
    xb = kq_cases.synthetic_x_bf16(m, k, seed=seed)
    return xb, torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()


def _unsplit(ctx, *args, **kw):
    from turbocider_b200 import cuda as tcc
    ctx.set_sm_limit(2)
    try:
        return tcc.qlinear(ctx, *args, **kw)
    finally:
        ctx.set_sm_limit(0)


@pytest.mark.parametrize("typ", [12, 13, 14])
@pytest.mark.parametrize("m,n,k,expect_split", [(256, 3072, 3072, 6),   # 12 tiles
                                                (300, 512, 2048, 8),    # 4 tiles, 1 super-block per share
                                                (200, 256, 768, 3),     # 1 tile, K = 3 super-blocks
                                                (1000, 640, 2560, 5),   # 12 tiles, odd panel count
                                                (129, 130, 512, 2)])    # ragged N and M
def test_split_k_matches_oracle_and_unsplit(ctx, typ, m, n, k, expect_split):
    from turbocider_b200 import cuda as tcc
    raw = tcc.quantize(typ, kq_cases.synthetic_weight(n, k, seed=m + n + typ))
    w = tcc.Weight.upload(ctx, typ, n, k, raw)
    xb, x = _x(m, k, m)
    kern, split = ctx.plan(w, m)
    assert kern == 2 and split == expect_split, (kern, split)
    ctx.set_sm_limit(2)
    assert ctx.plan(w, m) == (2, 1)
    ctx.set_sm_limit(0)
    y = tcc.qlinear(ctx, w, x, out_dtype=tcc.F32).cpu().numpy().astype(np.float64)
    y1 = _unsplit(ctx, w, x, out_dtype=tcc.F32).cpu().numpy().astype(np.float64)
    assert ctx.status() == 0
    assert oracle.rel_l2(y, oracle.qlinear_ref(xb, raw, typ, n, k, "bf16")) <= TIGHT
    assert oracle.rel_l2(y, y1) <= 1e-5
    # fp16 staging from bf16 X, fp16 out
    y16 = tcc.qlinear(ctx, w, x, out_dtype=tcc.F16, stage=tcc.STAGE_F16).float().cpu().numpy()
    assert oracle.rel_l2(y16, oracle.qlinear_ref(xb, raw, typ, n, k, "f32")) <= 1e-3
    w.free()


def test_split_k_ragged_segments_two_weights(ctx):
    """Three segments over two weights (image / text stream), every one
    longer than 128 rows, few tiles in total: split units of different
    segments and weights in one launch, one reduce per segment."""
    from turbocider_b200 import cuda as tcc
    n, k = 384, 1536
    raws = [tcc.quantize(t, kq_cases.synthetic_weight(n, k, seed=90 + t)) for t in (12, 12)]
    ws = [tcc.Weight.upload(ctx, 12, n, k, r) for r in raws]
    seg, sw = [0, 150, 410, 700], [0, 1, 0]
    xb, x = _x(700, k, 5)
    assert ctx.plan(ws[0], 700)[1] > 1
    y = tcc.qlinear(ctx, ws, x, seg_offsets=seg, seg_weight=sw, out_dtype=tcc.F32).cpu().numpy()
    y1 = _unsplit(ctx, ws, x, seg_offsets=seg, seg_weight=sw, out_dtype=tcc.F32).cpu().numpy()
    assert ctx.status() == 0
    for i in range(3):
        a, b = seg[i], seg[i + 1]
        ref = oracle.qlinear_ref(xb[a:b], raws[sw[i]], 12, n, k, "bf16")
        assert oracle.rel_l2(y[a:b], ref) <= TIGHT, i
    assert oracle.rel_l2(y, y1) <= 1e-5


@pytest.mark.parametrize("out_dtype,bound", [(0, 1e-4), (1, 1e-3), (2, 3e-3)])
def test_split_k_fused_epilogues(ctx, out_dtype, bound):
    """Bias + GELU, SwiGLU (with gate / up biases) and the per-segment gated
    residual through the split-K reduce."""
    import torch
    from turbocider_b200 import cuda as tcc
    k, m = 2048, 260
    xb, x = _x(m, k, 8)
    rng = np.random.default_rng(4)
    # bias + GELU
    n = 512
    raw = tcc.quantize(14, kq_cases.synthetic_weight(n, k, seed=3))
    w = tcc.Weight.upload(ctx, 14, n, k, raw)
    bias = rng.standard_normal(n).astype(np.float32)
    y = tcc.qlinear(ctx, w, x, out_dtype=out_dtype, bias=torch.from_numpy(bias).cuda(), activation="gelu_tanh")
    ref = oracle.epilogue_ref(oracle.qlinear_ref(xb, raw, 14, n, k, "bf16"), bias=bias, activation="gelu_tanh")
    assert oracle.rel_l2(y.float().cpu().numpy(), ref) <= bound
    # SwiGLU
    f = 256
    rg = tcc.quantize(12, kq_cases.synthetic_weight(f, k, seed=6))
    ru = tcc.quantize(12, kq_cases.synthetic_weight(f, k, seed=7))
    wg = tcc.Weight.upload_glu(ctx, 12, f, k, rg, ru)
    gb = rng.standard_normal(2 * f).astype(np.float32)
    y = tcc.qlinear(ctx, wg, x, out_dtype=out_dtype, bias=torch.from_numpy(gb).cuda())
    acc = np.concatenate([oracle.qlinear_ref(xb, rg, 12, f, k, "bf16"), oracle.qlinear_ref(xb, ru, 12, f, k, "bf16")],
                         axis=1)
    assert oracle.rel_l2(y.float().cpu().numpy(), oracle.epilogue_ref(acc, bias=gb, glu=True)) <= bound
    # gated residual, two segments with their own gate rows
    seg, seg_gate = [0, 130, m], [1, 0]
    gate = rng.standard_normal((2, n)).astype(np.float32)
    tdt = {0: torch.float32, 1: torch.float16, 2: torch.bfloat16}[out_dtype]
    res = torch.from_numpy(rng.standard_normal((m, n)).astype(np.float32)).to(tdt).cuda()
    res_host = res.float().cpu().numpy()
    y = tcc.qlinear(ctx, w, x, seg_offsets=seg, out_dtype=out_dtype, gate=torch.from_numpy(gate).cuda(),
                    residual=res, seg_gate=seg_gate)
    rows = np.array([1] * 130 + [0] * (m - 130))
    ref = oracle.epilogue_ref(oracle.qlinear_ref(xb, raw, 14, n, k, "bf16"), gate=gate, residual=res_host,
                              gate_rows=rows)
    assert oracle.rel_l2(y.float().cpu().numpy(), ref) <= bound
    assert ctx.status() == 0
    for ww in (w, wg):
        ww.free()
