"""GPU parity at exactly the configuration bench.py measures (BASELINE
configs[4], the Z-Image-style stack at M = 8448): fp16 activations as given
and W staged fp16 (TC_STAGE_F16_X16), the Q4_K qkv projection, the SwiGLU
w1 / w3 pair as one interleaved weight with biases (silu(w1 x + b1) *
(w3 x + b3) in the epilogue), and the Q6_K ffn_down at K = 10240, with fp16
and bf16 outputs.

Oracle: the reference decoder's f32 dequantisation and an fp64 matmul of the
same fp16 X rows (oracle.qlinear_ref, restating
tools/native/qwen21_gguf_import_probe.cpp:57-74), with the SwiGLU applied in
fp64 (oracle.epilogue_ref).  64 sampled rows, every output column.
Bars (rel-L2): fp16 output <= 1e-3 (output rounding
included); bf16 output <= 3e-3 (bf16 output rounding alone is ~1.6e-3);
f32 output against the oracle that stages W in fp16 as the kernel does
(oracle "f16k") <= 1e-4.
"""
from __future__ import annotations

import numpy as np
import pytest

import kq_cases
from oracle import oracle

pytestmark = pytest.mark.gpu

M = 8448
HIDDEN, FFN = 3840, 10240


@pytest.fixture(scope="module")
def x16():
    import torch
    xh = kq_cases.synthetic_x_f16(M, FFN, seed=41)
    return xh, torch.from_numpy(xh.view(np.int16)).view(torch.float16).cuda()


def _rows():
    return np.sort(np.random.default_rng(7).choice(M, 64, replace=False))


@pytest.mark.parametrize("typ,n,k", [(12, 3 * HIDDEN, HIDDEN), (14, HIDDEN, FFN), (12, HIDDEN, FFN)])
def test_bench_linear_fp16_io(ctx, x16, typ, n, k):
    import torch
    from turbocider_b200 import cuda as tcc
    xh_all, x_all = x16
    xh, x = np.ascontiguousarray(xh_all[:, :k]), x_all[:, :k].contiguous()
    raw = tcc.quantize(typ, kq_cases.synthetic_weight(n, k, seed=n + k))
    w = tcc.Weight.upload(ctx, typ, n, k, raw)
    rows = _rows()
    ref = oracle.qlinear_ref(xh[rows], raw, typ, n, k, "f32", x_dtype="f16")
    idx = torch.from_numpy(rows).cuda()
    y16 = tcc.qlinear(ctx, w, x, out_dtype=tcc.F16, stage=tcc.STAGE_F16_X16)
    e16 = oracle.rel_l2(y16.index_select(0, idx).float().cpu().numpy(), ref)
    yb = tcc.qlinear(ctx, w, x, out_dtype=tcc.BF16, stage=tcc.STAGE_F16_X16)
    eb = oracle.rel_l2(yb.index_select(0, idx).float().cpu().numpy(), ref)
    y32 = tcc.qlinear(ctx, w, x, out_dtype=tcc.F32, stage=tcc.STAGE_F16_X16)
    e32 = oracle.rel_l2(y32.index_select(0, idx).cpu().numpy(),
                        oracle.qlinear_ref(xh[rows], raw, typ, n, k, "f16k", x_dtype="f16"))
    assert ctx.status() == 0
    print(f"type {typ} [{n}, {k}]: fp16 out {e16:.2e}, bf16 out {eb:.2e}, f32 out vs fp16-staged {e32:.2e}")
    assert e16 <= 1e-3
    assert eb <= 3e-3
    assert e32 <= 1e-4
    w.free()


@pytest.mark.parametrize("out_dtype,bar", [(1, 1e-3), (2, 3e-3)])
def test_bench_swiglu_fp16_io(ctx, x16, out_dtype, bar):
    """The bench's FFN input projection: w1 / w3 [10240, 3840] Q4_K as one
    interleaved SwiGLU weight, with a gate and an up bias."""
    import torch
    from turbocider_b200 import cuda as tcc
    xh_all, x_all = x16
    k = HIDDEN
    xh, x = np.ascontiguousarray(xh_all[:, :k]), x_all[:, :k].contiguous()
    r1 = tcc.quantize(12, kq_cases.synthetic_weight(FFN, k, seed=61))
    r3 = tcc.quantize(12, kq_cases.synthetic_weight(FFN, k, seed=62))
    w = tcc.Weight.upload_glu(ctx, 12, FFN, k, r1, r3)
    bias = (np.random.default_rng(63).standard_normal(2 * FFN) * 0.1).astype(np.float32)
    bias_d = torch.from_numpy(bias).cuda()
    y = tcc.qlinear(ctx, w, x, out_dtype=out_dtype, stage=tcc.STAGE_F16_X16, bias=bias_d)
    assert ctx.status() == 0
    assert y.shape == (M, FFN)
    rows = _rows()
    acc = np.concatenate([oracle.qlinear_ref(xh[rows], r1, 12, FFN, k, "f32", x_dtype="f16"),
                          oracle.qlinear_ref(xh[rows], r3, 12, FFN, k, "f32", x_dtype="f16")], axis=1)
    ref = oracle.epilogue_ref(acc, bias=bias, glu=True)
    got = y.index_select(0, torch.from_numpy(rows).cuda()).float().cpu().numpy()
    e = oracle.rel_l2(got, ref)
    print(f"SwiGLU out dtype {out_dtype}: rel-L2 {e:.2e}")
    assert e <= bar
    w.free()
