"""GPU parity of the fused epilogues of tc_cuda_qlinear_ex and of fp16 output.

Each kernel family runs every epilogue: the GEMV (5 rows), the one-CTA GEMM
(100 rows) and the 2-CTA pair GEMM (300 rows).  The oracle is the fp64
product of the same staged weights (oracle.qlinear_ref) followed by the fp64
epilogue restatement (oracle.epilogue_ref).

Tolerances (relative L2 over the whole output):
  * f32 output: GEMM <= 1e-4 against the oracle staged like the kernel (bf16),
    GEMV <= 1e-5 against the exact-decode oracle (only fp32 summation order
    and the epilogue's fp32 arithmetic differ);
  * f16 output: <= 1e-3 (fp16 rounding of the result);
  * bf16 output: <= 3e-3 (bf16 rounding of the result).
"""
from __future__ import annotations

import numpy as np
import pytest

import kq_cases
from oracle import oracle

pytestmark = pytest.mark.gpu

# (rows of X, forced path, staging of the oracle, f32 bound)
PATHS = {"gemv": (5, 0, "f32", 1e-5), "one_cta": (100, 3, "bf16", 1e-4), "pair": (300, 0, "bf16", 1e-4)}
OUT_BOUND = {0: None, 1: 1e-3, 2: 3e-3}


def _x(m, k, seed):
    import torch
    xb = kq_cases.synthetic_x_bf16(m, k, seed=seed)
    return xb, torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()


def _run(ctx, path, *args, **kw):
    from turbocider_b200 import cuda as tcc
    ctx.set_path(path)
    try:
        y = tcc.qlinear(ctx, *args, **kw)
    finally:
        ctx.set_path(0)
    assert ctx.status() == 0
    return y.float().cpu().numpy().astype(np.float64)


def _bound(out_dtype, f32_bound):
    return f32_bound if out_dtype == 0 else OUT_BOUND[out_dtype]


@pytest.mark.parametrize("where", list(PATHS))
@pytest.mark.parametrize("typ", [12, 14])
@pytest.mark.parametrize("act", [None, "gelu_tanh", "gelu_erf"])
@pytest.mark.parametrize("out_dtype", [0, 1, 2])
def test_bias_and_gelu(ctx, where, typ, act, out_dtype):
    import torch
    from turbocider_b200 import cuda as tcc
    m, path, staging, f32b = PATHS[where]
    n, k = 384, 1024
    raw = tcc.quantize(typ, kq_cases.synthetic_weight(n, k, seed=typ + 3))
    w = tcc.Weight.upload(ctx, typ, n, k, raw)
    xb, x = _x(m, k, 11)
    bias = np.random.default_rng(5).standard_normal(n).astype(np.float32)
    y = _run(ctx, path, w, x, out_dtype=out_dtype, bias=torch.from_numpy(bias).cuda(), activation=act)
    ref = oracle.epilogue_ref(oracle.qlinear_ref(xb, raw, typ, n, k, staging), bias=bias, activation=act)
    assert oracle.rel_l2(y, ref) <= _bound(out_dtype, f32b)


def _glu_case(ctx, typ, f, k, seed, col_begin=0, col_count=0):
    from turbocider_b200 import cuda as tcc
    rg = tcc.quantize(typ, kq_cases.synthetic_weight(f, k, seed=seed))
    ru = tcc.quantize(typ, kq_cases.synthetic_weight(f, k, seed=seed + 1))
    w = tcc.Weight.upload_glu(ctx, typ, f, k, rg, ru, col_begin, col_count)
    return rg, ru, w


@pytest.mark.parametrize("where", list(PATHS))
@pytest.mark.parametrize("typ", [12, 13, 14])
@pytest.mark.parametrize("out_dtype", [0, 2])
def test_swiglu(ctx, where, typ, out_dtype):
    """silu(X Wg^T + bg) * (X Wu^T + bu) from one interleaved weight."""
    import torch
    from turbocider_b200 import cuda as tcc
    m, path, staging, f32b = PATHS[where]
    f, k = 320, 768
    rg, ru, w = _glu_case(ctx, typ, f, k, seed=20 + typ)
    assert (w.n, w.n_out, w.glu) == (2 * f, f, True)
    xb, x = _x(m, k, 12)
    bias = np.random.default_rng(6).standard_normal(2 * f).astype(np.float32) * 0.5
    y = _run(ctx, path, w, x, out_dtype=out_dtype, bias=torch.from_numpy(bias).cuda())
    assert y.shape == (m, f)
    acc = np.concatenate([oracle.qlinear_ref(xb, rg, typ, f, k, staging), oracle.qlinear_ref(xb, ru, typ, f, k, staging)],
                         axis=1)
    ref = oracle.epilogue_ref(acc, bias=bias, glu=True)
    assert oracle.rel_l2(y, ref) <= _bound(out_dtype, f32b)


def test_swiglu_shard_and_dequant_order(ctx):
    """A column shard of a SwiGLU weight holds gate rows c and up rows c of its
    columns, interleaved in 8-row groups (visible through tc_cuda_dequant)."""
    from turbocider_b200 import cuda as tcc
    f, k, c0, cn = 256, 512, 64, 96
    rg, ru, w = _glu_case(ctx, 12, f, k, seed=40, col_begin=c0, col_count=cn)
    assert (w.n, w.n_out) == (2 * cn, cn)
    got = tcc.dequant(ctx, w, tcc.F32).cpu().numpy()
    dg = oracle.decode_checked(rg, 12, f, k, 0)[c0:c0 + cn]
    du = oracle.decode_checked(ru, 12, f, k, 0)[c0:c0 + cn]
    want = np.empty((2 * cn, k), np.float32)
    for grp in range(cn // 8):
        want[16 * grp:16 * grp + 8] = dg[8 * grp:8 * grp + 8]
        want[16 * grp + 8:16 * grp + 16] = du[8 * grp:8 * grp + 8]
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("where", list(PATHS))
@pytest.mark.parametrize("out_dtype", [0, 1, 2])
def test_gated_residual_per_segment(ctx, where, out_dtype):
    """Two ragged segments (image / text stream) with their own weights and
    gate vectors: y = residual + gate[seg_gate[s]] * (X W_s^T + b)."""
    import torch
    from turbocider_b200 import cuda as tcc
    m, path, staging, f32b = PATHS[where]
    n, k = 256, 512
    ra = tcc.quantize(12, kq_cases.synthetic_weight(n, k, seed=50))
    rb = tcc.quantize(14, kq_cases.synthetic_weight(n, k, seed=51))
    wa, wb = tcc.Weight.upload(ctx, 12, n, k, ra), tcc.Weight.upload(ctx, 14, n, k, rb)
    split = m // 3 if m > 16 else 2
    segs = [0, split, m]
    xb, x = _x(m, k, 13)
    rng = np.random.default_rng(7)
    bias = rng.standard_normal(n).astype(np.float32)
    gate = rng.standard_normal((3, n)).astype(np.float32)
    tdt = tcc._torch_dtype(out_dtype)
    res = torch.randn(m, n, device="cuda").to(tdt)
    y = _run(ctx, path, [wa, wb], x, seg_offsets=segs, seg_weight=[1, 0], out_dtype=out_dtype,
             bias=torch.from_numpy(bias).cuda(), gate=torch.from_numpy(gate).cuda(), residual=res, seg_gate=[2, 0])
    acc = np.concatenate([oracle.qlinear_ref(xb[:split], rb, 14, n, k, staging),
                          oracle.qlinear_ref(xb[split:], ra, 12, n, k, staging)])
    rows = np.array([2] * split + [0] * (m - split))
    ref = oracle.epilogue_ref(acc, bias=bias, gate=gate, residual=res.float().cpu().numpy(), gate_rows=rows)
    assert oracle.rel_l2(y, ref) <= _bound(out_dtype, f32b)


@pytest.mark.parametrize("where", list(PATHS))
def test_gated_residual_in_place(ctx, where):
    """hidden += gate * (X W^T): the residual is the output tensor itself."""
    import torch
    from turbocider_b200 import cuda as tcc
    m, path, staging, f32b = PATHS[where]
    n, k = 384, 768
    raw = tcc.quantize(12, kq_cases.synthetic_weight(n, k, seed=60))
    w = tcc.Weight.upload(ctx, 12, n, k, raw)
    xb, x = _x(m, k, 14)
    gate = torch.randn(1, n, device="cuda")
    hidden = torch.randn(m, n, device="cuda")
    before = hidden.cpu().numpy().astype(np.float64)
    _run(ctx, path, w, x, out_dtype=tcc.F32, gate=gate, residual=hidden, seg_gate=[0], out=hidden)
    ref = oracle.epilogue_ref(oracle.qlinear_ref(xb, raw, 12, n, k, staging), gate=gate.cpu().numpy(),
                              residual=before, gate_rows=np.zeros(m, int))
    assert oracle.rel_l2(hidden.cpu().numpy(), ref) <= f32b


@pytest.mark.parametrize("where", list(PATHS))
@pytest.mark.parametrize("typ", [12, 13, 14])
def test_f16_output_plain(ctx, where, typ):
    """fp16 Y (the reference's output dtype for fp16 activations), no epilogue;
    the pair kernel writes it with TMA stores."""
    from turbocider_b200 import cuda as tcc
    m, path, staging, _ = PATHS[where]
    n, k = 512, 1024
    raw = tcc.quantize(typ, kq_cases.synthetic_weight(n, k, seed=70))
    w = tcc.Weight.upload(ctx, typ, n, k, raw)
    xb, x = _x(m, k, 15)
    y = _run(ctx, path, w, x, out_dtype=tcc.F16)
    assert oracle.rel_l2(y, oracle.qlinear_ref(xb, raw, typ, n, k, staging)) <= 1e-3


def test_f16_everything_fp16_activations(ctx):
    """fp16 X (TC_STAGE_F16_X16), fp16 Y, SwiGLU + bias: the reference's GGUF
    execution dtypes; <= 1e-3 against the fp32-decode oracle."""
    import torch
    from turbocider_b200 import cuda as tcc
    f, k, m = 256, 1024, 600
    rg, ru, w = _glu_case(ctx, 12, f, k, seed=80)
    xh = kq_cases.synthetic_x_f16(m, k, seed=16)
    x = torch.from_numpy(xh.view(np.int16)).view(torch.float16).cuda()
    bias = np.random.default_rng(8).standard_normal(2 * f).astype(np.float32) * 0.1
    y = tcc.qlinear(ctx, w, x, out_dtype=tcc.F16, stage=tcc.STAGE_F16_X16, bias=torch.from_numpy(bias).cuda())
    assert ctx.status() == 0
    acc = np.concatenate([oracle.qlinear_ref(xh, rg, 12, f, k, "f32", x_dtype="f16"),
                          oracle.qlinear_ref(xh, ru, 12, f, k, "f32", x_dtype="f16")], axis=1)
    ref = oracle.epilogue_ref(acc, bias=bias, glu=True)
    assert oracle.rel_l2(y.float().cpu().numpy(), ref) <= 1e-3


def test_epilogue_argument_errors(ctx):
    import ctypes as C
    import torch
    from turbocider_b200 import cuda as tcc
    n, k = 256, 512
    raw = tcc.quantize(12, kq_cases.synthetic_weight(n, k, seed=90))
    w = tcc.Weight.upload(ctx, 12, n, k, raw)
    rg, ru, wg = _glu_case(ctx, 12, 64, k, seed=91)
    x = torch.zeros(40, k, dtype=torch.bfloat16, device="cuda")
    y = torch.empty(40, n, device="cuda")
    lib = tcc.lib()

    def call(weight, epi, out=y):
        h = (C.c_void_p * 1)(weight.handle)
        offs = (C.c_int32 * 2)(0, 40)
        return lib.tc_cuda_qlinear_ex(ctx.handle, h, 1, offs, None, 1, x.data_ptr(), out.data_ptr(), 0, 0, 0,
                                      C.byref(epi), None)

    def err():
        return lib.tc_cuda_last_error().decode()

    e = tcc.Epilogue(flags=tcc.EPI_SWIGLU)
    assert call(w, e) == 1 and "needs a weight from tc_cuda_weight_upload_glu" in err()
    assert call(wg, tcc.Epilogue(flags=tcc.EPI_BIAS, bias=y.data_ptr())) == 1 and "needs TC_EPI_SWIGLU" in err()
    assert call(w, tcc.Epilogue(flags=tcc.EPI_GELU_TANH | tcc.EPI_GELU_ERF)) == 1 and "at most one activation" in err()
    assert call(w, tcc.Epilogue(flags=tcc.EPI_BIAS)) == 1 and "needs a bias vector" in err()
    assert call(w, tcc.Epilogue(flags=1 << 9)) == 1 and "unknown epilogue flag" in err()
    g = torch.zeros(1, n, device="cuda")
    e = tcc.Epilogue(flags=tcc.EPI_GATE_RESIDUAL, gate=g.data_ptr(), residual=y.data_ptr(), n_gate_rows=0)
    assert call(w, e) == 1 and "gate row out of range" in err()
    with pytest.raises(tcc.DecodeError, match="multiple of 8"):
        tcc.Weight.upload_glu(ctx, 12, 64, k, rg, ru, 0, 12)
    with pytest.raises(tcc.BackendError, match="SwiGLU"):
        tcc.qlinear_batched(ctx, [wg], x[:4])
    assert ctx.status() == 0
