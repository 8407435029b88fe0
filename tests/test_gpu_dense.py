"""GPU checks of dense ("passthrough") weights: the F32 / F16 / BF16 and
Q4_0 / Q4_1 / Q5_0 / Q5_1 / Q8_0 tensors of a K-quant model file.

* tc_cuda_weight_upload keeps them resident; tc_cuda_dequant is bit-exact to
  the reference decoder (through the C port) for every target dtype;
* tc_cuda_qlinear runs them as a library GEMM with fp32 accumulation: f32
  output within 1e-4 (relative L2) of the fp64 oracle that stages W and X like
  the call (bf16, or fp16 for the fp16 modes), fused epilogues and bf16 output
  within 3e-3; K need not be a multiple of 256;
* weights whose values leave the fp16 range refuse the fp16 modes.
"""
from __future__ import annotations

import random
import struct

import numpy as np
import pytest

import kq_cases
from oracle import oracle

pytestmark = pytest.mark.gpu

TIGHT = 1e-4


def dense_raw(typ: int, n: int, k: int, seed: int) -> bytes:
    """Raw GGUF rows [n, k]: N(0, 0.05) values for the floating-point types,
    random blocks (the reference tests' generator) for the block types."""
    if typ in (0, 1, 30):
        w = np.random.default_rng(seed).standard_normal((n, k)).astype(np.float32) * np.float32(0.05)
        if typ == 0:
            return w.tobytes()
        if typ == 1:
            return w.astype(np.float16).tobytes()
        return oracle.f32_to_bf16_bits(w).tobytes()
    rng = random.Random(seed)
    elements, _ = kq_cases.TYPES[typ]
    return b"".join(kq_cases.random_block(typ, rng) for _ in range(n * k // elements))


TYPES = [0, 1, 30, 2, 3, 6, 7, 8]


@pytest.mark.parametrize("typ", TYPES)
def test_dense_dequant_bit_exact(ctx, typ):
    from turbocider_b200 import cuda as tcc
    n, k = 130, 96 if typ not in (0, 1, 30) else 50
    raw = dense_raw(typ, n, k, seed=typ)
    w = tcc.Weight.upload(ctx, typ, n, k, raw)
    assert (w.n, w.k) == (n, k)
    for dt in (0, 1, 2):
        got = tcc.dequant(ctx, w, dt).cpu()
        ref = oracle.decode_checked(raw, typ, n, k, dt)
        got_np = got.view(__import__("torch").int16).numpy().view(np.uint16) if dt else got.numpy()
        assert np.array_equal(np.ascontiguousarray(got_np).view(np.uint8), np.ascontiguousarray(ref).view(np.uint8))
    assert ctx.status() == 0
    # a row shard
    s = tcc.Weight.upload(ctx, typ, n, k, raw, n_begin=33, n_count=64)
    got = tcc.dequant(ctx, s, tcc.F32).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), oracle.decode_checked(raw, typ, n, k, 0)[33:97].view(np.uint32))


@pytest.mark.parametrize("typ", TYPES)
@pytest.mark.parametrize("m", [3, 300])
def test_dense_linear(ctx, typ, m):
    import torch
    from turbocider_b200 import cuda as tcc
    n, k = 192, 160 if typ not in (0, 1, 30) else 72
    raw = dense_raw(typ, n, k, seed=10 + typ)
    w = tcc.Weight.upload(ctx, typ, n, k, raw)
    xb = kq_cases.synthetic_x_bf16(m, k, seed=m)
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()
    y = tcc.qlinear(ctx, w, x, out_dtype=tcc.F32).cpu().numpy()
    assert ctx.status() == 0
    assert oracle.rel_l2(y, oracle.qlinear_ref(xb, raw, typ, n, k, "bf16")) <= TIGHT
    # fp16 activations and fp16 output, as the reference's GGUF execution runs
    xh = kq_cases.synthetic_x_f16(m, k, seed=m + 1)
    xf = torch.from_numpy(xh.view(np.int16)).view(torch.float16).cuda()
    yh = tcc.qlinear(ctx, w, xf, out_dtype=tcc.F16, stage=tcc.STAGE_F16_X16).float().cpu().numpy()
    assert oracle.rel_l2(yh, oracle.qlinear_ref(xh, raw, typ, n, k, "f16", x_dtype="f16")) <= 1e-3
    # fused epilogue: bias, tanh GELU, gated residual; bf16 output
    rng = np.random.default_rng(typ)
    bias = rng.standard_normal(n).astype(np.float32)
    gate = rng.standard_normal((1, n)).astype(np.float32)
    res = torch.randn(m, n, device="cuda").to(torch.bfloat16)
    yb = tcc.qlinear(ctx, w, x, out_dtype=tcc.BF16, bias=torch.from_numpy(bias).cuda(), activation="gelu_tanh",
                     gate=torch.from_numpy(gate).cuda(), residual=res, seg_gate=[0]).float().cpu().numpy()
    ref = oracle.epilogue_ref(oracle.qlinear_ref(xb, raw, typ, n, k, "bf16"), bias=bias, activation="gelu_tanh",
                              gate=gate, residual=res.float().cpu().numpy(), gate_rows=np.zeros(m, int))
    assert oracle.rel_l2(yb, ref) <= 3e-3
    assert ctx.status() == 0


def test_dense_and_kquant_segments_in_one_call(ctx):
    """Segments on a Q4_K weight and on a Q8_0 weight of the same shape."""
    import torch
    from turbocider_b200 import cuda as tcc
    n, k = 256, 512
    rq = tcc.quantize(12, kq_cases.synthetic_weight(n, k, seed=3))
    rd = dense_raw(8, n, k, seed=4)
    wq, wd = tcc.Weight.upload(ctx, 12, n, k, rq), tcc.Weight.upload(ctx, 8, n, k, rd)
    segs = [0, 200, 260, 264]
    xb = kq_cases.synthetic_x_bf16(segs[-1], k, seed=5)
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()
    y = tcc.qlinear(ctx, [wq, wd], x, seg_offsets=segs, seg_weight=[0, 1, 0], out_dtype=tcc.F32).cpu().numpy()
    assert ctx.status() == 0
    assert oracle.rel_l2(y[:200], oracle.qlinear_ref(xb[:200], rq, 12, n, k, "bf16")) <= TIGHT
    assert oracle.rel_l2(y[200:260], oracle.qlinear_ref(xb[200:260], rd, 8, n, k, "bf16")) <= TIGHT
    assert oracle.rel_l2(y[260:], oracle.qlinear_ref(xb[260:], rq, 12, n, k, "f32")) <= 1e-5


def test_dense_fp16_range_and_errors(ctx):
    import torch
    from turbocider_b200 import cuda as tcc
    n, k = 8, 32
    w = np.full((n, k), 0.5, np.float32)
    w[3, 7] = 1e6                      # beyond fp16
    wt = tcc.Weight.upload(ctx, 0, n, k, w.tobytes())
    x = torch.ones(4, k, dtype=torch.bfloat16, device="cuda")
    y = tcc.qlinear(ctx, wt, x, out_dtype=tcc.F32)
    assert abs(float(y[0, 3]) - (1e6 + 15.5)) < 1e6 * 2 ** -7
    with pytest.raises(tcc.BackendError, match="fp16 range"):
        tcc.qlinear(ctx, wt, x, stage=tcc.STAGE_F16)
    bad = np.zeros((2, 32), np.float32)
    bad[1, 5] = np.inf
    with pytest.raises(tcc.DecodeError, match="nonfinite"):
        tcc.Weight.upload(ctx, 0, 2, 32, bad.tobytes())
    big = np.full((1, 4), struct.unpack("<f", struct.pack("<I", 0x7F7FFFFF))[0], np.float32)
    with pytest.raises(tcc.DecodeError, match="BF16 conversion overflow"):
        tcc.Weight.upload(ctx, 0, 1, 4, big.tobytes())
    with pytest.raises(tcc.DecodeError, match="invalid source geometry"):
        tcc.Weight.upload(ctx, 8, 2, 48, dense_raw(8, 2, 64, seed=1))
    with pytest.raises(tcc.BackendError, match="dense weights"):
        tcc.qlinear_batched(ctx, [wt], x)
    assert ctx.status() == 0


@pytest.mark.parametrize("typ,n,k,m", [(0, 40, 33, 5), (1, 130, 100, 300), (30, 96, 7, 129),
                                       (8, 3072, 4096, 700), (2, 1000, 2048, 64)])
def test_dense_tensor_core_gemm_shapes(ctx, typ, n, k, m):
    """The dense GEMM (TMA-fed tcgen05, no library GEMM): K not a multiple of
    8 (X copied to a 16-byte row pitch, boxes past K zero-filled), N not a
    multiple of 128, several token tiles, a realistic Q8_0 size."""
    import torch
    from turbocider_b200 import cuda as tcc
    raw = dense_raw(typ, n, k, seed=n + k)
    w = tcc.Weight.upload(ctx, typ, n, k, raw)
    xb = kq_cases.synthetic_x_bf16(m, k, seed=k)
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()
    y = tcc.qlinear(ctx, w, x, out_dtype=tcc.F32).cpu().numpy()
    assert ctx.status() == 0
    assert oracle.rel_l2(y, oracle.qlinear_ref(xb, raw, typ, n, k, "bf16")) <= TIGHT
    y16 = tcc.qlinear(ctx, w, x, out_dtype=tcc.F16, stage=tcc.STAGE_F16).float().cpu().numpy()
    assert oracle.rel_l2(y16, oracle.qlinear_ref(xb, raw, typ, n, k, "f16")) <= 1e-3
    w.free()
