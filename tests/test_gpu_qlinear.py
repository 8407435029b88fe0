"""GPU parity of the quantised linear (tc_cuda_qlinear) against the fp64
oracle (reference decoder semantics + fp64 matmul).

Tolerances (relative L2 over the whole output):
  * fp32 output vs the oracle that stages W exactly as the kernel does
    (bf16 by default: the reference decoder's bf16 values; fp16 staging:
    oracle "f16k", fp16(code * fp16(d sc) - fp16(dmin m))):   <= 1e-4  (TIGHT)
    -- only the kernel's fp32 accumulation order differs;
  * warp GEMV (exact fp32 dequant) vs the fp32-decode oracle: <= 1e-5;
  * fp16 staging vs the fp32-decode oracle:                  <= 1e-3  (north-star bar);
  * bf16 staging vs the fp32-decode oracle:                  <= 3e-3  (bf16 W rounding
    alone costs ~1.6e-3);
  * bf16 output vs the staged oracle:                        <= 3e-3  (bf16 output rounding).
At the full config-5 sizes a sampled-row check is used (every row of the
sample against the oracle), since the full fp64 oracle would take minutes.
"""
from __future__ import annotations

import numpy as np
import pytest

import kq_cases
from oracle import oracle

pytestmark = pytest.mark.gpu

TIGHT = 1e-4


def _setup(ctx, typ, n, k, m, wseed=0, xseed=1):
    import torch
    from turbocider_b200 import cuda as tcc
    raw = tcc.quantize(typ, kq_cases.synthetic_weight(n, k, seed=wseed))
    weight = tcc.Weight.upload(ctx, typ, n, k, raw)
    xb = kq_cases.synthetic_x_bf16(m, k, seed=xseed)
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()
    return raw, weight, xb, x


def _run(ctx, weight, x, out_dtype, stage=0, path=0, seg=None, seg_w=None, weights=None):
    from turbocider_b200 import cuda as tcc
    ctx.set_path(path)
    try:
        y = tcc.qlinear(ctx, weights or weight, x, seg_offsets=seg, seg_weight=seg_w, out_dtype=out_dtype, stage=stage)
    finally:
        ctx.set_path(0)
    assert ctx.status() == 0
    return y.float().cpu().numpy().astype(np.float64)


@pytest.mark.parametrize("typ", [12, 13, 14])
def test_gemm_config1_shape(ctx, typ):
    """Config 1 (M=256, N=3072, K=3072) through the tcgen05 GEMM."""
    from turbocider_b200 import cuda as tcc
    n = k = 3072
    raw, w, xb, x = _setup(ctx, typ, n, k, 256)
    y = _run(ctx, w, x, tcc.F32)
    e_staged = oracle.rel_l2(y, oracle.qlinear_ref(xb, raw, typ, n, k, "bf16"))
    e_f32 = oracle.rel_l2(y, oracle.qlinear_ref(xb, raw, typ, n, k, "f32"))
    print(f"type {typ}: rel-L2 vs bf16-staged oracle {e_staged:.2e}, vs f32-decode oracle {e_f32:.2e}")
    assert e_staged <= TIGHT
    assert e_f32 <= 3e-3
    yb = _run(ctx, w, x, tcc.BF16)
    assert oracle.rel_l2(yb, oracle.qlinear_ref(xb, raw, typ, n, k, "bf16")) <= 3e-3


@pytest.mark.parametrize("typ", [12, 13, 14])
def test_gemm_fp16_staging_meets_1e3_vs_f32_decode(ctx, typ):
    from turbocider_b200 import cuda as tcc
    n, k, m = 1024, 2048, 384
    raw, w, xb, x = _setup(ctx, typ, n, k, m, wseed=11)
    y = _run(ctx, w, x, tcc.F32, stage=tcc.STAGE_F16)
    assert oracle.rel_l2(y, oracle.qlinear_ref(xb, raw, typ, n, k, "f16k")) <= TIGHT
    e = oracle.rel_l2(y, oracle.qlinear_ref(xb, raw, typ, n, k, "f32"))
    print(f"type {typ} fp16 staging vs f32 decode: {e:.2e}")
    assert e <= 1e-3


@pytest.mark.parametrize("path", [2, 3])
@pytest.mark.parametrize("typ", [12, 13, 14])
@pytest.mark.parametrize("m,n,k", [(17, 200, 512), (129, 384, 1024), (300, 256, 768), (64, 130, 256),
                                   (1000, 640, 2560), (520, 1920, 512)])
def test_gemm_ragged_edges(ctx, typ, m, n, k, path):
    """M and N not multiples of the tile: every one-CTA BN variant (64/128/256,
    path 3) and the 2-CTA 256 x 256 tile (path 2, M > 128), including odd panel
    counts (N = 384, 640, 1920 -> 3, 5, 15 panels of 128 rows)."""
    from turbocider_b200 import cuda as tcc
    raw, w, xb, x = _setup(ctx, typ, n, k, m, wseed=m + n)
    y = _run(ctx, w, x, tcc.F32, path=path)
    assert oracle.rel_l2(y, oracle.qlinear_ref(xb, raw, typ, n, k, "bf16")) <= TIGHT


@pytest.mark.parametrize("typ", [12, 13, 14])
@pytest.mark.parametrize("ldy", [640, 648, 645])
def test_gemm_bf16_out_row_stride(ctx, typ, ldy):
    """bf16 output into a wider buffer (row stride ldy): TMA-stored tiles when
    the row pitch is a multiple of 16 bytes (640, 648), plain stores otherwise
    (645); columns past N stay untouched."""
    import torch
    from turbocider_b200 import cuda as tcc
    m, n, k = 300, 640, 768
    raw, w, xb, x = _setup(ctx, typ, n, k, m, wseed=ldy)
    big = torch.full((m, ldy), 7.0, dtype=torch.bfloat16, device=x.device)
    out = big[:, :n]
    tcc.qlinear(ctx, w, x, out=out)
    assert ctx.status() == 0
    y = out.float().cpu().numpy().astype(np.float64)
    assert oracle.rel_l2(y, oracle.qlinear_ref(xb, raw, typ, n, k, "bf16")) <= 3e-3
    if ldy > n:
        assert bool((big[:, n:] == 7.0).all())
    ctx.set_path(3)
    try:
        y1 = tcc.qlinear(ctx, w, x).float().cpu().numpy().astype(np.float64)
    finally:
        ctx.set_path(0)
    assert oracle.rel_l2(y, y1) <= 3e-3


@pytest.mark.parametrize("typ", [12, 13, 14])
@pytest.mark.parametrize("m", [1, 2, 3, 4, 16])
def test_gemv_config2_shape(ctx, typ, m):
    """Config 2 (K=12288, N=3072, M in {1..16}) through the warp GEMV."""
    from turbocider_b200 import cuda as tcc
    n, k = 3072, 12288
    raw, w, xb, x = _setup(ctx, typ, n, k, m, wseed=2)
    y = _run(ctx, w, x, tcc.F32)
    assert oracle.rel_l2(y, oracle.qlinear_ref(xb, raw, typ, n, k, "f32")) <= 1e-5
    yb = _run(ctx, w, x, tcc.BF16)
    assert oracle.rel_l2(yb, oracle.qlinear_ref(xb, raw, typ, n, k, "f32")) <= 3e-3


@pytest.mark.parametrize("typ", [12, 13, 14])
@pytest.mark.parametrize("m", [1, 5, 16])
@pytest.mark.parametrize("n,k", [(64, 12288), (16, 12288), (1000, 2048), (48, 3072), (16, 4096)])
def test_gemv_k_split_reductions(ctx, typ, m, n, k):
    """The GEMV's K-slice sums through the workspace and the last-arriving CTA
    of each row tile.  One token (16-row tiles, K also split across the
    CTA's warps): 6 slices at k=12288, 1 at n=1000 / n=48, 2 at n=16, k=4096;
    several tokens (64-row tiles): 24 slices at k=12288, 4 (n=1000), 6
    (n=48), 8 (n=16, k=4096).  Each runs twice, so a tile counter not left
    at zero by the first call would break the second."""
    from turbocider_b200 import cuda as tcc
    raw, w, xb, x = _setup(ctx, typ, n, k, m, wseed=n + m)
    ref = oracle.qlinear_ref(xb, raw, typ, n, k, "f32")
    for _ in range(2):
        y = _run(ctx, w, x, tcc.F32)
        assert oracle.rel_l2(y, ref) <= 1e-5
    assert ctx.status() == 0


def test_forced_paths_agree(ctx):
    """M=40 through the GEMV (forced) and through the GEMM."""
    from turbocider_b200 import cuda as tcc
    n, k, m = 512, 1024, 40
    raw, w, xb, x = _setup(ctx, 12, n, k, m, wseed=4)
    yv = _run(ctx, w, x, tcc.F32, path=1)
    yg = _run(ctx, w, x, tcc.F32, path=2)
    assert oracle.rel_l2(yv, oracle.qlinear_ref(xb, raw, 12, n, k, "f32")) <= 1e-5
    assert oracle.rel_l2(yg, oracle.qlinear_ref(xb, raw, 12, n, k, "bf16")) <= TIGHT


def test_ragged_segments_two_weights(ctx):
    """Three request segments packed along M (image / text streams): two use
    weight A, one uses weight B; the 3-row segment goes to the GEMV."""
    import torch
    from turbocider_b200 import cuda as tcc
    n, k = 384, 1024
    segs = [0, 512, 515, 772]
    ra = tcc.quantize(12, kq_cases.synthetic_weight(n, k, seed=21))
    rb = tcc.quantize(12, kq_cases.synthetic_weight(n, k, seed=22))
    wa, wb = tcc.Weight.upload(ctx, 12, n, k, ra), tcc.Weight.upload(ctx, 12, n, k, rb)
    xb = kq_cases.synthetic_x_bf16(segs[-1], k, seed=23)
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()
    y = _run(ctx, None, x, tcc.F32, seg=segs, seg_w=[0, 1, 0], weights=[wa, wb])
    ya = oracle.qlinear_ref(xb, ra, 12, n, k, "bf16")
    yb = oracle.qlinear_ref(xb, rb, 12, n, k, "bf16")
    yf = oracle.qlinear_ref(xb, ra, 12, n, k, "f32")
    assert oracle.rel_l2(y[0:512], ya[0:512]) <= TIGHT
    assert oracle.rel_l2(y[512:515], oracle.qlinear_ref(xb[512:515], rb, 12, n, k, "f32")) <= 1e-5
    assert oracle.rel_l2(y[515:772], ya[515:772]) <= TIGHT
    assert oracle.rel_l2(y[0:512], yf[0:512]) <= 3e-3
    del yb


def test_ragged_segments_three_types(ctx):
    """Segments on Q4_K, Q5_K and Q6_K weights of one shape in one call (the
    Q4_K_M mix puts different types behind the same projection in different
    blocks); the pair kernel, the one-CTA kernel and the GEMV each get one."""
    import torch
    from turbocider_b200 import cuda as tcc
    n, k = 512, 1024
    segs = [0, 300, 340, 344, 600]
    types = [12, 13, 14]
    raws = [tcc.quantize(t, kq_cases.synthetic_weight(n, k, seed=40 + t)) for t in types]
    ws = [tcc.Weight.upload(ctx, t, n, k, r) for t, r in zip(types, raws)]
    xb = kq_cases.synthetic_x_bf16(segs[-1], k, seed=41)
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()
    seg_w = [1, 2, 0, 1]
    y = _run(ctx, None, x, tcc.F32, seg=segs, seg_w=seg_w, weights=ws)
    for i, wi in enumerate(seg_w):
        a, b = segs[i], segs[i + 1]
        staging = "f32" if b - a <= 16 else "bf16"
        ref = oracle.qlinear_ref(xb[a:b], raws[wi], types[wi], n, k, staging)
        assert oracle.rel_l2(y[a:b], ref) <= (1e-5 if staging == "f32" else TIGHT), (i, types[wi])


def test_empty_and_zero_segments(ctx):
    import torch
    from turbocider_b200 import cuda as tcc
    raw, w, xb, x = _setup(ctx, 14, 256, 512, 130, wseed=8)
    y = _run(ctx, w, x, tcc.F32, seg=[0, 0, 130, 130])
    assert oracle.rel_l2(y, oracle.qlinear_ref(xb, raw, 14, 256, 512, "bf16")) <= TIGHT
    with pytest.raises(tcc.BackendError, match="non-decreasing"):
        tcc.qlinear(ctx, w, x, seg_offsets=[0, 100, 50])


@pytest.mark.parametrize("typ,n,k", [(12, 10240, 3840), (14, 3840, 10240), (13, 3840, 10240)])
def test_full_size_config5_sampled_rows(ctx, typ, n, k):
    """Config 5 sizes (M = 8448): every output column of 64 sampled rows."""
    from turbocider_b200 import cuda as tcc
    m = 8448
    raw, w, xb, x = _setup(ctx, typ, n, k, m, wseed=31)
    y = _run(ctx, w, x, tcc.F32)
    rows = np.random.default_rng(0).choice(m, 64, replace=False)
    ref = oracle.qlinear_ref(xb[rows], raw, typ, n, k, "bf16")
    assert oracle.rel_l2(y[rows], ref) <= TIGHT


@pytest.mark.parametrize("typ", [12, 13, 14])
@pytest.mark.parametrize("m", [64, 300])
def test_gemm_f16_staging_range_check(ctx, typ, m):
    """fp16 staging flags TC_STATUS_F16_OVERFLOW when a sub-block's values
    can leave the fp16 range (d = 65504), and stays quiet for in-range scales
    and for bf16 staging; m = 64 runs the one-CTA kernel, m = 300 the pair."""
    import torch
    from turbocider_b200 import cuda as tcc
    k = 1024
    x = torch.randn(m, k, device="cuda").to(torch.bfloat16)
    for scale, expect in ((65504.0, True), (0.03125, False)):
        raw = np.frombuffer(kq_cases.extreme_case(typ, scale), dtype=np.uint8)
        raw = np.tile(raw.reshape(2, -1), (128, 1)).reshape(-1)   # 256 rows x 1024
        w = tcc.Weight.upload(ctx, typ, 256, k, raw)
        tcc.qlinear(ctx, w, x, stage=tcc.STAGE_F16, out_dtype=tcc.F32)
        bits = ctx.status()
        assert bool(bits & tcc.STATUS_F16_OVERFLOW) == expect, (scale, bits)
        tcc.qlinear(ctx, w, x, stage=tcc.STAGE_BF16, out_dtype=tcc.F32)
        assert ctx.status() == 0
        w.free()


@pytest.mark.parametrize("typ", [12, 13, 14])
@pytest.mark.parametrize("m,n,k", [(300, 640, 768), (40, 512, 1024), (3, 256, 512), (1024, 1920, 1024)])
def test_gemm_f16_activations_meet_1e3(ctx, typ, m, n, k):
    """TC_STAGE_F16_X16: fp16 X as given, W staged fp16, every segment on the
    tensor-core GEMM (also the 3-row one).  Bound: rel-L2 <= 1e-3 against the
    dequant + fp32 matmul oracle and <= TIGHT against the
    oracle that stages W in fp16 too."""
    import torch
    from turbocider_b200 import cuda as tcc
    raw = tcc.quantize(typ, kq_cases.synthetic_weight(n, k, seed=m + 7))
    w = tcc.Weight.upload(ctx, typ, n, k, raw)
    xh = kq_cases.synthetic_x_f16(m, k, seed=m)
    x = torch.from_numpy(xh.view(np.int16)).view(torch.float16).cuda()
    y = tcc.qlinear(ctx, w, x, out_dtype=tcc.F32, stage=tcc.STAGE_F16_X16).cpu().numpy().astype(np.float64)
    assert ctx.status() == 0
    assert oracle.rel_l2(y, oracle.qlinear_ref(xh, raw, typ, n, k, "f16k", x_dtype="f16")) <= TIGHT
    e = oracle.rel_l2(y, oracle.qlinear_ref(xh, raw, typ, n, k, "f32", x_dtype="f16"))
    print(f"type {typ} m {m}: fp16 activations vs f32 decode {e:.2e}")
    assert e <= 1e-3
    yb = tcc.qlinear(ctx, w, x, out_dtype=tcc.BF16, stage=tcc.STAGE_F16_X16).float().cpu().numpy()
    assert oracle.rel_l2(yb, y) <= 3e-3
    with pytest.raises(tcc.BackendError, match="bf16 X"):
        ctx.set_path(1)
        try:
            tcc.qlinear(ctx, w, x, stage=tcc.STAGE_F16_X16)
        finally:
            ctx.set_path(0)


@pytest.mark.parametrize("m", [1, 4, 16])
def test_batched_gemv_matches_oracle(ctx, m):
    """tc_cuda_qlinear_batched: Q4_K, Q5_K and Q6_K weights of different N
    sharing K and X, one launch per type; each output against the fp32-decode
    oracle."""
    import torch
    from turbocider_b200 import cuda as tcc
    k = 1024
    specs = [(12, 512), (14, 384), (13, 256), (12, 100), (14, 1536), (12, 48), (13, 700)]
    raws, ws = [], []
    for i, (typ, n) in enumerate(specs):
        raw = tcc.quantize(typ, kq_cases.synthetic_weight(n, k, seed=200 + i))
        raws.append(raw)
        ws.append(tcc.Weight.upload(ctx, typ, n, k, raw))
    xb = kq_cases.synthetic_x_bf16(m, k, seed=m)
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()
    outs = tcc.qlinear_batched(ctx, ws, x, out_dtype=tcc.F32)
    assert ctx.status() == 0
    for (typ, n), raw, y in zip(specs, raws, outs):
        got = y.cpu().numpy().astype(np.float64)
        assert oracle.rel_l2(got, oracle.qlinear_ref(xb, raw, typ, n, k, "f32")) <= 1e-5
    with pytest.raises(tcc.BackendError, match="1..16 rows"):
        tcc.qlinear_batched(ctx, ws, torch.zeros(17, k, dtype=torch.bfloat16, device="cuda"))
