"""GPU test of the allocation-free entry point tc_cuda_qlinear_small_static.

It serves callers that cannot allocate device memory while running a linear
(pre-sized memory arenas, allocator callbacks, loops that cannot absorb
cudaMalloc's synchronisation): the split-K GEMV runs with its scratch in a
fixed static device array.  Its output must match the fp32-decode oracle
(decode_cpu_into(f32) + an fp64 matmul) and the existing entry point
(tc_cuda_qlinear, same kernel with a cudaMalloc'd workspace) within the GEMV
tolerance used elsewhere (rel-L2 <= 1e-5), on two calls in a row -- the second
call sees the array as the first one left it -- and its status word, read with
tc_cuda_small_static_status, must stay clear.  This file is collected last.
"""
from __future__ import annotations

import numpy as np
import pytest

import kq_cases
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("typ,n,k,m", [(14, 3072, 12288, 4), (12, 1000, 4096, 1), (14, 512, 2048, 16),
                                       (12, 2048, 3072, 2)])
def test_static_scratch_matches_qlinear_twice(ctx, typ, n, k, m):
    import torch
    from turbocider_b200 import cuda as tcc
    raw = tcc.quantize(typ, kq_cases.synthetic_weight(n, k, seed=n + m))
    w = tcc.Weight.upload(ctx, typ, n, k, raw)
    xb = kq_cases.synthetic_x_bf16(m, k, seed=m + 3)
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()
    ref = tcc.qlinear(ctx, w, x, out_dtype=tcc.F32).cpu().numpy()
    want = oracle.qlinear_ref(xb, raw, typ, n, k, "f32")
    assert oracle.rel_l2(ref, want) <= 1e-5
    for _ in range(2):
        y = torch.full((m, n), float("nan"), device="cuda", dtype=torch.float32)
        tcc.qlinear_small_static(w, x, out_dtype=tcc.F32, out=y)
        torch.cuda.synchronize()
        got = y.cpu().numpy()
        assert np.isfinite(got).all()
        assert oracle.rel_l2(got, want) <= 1e-5
        assert oracle.rel_l2(got, ref) <= 1e-5
        assert tcc.small_static_status(0) == 0
    yb = tcc.qlinear_small_static(w, x, out_dtype=tcc.BF16)
    assert oracle.rel_l2(yb.float().cpu().numpy(), want) <= 3e-3
    assert tcc.small_static_status(0) == 0
    assert ctx.status() == 0


def test_static_scratch_covers_large_shapes_and_rejects_bad_rows(ctx):
    """The GEMV's scratch is at most 4.6 MiB of partials (K slices x row
    tiles < 1184, 4 KiB each) plus one counter per 16 weight rows, inside the 8
    MiB array, whose size check remains as a guard.  Large weights (22016
    and 37824 rows, with and without a K split) run and match the context
    path and the oracle; row counts outside 1..16 are rejected."""
    import torch
    from turbocider_b200 import cuda as tcc
    n, k = 22016, 8448
    raw = tcc.quantize(12, kq_cases.synthetic_weight(n, k, seed=5))
    w = tcc.Weight.upload(ctx, 12, n, k, raw)
    x = torch.randn(1, k, device="cuda").to(torch.bfloat16)
    ref = tcc.qlinear(ctx, w, x, out_dtype=tcc.F32).cpu().numpy()
    got = tcc.qlinear_small_static(w, x, out_dtype=tcc.F32).cpu().numpy()
    assert oracle.rel_l2(got, ref) <= 1e-5
    xb = x.view(torch.int16).cpu().numpy().view(np.uint16)
    rows = np.arange(0, n, 7)   # every 7th output column against the fp32-decode oracle
    sub = raw.reshape(n, -1)[rows]
    assert oracle.rel_l2(got[:, rows], oracle.qlinear_ref(xb, sub, 12, len(rows), k, "f32")) <= 1e-5
    for n2, k2 in ((3072, 12288), (128, 256), (9000, 1024), (591 * 64, 1024)):
        w2 = tcc.Weight.upload(ctx, 14, n2, k2, tcc.quantize(14, kq_cases.synthetic_weight(n2, k2, seed=n2)))
        x2 = torch.randn(16, k2, device="cuda").to(torch.bfloat16)
        ref2 = tcc.qlinear(ctx, w2, x2, out_dtype=tcc.F32).cpu().numpy()
        assert oracle.rel_l2(tcc.qlinear_small_static(w2, x2, out_dtype=tcc.F32).cpu().numpy(), ref2) <= 1e-5
        w2.free()
    x17 = torch.zeros(17, k, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(tcc.BackendError, match="1..16 rows"):
        tcc.qlinear_small_static(w, x17)
    assert tcc.small_static_status(0) == 0
