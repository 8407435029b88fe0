"""Guard-byte canaries around the outputs of every linear kernel, in the
style of the reference's decoder tests (tests/native/test_gguf_execution.py:
100-128: a 0xA5-filled target, every byte outside the written elements must
survive).  Y is placed inside a larger 0xA5 buffer with a row pitch past N
and guard regions before the first and after the last row; after the call
every byte outside [m][0, N) must still be 0xA5.  Covers the warp GEMV, the
one-CTA and 2-CTA tensor-core GEMMs (direct stores, TMA stores, split-K
partials and reduce), the dense GEMM, with and without a fused epilogue, for
f32 / f16 / bf16 outputs and an odd row pitch (direct stores) as well as a
16-byte one (TMA stores)."""
from __future__ import annotations

import numpy as np
import pytest

import kq_cases
from oracle import oracle

pytestmark = pytest.mark.gpu

GUARD = 0xA5
CASES = [  # (label, weight type, n, k, m, forced path)
    ("gemv", 12, 200, 512, 5, 0),
    ("one_cta", 14, 200, 512, 100, 3),
    ("pair", 12, 3072, 512, 800, 0),           # 2-CTA, 48 tiles: no split
    ("pair_split", 13, 256, 2048, 300, 0),     # 2-CTA with split-K
    ("dense", 8, 200, 256, 150, 0),
]


def _weight(ctx, typ, n, k):
    from turbocider_b200 import cuda as tcc
    if typ in (12, 13, 14):
        raw = tcc.quantize(typ, kq_cases.synthetic_weight(n, k, seed=n + typ))
    else:
        import random
        rng = random.Random(n)
        raw = np.frombuffer(b"".join(kq_cases.random_block(typ, rng) for _ in range(n * k // 32)), np.uint8)
    return raw, tcc.Weight.upload(ctx, typ, n, k, raw)


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
@pytest.mark.parametrize("out_dtype", [0, 1, 2])
@pytest.mark.parametrize("pad", [13, 16])
@pytest.mark.parametrize("epi", [False, True])
def test_outputs_touch_nothing_else(ctx, case, out_dtype, pad, epi):
    import torch
    from turbocider_b200 import cuda as tcc
    label, typ, n, k, m, path = case
    raw, w = _weight(ctx, typ, n, k)
    xb = kq_cases.synthetic_x_bf16(m, k, seed=m)
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()
    item = 4 if out_dtype == 0 else 2
    ldy = n + pad
    lead = 64                                  # guard elements before row 0
    total = lead + m * ldy + 64                # and after the last row
    tdt = {0: torch.float32, 1: torch.float16, 2: torch.bfloat16}[out_dtype]
    buf = torch.full((total * item,), GUARD, dtype=torch.uint8, device="cuda")
    y = buf.view(tdt)[lead:lead + m * ldy].view(m, ldy)[:, :n]
    kw = {}
    if epi:
        kw = dict(bias=torch.randn(n, device="cuda"), activation="gelu_tanh")
    ctx.set_path(path)
    try:
        tcc.qlinear(ctx, w, x, out=y, out_dtype=out_dtype, **kw)
    finally:
        ctx.set_path(0)
    assert ctx.status() == 0
    host = buf.cpu().numpy()
    written = np.zeros(total * item, dtype=bool)
    for r in range(m):
        a = (lead + r * ldy) * item
        written[a:a + n * item] = True
    assert np.all(host[~written] == GUARD), f"{label}: bytes outside Y written"
    got = y.float().cpu().numpy().astype(np.float64)
    staging = "f32" if label == "gemv" else "bf16"
    ref = oracle.qlinear_ref(xb, raw, typ, n, k, staging)
    if epi:
        ref = oracle.epilogue_ref(ref, bias=kw["bias"].cpu().numpy(), activation="gelu_tanh")
    assert oracle.rel_l2(got, ref) <= {0: 1e-4, 1: 1e-3, 2: 3e-3}[out_dtype]
    w.free()
