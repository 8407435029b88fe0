"""One process driving two GPUs: a context on each device, and every kernel
family (2-CTA tensor-core GEMM, one-CTA GEMM, warp GEMV, static-scratch GEMV)
run on both, alternating.  The kernels' shared-memory opt-in and occupancy
are per-device launch settings, so each device must get its own; outputs are
checked against the oracle.  Skips with fewer than two GPUs."""
from __future__ import annotations

import numpy as np
import pytest

import kq_cases
from oracle import oracle

pytestmark = pytest.mark.gpu


def test_contexts_on_two_devices_in_one_process():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from turbocider_b200 import cuda as tcc
    n, k = 512, 1024
    raw = {typ: tcc.quantize(typ, kq_cases.synthetic_weight(n, k, seed=typ)) for typ in (12, 14)}
    ctxs = [tcc.Context(d) for d in (0, 1)]
    ws = {(d, typ): tcc.Weight.upload(ctxs[d], typ, n, k, raw[typ]) for d in (0, 1) for typ in (12, 14)}
    try:
        for rep in range(2):
            for d in (1, 0):            # device 1 first: its launches must not rely on device 0's set-up
                with torch.cuda.device(d):
                    for typ in (12, 14):
                        for m, path in ((300, 0), (96, 3), (4, 0)):
                            xb = kq_cases.synthetic_x_bf16(m, k, seed=m + d)
                            x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).to(f"cuda:{d}")
                            ctxs[d].set_path(path)
                            y = tcc.qlinear(ctxs[d], ws[(d, typ)], x, out_dtype=tcc.F32)
                            ctxs[d].set_path(0)
                            staging = "f32" if m <= 16 else "bf16"
                            err = oracle.rel_l2(y.cpu().numpy(), oracle.qlinear_ref(xb, raw[typ], typ, n, k, staging))
                            assert err <= (1e-5 if m <= 16 else 1e-4), (rep, d, typ, m, err)
                        xb = kq_cases.synthetic_x_bf16(2, k, seed=d)
                        x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).to(f"cuda:{d}")
                        y = tcc.qlinear_small_static(ws[(d, typ)], x, out_dtype=tcc.F32)
                        assert oracle.rel_l2(y.cpu().numpy(),
                                             oracle.qlinear_ref(xb, raw[typ], typ, n, k, "f32")) <= 1e-5
                    assert tcc.small_static_status(d) == 0
        for c in ctxs:
            assert c.status() == 0
    finally:
        for w in ws.values():
            w.free()
        for c in ctxs:
            c.close()
