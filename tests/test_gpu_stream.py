"""GPU checks of the loader / streaming path: host panel re-layout + panel
copy equals the device re-layout of the upload path bit for bit; weights
streamed per layer through two slots give exactly the results of resident
weights; a GGUF file read into pinned memory and uploaded matches the oracle."""
from __future__ import annotations

import numpy as np
import pytest

import kq_cases
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("typ", [12, 13, 14])
def test_host_relayout_equals_device_relayout(ctx, typ):
    import torch
    from turbocider_b200 import cuda as tcc
    n, k = 300, 768
    raw = tcc.quantize(typ, kq_cases.synthetic_weight(n, k, seed=9))
    a = tcc.Weight.upload(ctx, typ, n, k, raw)
    b = tcc.Weight.create(ctx, typ, n, k)
    panels = torch.from_numpy(tcc.relayout_host(typ, raw, n, k)).pin_memory()
    b.copy_panels(panels)
    da, db = tcc.dequant(ctx, a, tcc.F32), tcc.dequant(ctx, b, tcc.F32)
    torch.cuda.synchronize()
    assert ctx.status() == 0
    assert torch.equal(da, db)
    a.free()
    b.free()


def test_streamed_layers_equal_resident(ctx):
    """Four layers x two linears (Q4_K and Q6_K), streamed through two slots on
    a copy stream while the compute stream runs the GEMMs."""
    import torch
    from turbocider_b200 import cuda as tcc
    from turbocider_b200.stream import LayerStream
    m, k = 520, 768
    shapes = {"a": (12, 384, k), "b": (14, 256, k)}
    layers = []
    for layer in range(4):
        spec = {}
        for j, (name, (typ, n, kk)) in enumerate(shapes.items()):
            spec[name] = (typ, n, kk, tcc.quantize(typ, kq_cases.synthetic_weight(n, kk, seed=10 * layer + j)))
        layers.append(spec)
    x = torch.randn(m, k, device="cuda").to(torch.bfloat16)
    resident = [{nm: tcc.Weight.upload(ctx, t, n, kk, raw) for nm, (t, n, kk, raw) in spec.items()} for spec in layers]
    want = [{nm: tcc.qlinear(ctx, w, x, out_dtype=tcc.F32) for nm, w in lw.items()} for lw in resident]
    compute = torch.cuda.Stream()
    st = LayerStream(ctx, layers, torch.device("cuda", 0))
    for _ in range(2):   # two passes reuse the slots
        got = []
        with torch.cuda.stream(compute):
            st.begin(compute)
            for layer in range(4):
                w = st.acquire(layer, compute)
                got.append({nm: tcc.qlinear(ctx, w[nm], x, out_dtype=tcc.F32, stream=compute) for nm in shapes})
                st.release(layer, compute)
        compute.synchronize()
        assert ctx.status() == 0
        for layer in range(4):
            for nm in shapes:
                assert torch.equal(got[layer][nm], want[layer][nm]), (layer, nm)
    st.close()


def test_gguf_file_to_hbm(ctx, tmp_path):
    """gguf-py writes a container; tc_gguf_read fills pinned memory; the
    upload path brings it to HBM; the GEMM matches the oracle."""
    gguf = pytest.importorskip("gguf")
    import torch
    from turbocider_b200 import cuda as tcc
    path = tmp_path / "w.gguf"
    wr = gguf.GGUFWriter(str(path), "test")
    n, k, m = 640, 1024, 300
    raw = tcc.quantize(12, kq_cases.synthetic_weight(n, k, seed=77))
    wr.add_tensor("blk.0.attn_qkv.weight", raw.reshape(n, -1), raw_dtype=gguf.GGMLQuantizationType(12))
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()
    f = tcc.GGUFFile(path)
    info = f.tensor("blk.0.attn_qkv.weight")
    pinned = torch.empty(info["bytes"], dtype=torch.uint8, pin_memory=True)
    f.read("blk.0.attn_qkv.weight", out=pinned)
    w = tcc.Weight.upload(ctx, info["type"], info["rows"], info["columns"], pinned.numpy())
    xb = kq_cases.synthetic_x_bf16(m, k, seed=5)
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()
    y = tcc.qlinear(ctx, w, x, out_dtype=tcc.F32).cpu().numpy().astype(np.float64)
    assert ctx.status() == 0
    assert oracle.rel_l2(y, oracle.qlinear_ref(xb, raw, 12, n, k, "bf16")) <= 1e-4
    f.close()
