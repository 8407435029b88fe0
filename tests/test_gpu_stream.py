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


def _gguf_file(tmp_path, typ, n, k, seed):
    gguf = pytest.importorskip("gguf")
    from turbocider_b200 import cuda as tcc
    raw = tcc.quantize(typ, kq_cases.synthetic_weight(n, k, seed=seed))
    path = tmp_path / f"w{typ}.gguf"
    wr = gguf.GGUFWriter(str(path), "test")
    wr.add_tensor("w", raw.reshape(n, -1), raw_dtype=gguf.GGMLQuantizationType(typ))
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()
    return raw, tcc.GGUFFile(path)


@pytest.mark.parametrize("typ", [12, 13, 14])
def test_streaming_loader_equals_upload(ctx, tmp_path, typ):
    """tc_cuda_weight_load_gguf (read-ahead: pread of chunk i + 1 beside the
    copy and device re-layout of chunk i) gives the same panels as the
    synchronous upload, for the whole tensor and for a row shard, with
    chunks of 128 rows (many chunks, ragged last one)."""
    import torch
    from turbocider_b200 import cuda as tcc
    n, k = 1000, 2048
    raw, f = _gguf_file(tmp_path, typ, n, k, seed=typ + 40)
    for n_begin, n_count in ((0, 0), (256, 500)):
        w, stats = tcc.Weight.load_gguf(ctx, f, "w", n_begin, n_count, chunk_bytes=1)
        rows = n_count or n
        ref = tcc.Weight.upload(ctx, typ, n, k, raw, n_begin=n_begin, n_count=n_count)
        a = tcc.dequant(ctx, w, tcc.F32)
        b = tcc.dequant(ctx, ref, tcc.F32)
        assert torch.equal(a, b)
        want = oracle.decode_checked(raw.reshape(n, -1)[n_begin:n_begin + rows], typ, rows, k, oracle.F32)
        assert np.array_equal(a.cpu().numpy(), want)
        assert stats["bytes"] == rows * (k // 256) * {12: 144, 13: 176, 14: 210}[typ]
        assert stats["chunks"] == -(-rows // 128)
        w.free()
        ref.free()
    assert ctx.status() == 0
    f.close()


def test_streaming_loader_cancel_and_errors(ctx, tmp_path):
    """A set cancel flag returns Cancelled and publishes nothing; a row range
    past the tensor is rejected; the context stays usable."""
    from turbocider_b200 import cuda as tcc
    raw, f = _gguf_file(tmp_path, 12, 512, 1024, seed=3)
    flag = tcc.CancelFlag()
    flag.set()
    with pytest.raises(tcc.Cancelled):
        tcc.Weight.load_gguf(ctx, f, "w", cancel=flag)
    with pytest.raises(tcc.DecodeError, match="out of bounds"):
        tcc.Weight.load_gguf(ctx, f, "w", 500, 20)
    flag.clear()
    w, _ = tcc.Weight.load_gguf(ctx, f, "w", cancel=flag)
    assert np.array_equal(tcc.dequant(ctx, w, tcc.F32).cpu().numpy(),
                          oracle.decode_checked(raw, 12, 512, 1024, oracle.F32))
    w.free()
    assert ctx.status() == 0
    f.close()


def test_layer_stream_cancel(ctx):
    """LayerStream raises Cancelled at the next prefetch / acquire once its
    flag is set; the layers already acquired stay valid."""
    import torch
    from turbocider_b200 import cuda as tcc
    from turbocider_b200.stream import LayerStream
    n, k = 256, 512
    raw = tcc.quantize(12, kq_cases.synthetic_weight(n, k, seed=8))
    flag = tcc.CancelFlag()
    st = LayerStream(ctx, [{"w": (12, n, k, raw)} for _ in range(4)], "cuda:0", cancel=flag)
    compute = torch.cuda.Stream()
    st.begin(compute)
    w0 = st.acquire(0, compute)["w"]
    flag.set()
    with pytest.raises(tcc.Cancelled):
        st.acquire(1, compute)
    with pytest.raises(tcc.Cancelled):
        st.release(0, compute)    # would prefetch layer 2
    compute.synchronize()
    assert np.array_equal(tcc.dequant(ctx, w0, tcc.F32).cpu().numpy(),
                          oracle.decode_checked(raw, 12, n, k, oracle.F32))
    st.close()
    with pytest.raises(tcc.Cancelled):
        LayerStream(ctx, [{"w": (12, n, k, raw)}], "cuda:0", cancel=flag)
