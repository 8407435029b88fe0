"""GPU parity of the dequantisers through the C ABI: bit-exact against the
reference decoder (golden digests) and the oracle port.

* tc_cuda_decode (raw GGUF layout, strided slices, every registered type)
  reproduces every golden case, including the reference's errors (nonfinite
  input or scale, fp16 / bf16 overflow);
* tc_cuda_weight_upload + tc_cuda_dequant (panel layout) is bit-exact for
  every dtype, N not a multiple of the 128-row panel, and sharded uploads.
"""
from __future__ import annotations

import hashlib

import numpy as np
import pytest

import kq_cases
from oracle import oracle

pytestmark = pytest.mark.gpu

GUARD = 0xA5


def _dev(raw: bytes):
    import torch
    return torch.frombuffer(bytearray(raw), dtype=torch.uint8).cuda()


def _gpu_decode(ctx, raw, typ, rows, cols, dtype, col_begin=0, ncols=None, column_stride=None):
    """Decode on the GPU into a guarded strided target; returns the digest (or
    'error: msg') of the values packed contiguously, and checks the guards."""
    import torch
    from turbocider_b200 import cuda as tcc
    ncols = cols - col_begin if ncols is None else ncols
    item = 4 if dtype == 0 else 2
    cs = column_stride or item
    rs = (ncols - 1) * cs + item + 8
    size = (rows - 1) * rs + (ncols - 1) * cs + item + 16
    target = torch.full((size,), GUARD, dtype=torch.uint8, device="cuda")
    try:
        tcc.decode(ctx, typ, _dev(raw), rows, cols, 0, rows, col_begin, ncols, dtype, target, rs, cs)
    except tcc.DecodeError as e:
        return "error: " + str(e)
    host = target.cpu().numpy()
    touched = np.zeros(size, dtype=bool)
    vals = bytearray()
    for r in range(rows):
        for c in range(ncols):
            o = r * rs + c * cs
            touched[o:o + item] = True
            vals += host[o:o + item].tobytes()
    assert np.all(host[~touched] == GUARD), "guard bytes overwritten"
    return hashlib.sha256(bytes(vals)).hexdigest()


def test_decode_seed6409_bit_exact(ctx, golden):
    g = golden["cases"]["seed6409"]
    for typ, trial, raw, rows, cols in kq_cases.seed6409_cases():
        for dt in (0, 1, 2):
            assert _gpu_decode(ctx, raw, typ, rows, cols, dt) == g[str(typ)][trial][dt], (typ, trial, dt)
    assert ctx.status() == 0


def test_decode_slices_and_strides_bit_exact(ctx, golden):
    g = golden["cases"]["seed20260930"]
    for typ, raw, rows, cols, slices in kq_cases.seed20260930_cases():
        for i, (b, n) in enumerate(slices):
            for dt in (0, 1, 2):
                got = _gpu_decode(ctx, raw, typ, rows, cols, dt, col_begin=b, ncols=n, column_stride=8)
                assert got == g[str(typ)][i][dt], (typ, b, n, dt)


def test_decode_unaligned_strides(ctx, golden):
    """Odd column strides (targets not aligned to the item size) for every
    registered type: byte-wise stores, same values as the golden digests."""
    g = golden["cases"]["seed20260930"]
    for typ, raw, rows, cols, slices in kq_cases.seed20260930_cases():
        for i, (b, n) in enumerate(slices):
            for dt in (0, 1, 2):
                item = 4 if dt == 0 else 2
                got = _gpu_decode(ctx, raw, typ, rows, cols, dt, col_begin=b, ncols=n, column_stride=item + 1)
                assert got == g[str(typ)][i][dt], (typ, b, n, dt)


def test_decode_passthrough_types(ctx, golden):
    """F32 / F16 / BF16 and Q4_0 / Q4_1 / Q5_0 / Q5_1 / Q8_0 value rules:
    nonfinite inputs and scales, fp16 / bf16 overflow, subnormals."""
    g = golden["cases"]["passthrough"]
    for name, typ, raw, rows, cols in kq_cases.passthrough_cases():
        for dt in (0, 1, 2):
            assert _gpu_decode(ctx, raw, typ, rows, cols, dt) == g[name][dt], (name, dt)
    assert ctx.status() == 0


def test_decode_pattern_extreme_nonfinite(ctx, golden):
    c = golden["cases"]
    for typ in kq_cases.K_TYPES:
        for rows in (1, 3, 17):
            for cols in (256, 512, 1024):
                raw = kq_cases.pattern_case(typ, rows, cols)
                for dt in (0, 1, 2):
                    assert _gpu_decode(ctx, raw, typ, rows, cols, dt) == c["pattern"][f"{typ}/{rows}x{cols}"][dt]
        for scale in kq_cases.EXTREME_SCALES:
            raw = kq_cases.extreme_case(typ, scale)
            for dt in (0, 1, 2):
                assert _gpu_decode(ctx, raw, typ, 2, 1024, dt) == c["extreme"][f"{typ}/{scale!r}"][dt], (typ, scale, dt)
    for key, expect in c["nonfinite"].items():
        typ, where, bits = key.split("/")
        typ, bits = int(typ), int(bits, 16)
        raw = bytearray(kq_cases.extreme_case(typ, 1.0))
        off = 208 if typ == 14 else (0 if where == "d" else 2)
        raw[off:off + 2] = bits.to_bytes(2, "little")
        for dt in (0, 1, 2):
            assert _gpu_decode(ctx, bytes(raw), typ, 2, 1024, dt) == expect[dt]


def test_decode_geometry_errors(ctx):
    import torch
    from turbocider_b200 import cuda as tcc
    raw = _dev(kq_cases.pattern_case(12, 2, 512))
    tgt = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    cases = [
        (dict(rows=3), "row slice out of bounds"),
        (dict(cols=300), "invalid source geometry"),
        (dict(column_begin=500, columns=20), "invalid decode slice"),
        (dict(column_stride=1), "invalid/overlapping column stride"),
        (dict(row_stride=8), "invalid/overlapping row stride"),
        (dict(dtype=7), "gguf_decode: invalid target dtype"),
    ]
    for over, msg in cases:
        a = dict(rows=2, cols=512, column_begin=0, columns=4, dtype=0, row_stride=64, column_stride=4)
        a.update(over)
        with pytest.raises(tcc.DecodeError, match=msg):
            tcc.decode(ctx, 12, raw, 2, a["cols"], 0, a["rows"], a["column_begin"], a["columns"], a["dtype"], tgt,
                       a["row_stride"], a["column_stride"])
    with pytest.raises(tcc.DecodeError, match="decode target too short"):
        tcc.decode(ctx, 12, raw, 2, 512, 0, 2, 0, 512, 0, tgt[:100], 2048, 4)


@pytest.mark.parametrize("typ", [12, 13, 14])
@pytest.mark.parametrize("n,k", [(200, 512), (128, 256), (384, 3072)])
def test_panel_dequant_bit_exact(ctx, typ, n, k):
    from turbocider_b200 import cuda as tcc
    w = kq_cases.synthetic_weight(n, k, seed=n + k + typ)
    raw = tcc.quantize(typ, w)
    weight = tcc.Weight.upload(ctx, typ, n, k, raw)
    assert (weight.n, weight.k) == (n, k)
    for dt in (0, 1, 2):
        got = tcc.dequant(ctx, weight, dt).cpu()
        ref = oracle.decode_checked(raw, typ, n, k, dt)
        got_np = got.view(__import__("torch").int16).numpy().view(np.uint16) if dt else got.numpy()
        assert np.array_equal(np.ascontiguousarray(got_np).view(np.uint8), np.ascontiguousarray(ref).view(np.uint8)), dt
    assert ctx.status() == 0


def test_panel_dequant_shard(ctx):
    from turbocider_b200 import cuda as tcc
    n, k = 512, 1024
    raw = tcc.quantize(14, kq_cases.synthetic_weight(n, k, seed=3))
    full = oracle.decode_checked(raw, 14, n, k, 0)
    for begin, count in [(0, 128), (128, 256), (300, 212)]:
        shard = tcc.Weight.upload(ctx, 14, n, k, raw, n_begin=begin, n_count=count)
        assert shard.n == count
        got = tcc.dequant(ctx, shard, 0).cpu().numpy()
        assert np.array_equal(got.view(np.uint32), full[begin:begin + count].view(np.uint32))


def test_upload_rejects_nonfinite_scale(ctx):
    from turbocider_b200 import cuda as tcc
    for typ in (12, 13, 14):
        raw = bytearray(tcc.quantize(typ, kq_cases.synthetic_weight(4, 512, seed=9)))
        off = 208 if typ == 14 else 2
        raw[off + tcc.BLOCK_BYTES[typ] * 5:off + tcc.BLOCK_BYTES[typ] * 5 + 2] = (0x7C00).to_bytes(2, "little")
        with pytest.raises(tcc.DecodeError, match="nonfinite"):
            tcc.Weight.upload(ctx, typ, 4, 512, bytes(raw))


def test_panel_dequant_f16_overflow_sets_status(ctx):
    from turbocider_b200 import cuda as tcc
    raw = kq_cases.extreme_case(12, 65504.0)
    w = tcc.Weight.upload(ctx, 12, 2, 1024, raw)
    tcc.dequant(ctx, w, 1)
    assert ctx.status() & tcc.STATUS_F16_OVERFLOW
    tcc.dequant(ctx, w, 2)
    assert ctx.status() == 0


def _gpu_gather(ctx, raw, typ, rows, cols, idx, dtype, col_begin=0, ncols=None):
    """Device gather into a guarded target with an odd row pitch; returns the
    values (uint8 bytes of each target row) or 'error: msg'."""
    import torch
    from turbocider_b200 import cuda as tcc
    ncols = cols - col_begin if ncols is None else ncols
    item = 4 if dtype == 0 else 2
    rs = ncols * item + 6
    size = (len(idx) - 1) * rs + ncols * item + 16
    target = torch.full((size,), GUARD, dtype=torch.uint8, device="cuda")
    ind = torch.tensor(np.asarray(idx, dtype=np.int64), device="cuda")
    try:
        tcc.decode_gather(ctx, typ, _dev(raw), rows, cols, ind, col_begin, ncols, dtype, target, rs, item)
    except tcc.DecodeError as e:
        return "error: " + str(e)
    host = target.cpu().numpy()
    out = np.stack([host[r * rs:r * rs + ncols * item] for r in range(len(idx))])
    touched = np.zeros(size, dtype=bool)
    for r in range(len(idx)):
        touched[r * rs:r * rs + ncols * item] = True
    assert np.all(host[~touched] == GUARD), "guard bytes overwritten"
    return out


def test_decode_gather_bit_exact(ctx):
    """tc_cuda_decode_gather against the reference's own decode_cpu_gather
    (its probe's gather mode; the C port where the reference was not built)
    on the seed-20260930 blocks of every registered type: duplicated and
    reordered rows, a column slice, all three target dtypes."""
    which = "ref" if oracle.ref() is not None else "port"
    for typ, raw, rows, cols, slices in kq_cases.seed20260930_cases():
        for idx in ([2, 0, 2, 1], [1], [0, 0, 0]):
            for cb, nc in slices[:2]:
                for dt in (0, 1, 2):
                    rc, want, err = oracle.decode_gather(raw, typ, rows, cols, idx, dt, which, col_begin=cb, ncols=nc)
                    got = _gpu_gather(ctx, raw, typ, rows, cols, idx, dt, cb, nc)
                    if rc:
                        assert got == "error: " + err, (typ, idx, dt, got, err)
                    else:
                        assert not isinstance(got, str), (typ, idx, dt, got)
                        assert np.array_equal(got.view(np.uint8).reshape(len(idx), -1),
                                              want.view(np.uint8).reshape(len(idx), -1)), (typ, idx, dt)


def test_decode_gather_errors(ctx):
    """The reference's gather rejections: an index past the matrix, indices
    overlapping the target, an empty index list (validate's slice check)."""
    import torch
    from turbocider_b200 import cuda as tcc
    raw = kq_cases.pattern_case(12, 4, 512)
    assert _gpu_gather(ctx, raw, 12, 4, 512, [1, 4], 0) == "error: gather row out of bounds"
    assert oracle.decode_gather(raw, 12, 4, 512, [1, 4], 0, "port")[2] == "gather row out of bounds"
    buf = torch.zeros(4096, dtype=torch.int64, device="cuda")
    with pytest.raises(tcc.DecodeError, match="gather indices overlap target"):
        tcc.decode_gather(ctx, 12, _dev(raw), 4, 512, buf[:2], 0, 8, 0, buf, 64, 4)
    with pytest.raises(tcc.DecodeError, match="invalid decode slice"):
        tcc.decode_gather(ctx, 12, _dev(raw), 4, 512, buf[:0], 0, 8, 0, buf[64:], 64, 4)
    assert ctx.status() == 0
