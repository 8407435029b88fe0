"""GGUF directory reader (tc_gguf_*) against the reference parser.

Fixtures are GGUF byte strings built here in the layout the reference's own
directory tests use (tests/native/test_gguf_execution.py:26-51 and
tests/native/test_native_gguf.py:11-25); the cases restate those tests' valid
and invalid files (bounds, alignment, duplicates, overlap, block alignment,
metadata arrays, parse limits, header truncation, split sets).  Each file
goes through our reader and, where the reference sources were built
(oracle/_ref/gguf_probe, the reference's probe executable over
read_directory), through the reference: accept/reject and, when accepted,
tensor count, data offset and every tensor's type / rows / columns / file
offset / bytes must agree; rejection messages must name the same reason.
Without the probe (on a GPU box) the accepted files are checked against the
values the fixture builder implies.  gguf-py (an independent writer/reader)
provides real K-quant containers for the payload-read checks.
"""
from __future__ import annotations

import math
import struct
import subprocess
from pathlib import Path

import numpy as np
import pytest

from turbocider_b200 import cuda as tcc

PROBE = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "gguf_probe"
TYPES = {0: (1, 4), 1: (1, 2), 2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 8: (32, 34),
         12: (256, 144), 13: (256, 176), 14: (256, 210), 30: (1, 2)}


def text(value: str) -> bytes:
    raw = value.encode()
    return struct.pack("<Q", len(raw)) + raw


def metadata(key, typ, value) -> bytes:
    fmt = {0: "B", 1: "b", 2: "H", 3: "h", 4: "I", 5: "i", 6: "f", 7: "B", 10: "Q", 11: "q", 12: "d"}
    return text(key) + struct.pack("<I", typ) + (text(value) if typ == 8 else struct.pack("<" + fmt[typ], value))


def fixture(entries, meta=(), alignment=32, payload=None) -> bytes:
    """entries: (name, ggml type, disk dims[, relative offset]); tensors are laid
    out back to back at `alignment` unless an offset is given."""
    head = struct.pack("<IIQQ", 0x46554747, 3, len(entries), len(meta)) + b"".join(meta)
    offset = end = 0
    for e in entries:
        name, typ, dims = e[:3]
        pos = e[3] if len(e) == 4 else offset
        elems, block = TYPES.get(typ, (1, 1))
        size = math.prod(dims) // elems * block
        head += text(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        head += struct.pack("<IQ", typ, pos)
        offset = (pos + size + alignment - 1) // alignment * alignment
        end = max(end, pos + size)
    body = bytes(min(end, 1 << 20)) if payload is None else payload
    return head + bytes((-len(head)) % alignment) + body


def ours(path, limit=None):
    try:
        f = tcc.GGUFFile(path, limit)
    except tcc.GGUFError as e:
        return False, str(e), None
    out = (len(f.tensors), f.data_offset,
           [(t["name"], t["type"], t["rows"], t["columns"], t["file_offset"], t["bytes"]) for t in f.tensors])
    f.close()
    return True, "", out


def reference(path, names, limit=None):
    if not PROBE.exists():
        return None
    mode = ["limit", str(path), limit] if limit else ["inspect", str(path)]
    r = subprocess.run([str(PROBE), *mode], capture_output=True, text=True, timeout=20)
    if r.returncode:
        return False, r.stderr.strip(), None
    count, data_offset, _ = r.stdout.split()[1:4]
    tensors = []
    for name in names:
        t = subprocess.run([str(PROBE), "tensor", str(path), name], capture_output=True, text=True, timeout=20)
        typ, rows, cols, off, nb = (int(v) for v in t.stdout.splitlines()[1].split()[1:6])
        tensors.append((name, typ, rows, cols, off, nb))
    return True, "", (int(count), int(data_offset), tensors)


def agree(tmp_path, data, names=(), limit=None, expect_ok=None):
    path = tmp_path / "f.gguf"
    path.write_bytes(data)
    got = ours(path, limit)
    ref = reference(path, list(names), limit)
    if ref is not None:
        assert got[0] == ref[0], (got, ref)
        if got[0]:
            assert got[2] == ref[2]
        else:
            # same reason text (the reference prints what() of its exception)
            assert got[1] == ref[1], (got[1], ref[1])
    if expect_ok is not None:
        assert got[0] == expect_ok, got
    return got


@pytest.mark.parametrize("typ", sorted(TYPES))
def test_every_registered_type(tmp_path, typ):
    elems = TYPES[typ][0]
    ok, _, info = agree(tmp_path, fixture([("w", typ, [max(elems, 32), 3])]), ["w"], expect_ok=True)
    count, data_offset, tensors = info
    assert count == 1 and tensors[0][1:4] == (typ, 3, max(elems, 32))
    assert tensors[0][5] == 3 * max(elems, 32) // elems * TYPES[typ][1]


INVALID = {
    "truncated payload": fixture([("w", 8, [32, 2])])[:-1],
    "unaligned offset": fixture([("w", 8, [32], 1)]),
    "duplicate tensor": fixture([("w", 8, [32]), ("w", 8, [32])]),
    "overlap": fixture([("a", 8, [32], 0), ("b", 8, [32], 0)]),
    "row not block aligned": fixture([("w", 8, [31])]),
    "k-quant row not block aligned": fixture([("w", 12, [32])]),
    "zero dimension": fixture([("w", 0, [0])]),
    "huge dimension": fixture([("w", 0, [2 ** 32])])[:256],
    "alignment not power of two": fixture([("w", 8, [32])], [metadata("general.alignment", 4, 3)]),
    "duplicate metadata key": fixture([("w", 8, [32])], [metadata("k", 4, 1), metadata("k", 4, 2)]),
    "bad boolean 2": fixture([("w", 8, [32])], [metadata("bool", 7, 2)]),
    "bad boolean 255": fixture([("w", 8, [32])], [metadata("bool", 7, 255)]),
    "bad boolean in array": fixture([("w", 8, [32])], [text("b") + struct.pack("<IIQB", 9, 7, 1, 2)]),
    "unsupported ggml type": fixture([("w", 15, [32])]),
    "empty": b"",
    "not gguf": b"nope",
    "version 4": struct.pack("<IIQQ", 0x46554747, 4, 1, 0),
    "tensor count overflow": struct.pack("<IIQQ", 0x46554747, 3, 2 ** 64 - 1, 0),
    "metadata count overflow": struct.pack("<IIQQQ", 0x46554747, 3, 1, 0, 2 ** 64 - 1),
}


@pytest.mark.parametrize("case", sorted(INVALID))
def test_invalid_files_rejected_like_the_reference(tmp_path, case):
    agree(tmp_path, INVALID[case], expect_ok=False)


def test_header_truncations(tmp_path):
    valid = fixture([("w", 8, [32])])
    for cut in (23, 35, len(valid) - 1):
        agree(tmp_path, valid[:cut], expect_ok=False)


def test_metadata_arrays_nesting_and_limits(tmp_path):
    array = text("array") + struct.pack("<IIQ", 9, 8, 2) + text("a") + text("b")
    nested = text("nested") + struct.pack("<IIQ", 9, 9, 1) + struct.pack("<IQ", 4, 2) + struct.pack("<II", 1, 2)
    meta = [array, nested, metadata("general.name", 8, "test"), metadata("signed", 5, -7),
            metadata("float", 6, 1.5), metadata("double", 12, -2.25), metadata("general.alignment", 4, 64)]
    data = fixture([("weight0", 8, [32]), ("weight1", 0, [1])], meta, alignment=64)
    agree(tmp_path, data, ["weight0", "weight1"], expect_ok=True)
    path = tmp_path / "f.gguf"
    f = tcc.GGUFFile(path)
    assert f.alignment == 64 and f.data_offset % 64 == 0
    assert f.meta("general.name") == "test" and f.meta("signed") == -7
    assert f.meta("float") == 1.5 and f.meta("double") == -2.25 and f.meta("array") == ("array", 2)
    with pytest.raises(tcc.GGUFError, match="gguf_metadata_missing"):
        f.meta("absent")
    f.close()
    for limit in ("retained", "directory", "string", "count", "array"):
        agree(tmp_path, data, limit=limit, expect_ok=False)


def test_directory_buffer_boundaries(tmp_path):
    """A directory longer than the read buffers, cut at buffer-sized
    boundaries: the cached window must never hide a truncated table."""
    meta = [metadata("general.name", 8, "x" * 5003),
            text("tokens") + struct.pack("<IIQ", 9, 8, 1203) +
            b"".join(text("symbol" * (1 + i % 19)) for i in range(1203))]
    data = fixture([("w", 8, [32])], meta)
    agree(tmp_path, data, ["w"], expect_ok=True)
    for cut in (4095, 4096, 4097, 8191, 8192, 8193, 65535, 65536, 65537):
        if cut < len(data):
            agree(tmp_path, data[:cut], expect_ok=False)


def test_split_sets(tmp_path):
    def shard(number, count=2, total=2, arch="qwen3", name=None):
        meta = [metadata("split.no", 2, number), metadata("split.count", 2, count),
                metadata("split.tensors.count", 5, total), metadata("general.architecture", 8, arch)]
        return fixture([(name or f"w{number}", 8, [32])], meta)
    first = tmp_path / "first.gguf"
    first.write_bytes(shard(0))
    second = tmp_path / "second.gguf"
    for raw, expected in [(shard(1), True), (shard(0), False), (shard(1, arch="other"), False),
                          (shard(1, total=3), False), (shard(1, name="w0"), False)]:
        second.write_bytes(raw)
        files = [tcc.GGUFFile(first), tcc.GGUFFile(second)]
        try:
            tcc.GGUFFile.validate_split(files)
            got = True
        except tcc.GGUFError:
            got = False
        assert got == expected
        if PROBE.exists():
            r = subprocess.run([str(PROBE), "split", str(first), str(second)], capture_output=True, timeout=20)
            assert (r.returncode == 0) == expected
    with pytest.raises(tcc.GGUFError, match="split"):
        tcc.GGUFFile.validate_split([tcc.GGUFFile(first)])


def test_payload_rows_read_back(tmp_path):
    rng = np.random.default_rng(5)
    rows, k = 7, 512
    payload = rng.integers(0, 256, rows * (k // 256) * 210, dtype=np.uint8).tobytes()
    data = fixture([("w", 14, [k, rows])], payload=payload)
    path = tmp_path / "f.gguf"
    path.write_bytes(data)
    f = tcc.GGUFFile(path)
    assert f.read("w").tobytes() == payload
    row = (k // 256) * 210
    assert f.read("w", 2, 3).tobytes() == payload[2 * row:5 * row]
    with pytest.raises(tcc.GGUFError, match="out of bounds"):
        f.read("w", 5, 3)
    f.close()


def test_gguf_py_kquant_file(tmp_path):
    """A container written by gguf-py (independent implementation) with Q4_K
    and Q6_K tensors: directory and payload bytes match gguf-py's reader."""
    gguf = pytest.importorskip("gguf")
    import kq_cases
    path = tmp_path / "model.gguf"
    w = gguf.GGUFWriter(str(path), "test")
    blobs = {}
    for name, typ, n, k in [("blk.0.attn_q.weight", 12, 8, 512), ("blk.0.ffn_down.weight", 14, 4, 768)]:
        raw = tcc.quantize(typ, kq_cases.synthetic_weight(n, k, seed=n + k))
        blobs[name] = (typ, n, k, raw)
        w.add_tensor(name, raw.reshape(n, -1), raw_dtype=gguf.GGMLQuantizationType(typ))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    ok, _, info = agree(tmp_path, path.read_bytes(), list(blobs), expect_ok=True)
    f = tcc.GGUFFile(path)
    r = gguf.GGUFReader(str(path))
    for t in r.tensors:
        typ, n, k, raw = blobs[t.name]
        mine = f.tensor(t.name)
        assert (mine["type"], mine["rows"], mine["columns"]) == (typ, n, k)
        assert mine["file_offset"] == int(t.data_offset)
        assert f.read(t.name).tobytes() == raw.tobytes() == np.asarray(t.data).tobytes()
    f.close()
