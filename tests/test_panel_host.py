"""Host-side panel re-layout (tc_relayout_host) on the CPU: every raw block
byte must land where the panel layout says (an independent numpy
restatement of that layout), rows past N zero; nonfinite scales rejected.
The device-side counterpart is compared with it on the GPU
(test_gpu_stream.py)."""
from __future__ import annotations

import numpy as np
import pytest

import kq_cases
from turbocider_b200 import cuda as tcc

PANEL = 128


def row_slot(r: int) -> int:
    return (r & ~3) | ((r + 2 * ((r >> 2) & 1)) & 3)


def unlayout(typ: int, panels: np.ndarray, n: int, k: int) -> np.ndarray:
    """Raw GGUF rows [n, k/256 * block] rebuilt from the panel layout."""
    kb, bb = k // 256, kq_cases.TYPES[typ][1]
    cb = PANEL * bb
    out = np.zeros((n, kb, bb), dtype=np.uint8)
    for r in range(n):
        p, rr = divmod(r, PANEL)
        s = row_slot(rr)
        for c in range(kb):
            ch = panels[(p * kb + c) * cb:(p * kb + c + 1) * cb]
            blk = out[r, c]
            if typ == 12:
                blk[0:4] = ch[17920 + rr * 4:17920 + rr * 4 + 4]
                blk[4:16] = ch[16384 + rr * 12:16384 + rr * 12 + 12]
                for q in range(4):
                    blk[16 + 32 * q:48 + 32 * q] = ch[q * 4096 + s * 32:q * 4096 + s * 32 + 32]
            elif typ == 13:
                # qs [4][128][32] @0 | qh [128][32] @16384 | sc [128][12] @20480 | dm [128][4] @22016
                blk[0:4] = ch[22016 + rr * 4:22016 + rr * 4 + 4]
                blk[4:16] = ch[20480 + rr * 12:20480 + rr * 12 + 12]
                blk[16:48] = ch[16384 + s * 32:16384 + s * 32 + 32]
                for q in range(4):
                    blk[48 + 32 * q:80 + 32 * q] = ch[q * 4096 + s * 32:q * 4096 + s * 32 + 32]
            else:
                for h in range(2):
                    for part in range(2):
                        o = ((h * 2 + part) * PANEL + s) * 32
                        blk[64 * h + 32 * part:64 * h + 32 * part + 32] = ch[o:o + 32]
                    o = 16384 + (h * PANEL + s) * 32
                    blk[128 + 32 * h:160 + 32 * h] = ch[o:o + 32]
                blk[192:208] = ch[24576 + rr * 16:24576 + rr * 16 + 16]
                blk[208:210] = ch[26624 + rr * 2:26624 + rr * 2 + 2]
    return out.reshape(n, -1)


@pytest.mark.parametrize("typ", [12, 13, 14])
@pytest.mark.parametrize("n,k,n_begin,n_count", [(300, 512, 0, 0), (256, 768, 64, 130), (5, 256, 0, 0)])
def test_relayout_host_places_every_byte(typ, n, k, n_begin, n_count):
    raw = tcc.quantize(typ, kq_cases.synthetic_weight(n, k, seed=n + k)).reshape(n, -1)
    panels = tcc.relayout_host(typ, raw, n, k, n_begin, n_count, threads=4)
    rows = n_count or n - n_begin
    assert panels.nbytes == tcc.panel_bytes(typ, rows, k) == -(-rows // PANEL) * (k // 256) * PANEL * \
        kq_cases.TYPES[typ][1]
    assert np.array_equal(unlayout(typ, panels, rows, k), raw[n_begin:n_begin + rows])
    # the rows past the weight's end in its last panel are zero
    full = unlayout(typ, panels, -(-rows // PANEL) * PANEL, k)
    assert not full[rows:].any()


@pytest.mark.parametrize("typ", [12, 13, 14])
def test_relayout_host_rejects_nonfinite_scale(typ):
    raw = bytearray(kq_cases.extreme_case(typ, 1.0))
    off = 208 if typ == 14 else 0
    raw[off:off + 2] = (0x7C00).to_bytes(2, "little")   # +inf
    with pytest.raises(tcc.DecodeError, match="nonfinite"):
        tcc.relayout_host(typ, bytes(raw), 2, 1024)
    assert tcc.panel_bytes(10, 128, 256) == 0
