"""The stream layout's permutation (go-whistle_b200/csrc/cq_lut_stream.cu,
api.cu stream_layout), checked on the CPU for every group width: each
lookup of the kernel's addressing reads the right table entry of the right
group, and every warp-wide lookup touches 32 distinct shared-memory banks
(no bank conflicts), for aligned and unaligned Rows views."""

from __future__ import annotations

import numpy as np
import pytest


def layout(src: np.ndarray, gb: int) -> np.ndarray:
    """api.cu stream_layout for the index bytes: [sc][i][row][16]."""
    out, row_bytes = src.shape
    P, NG, nsc = gb // 2, 32 // gb * 2, row_bytes // 64
    NG = 32 // P
    sidx = np.zeros(out * row_bytes, np.uint8)
    for r in range(out):
        lam = r & 31
        a, c = lam // P, lam % P
        for sc in range(nsc):
            ch = np.zeros(64, np.uint8)
            for slot in range(32):
                q, t = slot // P, slot % P
                o = P * ((q + a) % NG) + (t + c) % P
                ch[2 * slot:2 * slot + 2] = src[r, 64 * sc + 2 * o:64 * sc + 2 * o + 2]
            for i in range(4):
                base = ((sc * 4 + i) * out + r) * 16
                sidx[base:base + 16] = ch[16 * i:16 * i + 16]
    return sidx


@pytest.mark.parametrize("gb", [8, 16, 32, 64])
@pytest.mark.parametrize("row_bytes,out,row0", [(256, 70, 5), (1024, 40, 32), (128, 45, 0)])
def test_permutation_reads_right_entries_without_conflicts(gb, row_bytes, out, row0):
    P, NG = gb // 2, 32 // (gb // 2)
    rng = np.random.default_rng(gb + row_bytes)
    src = rng.integers(0, 256, (out, row_bytes), dtype=np.uint8)
    sidx = layout(src, gb)
    nsc = row_bytes // 64
    vout = out - row0
    for tile in range((vout + 31) // 32):
        banks = {}
        for lane in range(32):
            r = tile * 32 + lane
            if r >= vout:
                continue
            R = row0 + r
            lam = ((row0 & 31) + lane) & 31
            assert lam == R % 32
            a, c = lam // P, lam % P
            cb = []
            for b in range(64):
                slot, e = b >> 1, b & 1
                q, t = slot // P, slot % P
                cb.append(4 * (P * ((q + a) % NG) + (t + c) % P) + 2 * e)
            for sc in range(nsc):
                scl = sc % 4
                data = np.concatenate([sidx[((sc * 4 + i) * out + R) * 16:((sc * 4 + i) * out + R) * 16 + 16]
                                       for i in range(4)])
                for q in range(NG):
                    gl = (q + a) % NG
                    for t in range(P):
                        slot = P * q + t
                        for e in range(2):
                            byte, colb = int(data[2 * slot + e]), cb[2 * slot + e]
                            assert colb < 128
                            addr = 65536 + (scl >> 1) * 65536 + (scl & 1) * 128 + colb + 256 * byte
                            assert 65536 <= addr and addr + 2 <= 65536 + 131072
                            rel = addr - 65536
                            blk, rem = rel // 65536, rel % 65536
                            b, jj = rem // 256, (rem % 256) // 2
                            j = 256 * (sc // 4) + 128 * blk + jj
                            assert b == src[R, j] and (j % 64) // gb == gl
                            word = addr // 4
                            banks.setdefault((sc, q, t, e), {}).setdefault(word % 32, set()).add(word)
        for step, per_bank in banks.items():
            assert all(len(words) == 1 for words in per_bank.values()), step
