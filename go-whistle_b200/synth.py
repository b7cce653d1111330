"""Seeded synthetic inputs in the reference's formats (no corpora, no model
file exist in this image; these stand in for them with the shapes, sizes and
value distributions the benchmark configurations name).

- CQ tensors as cact.Packed holds them (internal/cact/packed.go:18-40): one
  sorted codebook per width, uniform index bytes (every code uniform), FP16
  norms with exponent uniform in 11..19 and a random mantissa (2^-4..2^4),
  as the reference's own tests draw them (internal/cq/cq_test.go:20-41).
- int8 KV caches: codes uniform in [-127, 127], scales uniform 0.01..0.05
  per (token, head); queries ~N(0, 1).
"""

from __future__ import annotations

import numpy as np

from .cq import Packed

# quantize.py's unit-variance Gaussian Lloyd-Max levels, as the reference's
# tests record them (internal/cact/cq_test.go:16-29); the whistle.cact
# codebooks are these over sqrt(group), rounded to float32.
LLOYD_MAX_UNIT = {
    2: [-1.5066708475715247, -0.45144060939344055, 0.4529474939511613, 1.5099326242547164],
    4: [-2.709990028558534, -2.0444556051349227, -1.5947570221842273, -1.233336191082712,
        -0.9222139662739897, -0.6395373737252813, -0.37266394934485414, -0.11445072030649898,
        0.14380628677643076, 0.4039889754802918, 0.6726933686864701, 0.9614053009735016,
        1.2755257831234952, 1.637058796059282, 2.0844263722579237, 2.7410141261982846],
}


def lloyd_max_codebook(bits: int, group: int) -> np.ndarray:
    """cact_test.go portCodebook: the stored whistle.cact levels."""
    return np.array([c / np.sqrt(group) for c in LLOYD_MAX_UNIT[bits]], np.float32)


def random_norms16(rng: np.random.Generator, n: int) -> np.ndarray:
    """FP16 norms 2^-4..2^4: exponent field 11..19, random mantissa."""
    exp = rng.integers(11, 20, size=n, dtype=np.uint16)
    man = rng.integers(0, 1024, size=n, dtype=np.uint16)
    return (exp << 10) | man


def random_packed(rng: np.random.Generator, out: int, in_: int, group: int, bits: int,
                  codebook: str = "baseline") -> Packed:
    """A random CQ tensor. codebook: "baseline" = sorted ~N(0, 0.02) (the
    benchmark configurations), "reference" = sorted ~N(0,1)/sqrt(G)
    (cq_test.go randomPacked), "lloyd" = the whistle.cact levels."""
    if codebook == "baseline":
        cb = np.sort(rng.normal(0.0, 0.02, size=1 << bits)).astype(np.float32)
    elif codebook == "reference":
        cb = np.sort(rng.normal(0.0, 1.0, size=1 << bits) / np.sqrt(group)).astype(np.float32)
    elif codebook == "lloyd":
        cb = lloyd_max_codebook(bits, group)
    else:
        raise ValueError(codebook)
    groups = (in_ + group - 1) // group
    row_bytes = groups * group * bits // 8
    index = rng.integers(0, 256, size=out * row_bytes, dtype=np.uint8)
    norms = random_norms16(rng, out * groups).astype("<u2").view(np.uint8)
    return Packed(Out=out, In=in_, Group=group, Bits=bits, Width=bits, Codebook=cb, Index=index, Norms=norms)


def algorithmic_bytes_gemv(out: int, in_: int, group: int, bits: int) -> int:
    """Bytes one batch-1 GEMV must move: packed index + FP16 norms + x + y +
    codebook, B = Out·RowBytes + 2·Out·Groups + 4·In + 4·Out + 4·2^bits."""
    groups = (in_ + group - 1) // group
    row_bytes = groups * group * bits // 8
    return out * row_bytes + 2 * out * groups + 4 * in_ + 4 * out + 4 * (1 << bits)


def random_kv(rng: np.random.Generator, rows: int, kv_heads: int, width: int):
    """An int8 cache: codes uniform in [-127, 127], scales U(0.01, 0.05)."""
    q = rng.integers(-127, 128, size=rows * kv_heads * width, dtype=np.int8)
    s = rng.uniform(0.01, 0.05, size=rows * kv_heads).astype(np.float32)
    return q, s
