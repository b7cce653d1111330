"""Float64 references and error bounds of the reference's own tests, in numpy.

Each function restates a helper of internal/cq/cq_test.go; these are what
the reference's TestKernels checks every kernel against.
"""

from __future__ import annotations

import numpy as np

LUT_Q = 8191


def sylvester(n: int) -> np.ndarray:
    """cq_test.go:44 sylvester: the ±1 Hadamard matrix of order n."""
    h = np.ones((1, 1))
    while h.shape[0] < n:
        h = np.block([[h, h], [h, -h]])
    return h


def unpack(p) -> np.ndarray:
    """The LSB-first codes of every row, [out][groups*group]."""
    idx = np.asarray(p.index, np.uint8).reshape(p.out, -1)
    if p.bits == 4:
        codes = np.stack([idx & 15, idx >> 4], axis=-1)
    else:
        codes = np.stack([(idx >> s) & 3 for s in (0, 2, 4, 6)], axis=-1)
    return codes.reshape(p.out, -1)


def norms(p) -> np.ndarray:
    groups = (p.in_ + p.group - 1) // p.group
    return np.asarray(p.norms16, np.uint16).view(np.float16).astype(np.float64).reshape(p.out, groups)


def dequant64(p) -> np.ndarray:
    """cq_test.go:70 dequant64: w[r, g] = H · cb[idx] · n / √G, cut to In."""
    G = p.group
    groups = (p.in_ + G - 1) // G
    h = sylvester(G)
    cb = np.asarray(p.codebook, np.float64)
    c = cb[unpack(p)].reshape(p.out, groups, G)
    n = norms(p)
    w = np.einsum("jk,rgk->rgj", h, c) * n[:, :, None] / np.sqrt(G)
    return w.reshape(p.out, groups * G)[:, : p.in_]


def cosine(a, b) -> float:
    a = np.asarray(a, np.float64).reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    return float(a @ b / np.sqrt((a @ a) * (b @ b)))


def rotated_bound(p, x) -> np.ndarray:
    """cq_test.go:111 rotatedBound."""
    G = p.group
    groups = (p.in_ + G - 1) // G
    k = groups * G + np.log2(G) + 8
    gamma = k * 2.0 ** -24 / (1 - k * 2.0 ** -24)
    cb = np.abs(np.asarray(p.codebook, np.float64))
    cabs = cb[unpack(p)].reshape(p.out, groups, G).sum(axis=2)
    xp = np.zeros(groups * G)
    xp[: p.in_] = np.abs(np.asarray(x, np.float64))
    xabs = xp.reshape(groups, G).sum(axis=1)
    return (gamma * norms(p) * cabs * xabs[None, :] / np.sqrt(G)).sum(axis=1)


def lut_bound(p, x) -> np.ndarray:
    """cq_test.go:141 lutBound."""
    G = p.group
    groups = (p.in_ + G - 1) // G
    h = sylvester(G)
    cb_max = float(np.max(np.abs(np.asarray(p.codebook, np.float64))))
    per = G * p.bits / 4
    xp = np.zeros(groups * G)
    xp[: p.in_] = np.asarray(x, np.float64)
    bound = np.zeros(p.out)
    n = norms(p)
    for g in range(groups):
        xt = h @ xp[g * G:(g + 1) * G]
        step = 4 // p.bits
        v = np.abs(xt[0::step])
        if p.bits == 2:
            v = v + np.abs(xt[1::step])
        mx = v.max()
        bound += 1.01 * n[:, g] * per * cb_max * mx / (2 * LUT_Q * np.sqrt(G))
    return bound


def tc_bound(p, x):
    """The tensor-core GEMM's rotated operands and per-element error bound
    (WC_GEMM_TENSOR_CORES in include/whistle_b200.h): returns (y64, bound),
    the float64 product of x [rows][In] with p and the bound on
    |y_tc - y64|. fp16 operands rounded once each (2^-10 for a product),
    the fp32 rotation, scaling and K-term accumulation, and fp16's
    subnormals below the power-of-two scales (the 2^-37 term)."""
    G = p.group
    groups = (p.in_ + G - 1) // G
    rows = x.shape[0]
    xp = np.zeros((rows, groups * G))
    xp[:, : p.in_] = x
    xh = np.einsum("jk,rgk->rgj", sylvester(G), xp.reshape(rows, groups, G)).reshape(rows, groups * G)
    cb = np.asarray(p.codebook, np.float64)
    w = (cb[unpack(p)].reshape(p.out, groups, G) * norms(p)[:, :, None] / np.sqrt(G)).reshape(p.out, groups * G)
    K = w.shape[1]
    gamma = 2.0 ** -10 + (K + np.log2(G) + 6) * 2.0 ** -24
    aw, ax = np.abs(w), np.abs(xh)
    amax = np.abs(x).max(axis=1, initial=0.0)[:, None]
    sub = 2.0 ** -37 * (G * amax * aw.sum(axis=1)[None, :] + aw.max(initial=0.0) * ax.sum(axis=1)[:, None])
    return xh @ w.T, gamma * (ax @ aw.T) + sub
