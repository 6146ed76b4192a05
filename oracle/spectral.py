"""Oracle (test infrastructure): spectral bases and the spectral Lerp FFN in numpy.

Reference: mcarbonell/delta-phase v1.3.0.

* :func:`hadamard_matrix` -- ``create_hadamard_matrix`` (delta_phase/spectral.py:4-12)
* :func:`dct2_matrix`     -- ``create_dct2_matrix``     (delta_phase/spectral.py:14-23)
* :func:`haar_matrix`     -- ``create_haar_matrix``     (delta_phase/spectral.py:25-35)
* :func:`lerp_ffn`        -- ``LearnableSubstrateLerpFFN.forward``
                             (delta_phase/layers.py:119-141)

The matrices are produced exactly as the reference does (entries rounded to
float32, since the reference stores them as float32 buffers) and then widened.
"""
from __future__ import annotations

import math

import numpy as np

BRANCHES = ("fwht", "dct", "haar")


def hadamard_matrix(n):
    """Sylvester Hadamard / sqrt(n) (spectral.py:4-12).  Like the reference, a
    non-power-of-two n yields the next power-of-two size."""
    H = np.ones((1, 1), dtype=np.float32)
    while H.shape[0] < n:
        H = np.block([[H, H], [H, -H]])
    return (H / np.float32(math.sqrt(n))).astype(np.float32)


def dct2_matrix(n):
    """Orthonormal DCT-II, row k = frequency (spectral.py:14-23)."""
    k = np.arange(n, dtype=np.float64)[:, None]
    i = np.arange(n, dtype=np.float64)[None, :]
    C = math.sqrt(2.0 / n) * np.cos(math.pi * k * (2 * i + 1) / (2.0 * n))
    C[0, :] = 1.0 / math.sqrt(n)
    return C.astype(np.float32)


def haar_matrix(n):
    """The reference's recursive "Haar" matrix (spectral.py:25-35): low rows are
    ``[H_{n/2}, H_{n/2}] / sqrt(2)`` and high row i pairs x[2i], x[2i+1].  It is not
    orthogonal.  n must be a power of two (the reference raises otherwise)."""
    if n == 1:
        return np.ones((1, 1), dtype=np.float32)
    if n % 2:
        raise RuntimeError("Sizes of tensors must match (haar of odd size)")
    sub = haar_matrix(n // 2)
    low = (np.concatenate([sub, sub], 1) / np.float32(math.sqrt(2))).astype(np.float32)
    high = np.zeros((n // 2, n), dtype=np.float32)
    idx = np.arange(n // 2)
    high[idx, 2 * idx] = np.float32(1.0 / math.sqrt(2))
    high[idx, 2 * idx + 1] = np.float32(-1.0 / math.sqrt(2))
    return np.concatenate([low, high], 0)


def matrices(d):
    return {"fwht": hadamard_matrix(d), "dct": dct2_matrix(d), "haar": haar_matrix(d)}


def lerp_ffn(x, params, dtype=np.float64):
    """``LearnableSubstrateLerpFFN.forward`` (layers.py:119-141).

    ``params`` holds the reference names: substrate_logits (3,), mat_fwht/mat_dct/
    mat_haar (d, d), phi1_*/phi2_*/w1_*/w2_* (nb, d), combine.weight (d, nb*d).
    x (..., d) -> (..., d).
    """
    x = np.asarray(x, dtype=dtype)
    logits = np.asarray(params["substrate_logits"], dtype=dtype)
    w = np.exp(logits - logits.max())
    w = w / w.sum()                                               # :120
    Wc = np.asarray(params["combine.weight"], dtype=dtype)
    y = 0.0
    for b, name in enumerate(BRANCHES):                            # :122-138
        M = np.asarray(params[f"mat_{name}"], dtype=dtype)
        h = (x @ M.T)[..., None, :]                                # F.linear(x, M)
        a = (np.cos(h + np.asarray(params[f"phi1_{name}"], dtype=dtype))
             * np.asarray(params[f"w1_{name}"], dtype=dtype)
             + np.sin(h + np.asarray(params[f"phi2_{name}"], dtype=dtype))
             * np.asarray(params[f"w2_{name}"], dtype=dtype))
        a = a.reshape(a.shape[:-2] + (-1,))                        # flatten(-2)
        c = a @ Wc.T                                               # combine
        y = y + w[b] * (c @ M)                                     # F.linear(c, M.t())
    return y                                                       # :141
