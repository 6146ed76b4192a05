"""Oracle (test infrastructure): the complex phasor delta rule, restated in numpy.

Reference: mcarbonell/delta-phase v1.3.0.

* :func:`chunkwise_delta`  -- ``_chunkwise_delta_reference``
  (delta_phase/kernels/triton_chunk_delta.py:211-252); identical to the inlined
  copy in ``DeltaPhaseHolographicBlock.forward`` (delta_phase/layers.py:203-236).
* :func:`recurrent_delta`  -- the token recurrence of
  ``DeltaPhaseHolographicBlock.step`` (delta_phase/layers.py:279-285) run over a
  whole sequence; the reference's own definition of correctness
  (tests/test_equivalence.py:18-56).
* :func:`decode_step`      -- one step of that recurrence (layers.py:279-285).
* :func:`complex_beta_step`, :func:`complex_beta_recurrent` -- the complex-beta
  Householder rule of ``ComplexBetaDeltaPhaseBlock`` (delta_phase/layers.py:294-418):
  one token, and its token loop over a sequence (layers.py:346-360).
* :func:`gram_matrix`      -- ``gram_matrix_reference``
  (triton_chunk_delta.py:192-208), the contract of the archived Triton Gram
  kernel (triton_chunk_delta.py:32-98).

All functions take numpy arrays and a ``dtype`` (float64 for parity checks,
float32 when timed as the CPU baseline).  Shapes follow the reference:
theta_k/theta_q/v ``(B, H, L, D)``, beta ``(B, H, L)``, state ``(B, H, Dv, D)``
complex with row = value channel, column = key channel.
"""
from __future__ import annotations

import numpy as np


def _cplx(dtype):
    return np.complex128 if np.dtype(dtype) == np.float64 else np.complex64


def phasor(theta, dtype=np.float64):
    """K = cos(theta) + i sin(theta)  (triton_chunk_delta.py:220-221)."""
    t = np.asarray(theta, dtype=dtype)
    return (np.cos(t) + 1j * np.sin(t)).astype(_cplx(dtype))


def unit_lower_inverse(lower):
    """Inverse of (I + lower) for strictly-lower ``lower`` (..., C, C).

    Restates ``torch.linalg.solve_triangular(I + L^T, I, upper=False)``
    (triton_chunk_delta.py:231-232) by forward substitution, row by row,
    vectorised over the leading batch axes.
    """
    C = lower.shape[-1]
    T = np.zeros_like(lower)
    eye = np.eye(C, dtype=lower.dtype)
    for i in range(C):
        # row i of T:  T[i] = e_i - sum_{k<i} lower[i,k] T[k]
        T[..., i, :] = eye[i] - np.einsum("...k,...kj->...j", lower[..., i, :i], T[..., :i, :])
    return T


def gram_matrix(theta_k, beta, dtype=np.float64):
    """Strictly-lower, row-beta-scaled phasor Gram (triton_chunk_delta.py:192-208).

    G[m, n] = beta_m * sum_d cos(theta_m,d - theta_n,d) / D  for m > n, else 0.
    theta_k (N, C, D), beta (N, C) -> (N, C, C).
    """
    th = np.asarray(theta_k, dtype=dtype)
    b = np.asarray(beta, dtype=dtype)
    D = th.shape[-1]
    c, s = np.cos(th), np.sin(th)
    g = (c @ np.swapaxes(c, -1, -2) + s @ np.swapaxes(s, -1, -2)) / D
    g = g * b[..., :, None]
    C = th.shape[-2]
    keep = np.tril(np.ones((C, C), dtype=bool), -1)
    return np.where(keep, g, 0.0).astype(dtype)


def chunkwise_delta(theta_k, theta_q, v, beta, chunk_size=64, initial_state=None,
                    dtype=np.float64):
    """Chunkwise WY delta rule (triton_chunk_delta.py:211-252).

    Returns ``(out (B,H,L,Dv) real, M (B,H,Dv,D) complex)``.  Like the reference,
    L must be a multiple of ``chunk_size`` (the reference ``view`` at :223-227).
    """
    tk = np.asarray(theta_k, dtype=dtype)
    tq = np.asarray(theta_q, dtype=dtype)
    vv = np.asarray(v, dtype=dtype)
    bb = np.asarray(beta, dtype=dtype)
    B, H, L, D = tk.shape
    Dv = vv.shape[-1]
    C = int(chunk_size)
    if L % C != 0:
        raise ValueError(f"L={L} is not a multiple of chunk_size={C}")
    inv_dk = 1.0 / float(D)
    cd = _cplx(dtype)
    K = phasor(tk, dtype)
    Q = phasor(tq, dtype)
    NC = L // C
    Kc = K.reshape(B, H, NC, C, D)
    Qc = Q.reshape(B, H, NC, C, D)
    Vc = vv.reshape(B, H, NC, C, Dv)
    bc = bb.reshape(B, H, NC, C)

    # :229-232  Gram, strictly-upper L = triu(G * beta_row, 1), T = (I + L^T)^-1
    gram = np.real(Kc @ np.conj(np.swapaxes(Kc, -1, -2))) * inv_dk
    Lmat = np.triu(gram * bc[..., :, None], 1)
    T = unit_lower_inverse(np.swapaxes(Lmat, -1, -2))

    # :234-238
    if initial_state is None:
        M = np.zeros((B, H, Dv, D), dtype=cd)
    else:
        M = np.array(initial_state, dtype=cd, copy=True)

    out = np.empty((B, H, NC, C, Dv), dtype=dtype)
    for c in range(NC):                                           # :241-249
        qc, kc, vc, bcc, tc = Qc[:, :, c], Kc[:, :, c], Vc[:, :, c], bc[:, :, c], T[:, :, c]
        v_old = np.swapaxes(np.real(M @ np.conj(np.swapaxes(kc, -1, -2))), -1, -2) * inv_dk
        E = tc @ (vc - v_old)
        U = bcc[..., None] * E
        o_inter = np.swapaxes(np.real(M @ np.conj(np.swapaxes(qc, -1, -2))), -1, -2) * inv_dk
        A_intra = np.tril(np.real(qc @ np.conj(np.swapaxes(kc, -1, -2)))) * inv_dk
        out[:, :, c] = A_intra @ U + o_inter
        M = M + np.swapaxes(U.astype(cd), -1, -2) @ kc
    return out.reshape(B, H, L, Dv), M


def decode_step(M, theta_k, theta_q, v, beta, dtype=np.float64):
    """One decode step (layers.py:279-285): read -> correct -> update -> read.

    M (B,H,Dv,D) complex; theta_k/theta_q (B,H,D); v (B,H,Dv); beta (B,H).
    Returns ``(out (B,H,Dv), M_new)``; the input state is not modified.
    """
    D = np.asarray(theta_k).shape[-1]
    inv_dk = 1.0 / float(D)
    cd = _cplx(dtype)
    k = phasor(theta_k, dtype)
    q = phasor(theta_q, dtype)
    vv = np.asarray(v, dtype=dtype)
    bb = np.asarray(beta, dtype=dtype)
    M = np.asarray(M, dtype=cd)
    v_old = np.real(np.einsum("bhoc,bhc->bho", M, np.conj(k))) * inv_dk
    err = vv - v_old
    Mn = M + bb[..., None, None] * (err.astype(cd)[..., :, None] * k[..., None, :])
    out = np.real(np.einsum("bhoc,bhc->bho", Mn, np.conj(q))) * inv_dk
    return out.astype(dtype), Mn


def recurrent_delta(theta_k, theta_q, v, beta, initial_state=None, dtype=np.float64):
    """Token-by-token recurrence over a whole sequence (layers.py:279-285 looped,
    as tests/test_equivalence.py:38-45 does through ``block.step``)."""
    tk = np.asarray(theta_k, dtype=dtype)
    B, H, L, D = tk.shape
    Dv = np.asarray(v).shape[-1]
    M = (np.zeros((B, H, Dv, D), dtype=_cplx(dtype)) if initial_state is None
         else np.array(initial_state, dtype=_cplx(dtype), copy=True))
    out = np.empty((B, H, L, Dv), dtype=dtype)
    for t in range(L):
        out[:, :, t], M = decode_step(M, tk[:, :, t], np.asarray(theta_q)[:, :, t],
                                      np.asarray(v)[:, :, t], np.asarray(beta)[:, :, t], dtype)
    return out, M


def complex_beta_step(M, theta_k, theta_q, v, phi, dtype=np.float64):
    """One token of ``ComplexBetaDeltaPhaseBlock`` (layers.py:402-407; the loop body of
    its ``forward``, layers.py:354-360): beta = 1 + e^{i phi} (layers.py:344, 397),
    v_old = Re(M conj(k)) / D, M <- M + beta (v - v_old) k^T, out = Re(M conj(q)) / D.

    M (B,H,Dv,D) complex; theta_k/theta_q (B,H,D); v (B,H,Dv); phi (B,H).
    Returns ``(out (B,H,Dv), M_new)``; the input state is not modified.
    """
    D = np.asarray(theta_k).shape[-1]
    inv_dk = 1.0 / float(D)
    cd = _cplx(dtype)
    k = phasor(theta_k, dtype)
    q = phasor(theta_q, dtype)
    vv = np.asarray(v, dtype=dtype)
    bt = (1.0 + phasor(phi, dtype)).astype(cd)
    M = np.asarray(M, dtype=cd)
    v_old = np.real(np.einsum("bhoc,bhc->bho", M, np.conj(k))) * inv_dk
    err = (vv - v_old).astype(cd)
    Mn = M + bt[..., None, None] * (err[..., :, None] * k[..., None, :])
    out = np.real(np.einsum("bhoc,bhc->bho", Mn, np.conj(q))) * inv_dk
    return out.astype(dtype), Mn


def complex_beta_recurrent(theta_k, theta_q, v, phi, initial_state=None, dtype=np.float64):
    """The token loop of ``ComplexBetaDeltaPhaseBlock.forward`` (layers.py:346-360) over
    a whole sequence.  theta_k/theta_q/v (B,H,L,D), phi (B,H,L).
    Returns ``(out (B,H,L,Dv), M (B,H,Dv,D) complex)``."""
    tk = np.asarray(theta_k, dtype=dtype)
    B, H, L, D = tk.shape
    Dv = np.asarray(v).shape[-1]
    M = (np.zeros((B, H, Dv, D), dtype=_cplx(dtype)) if initial_state is None
         else np.array(initial_state, dtype=_cplx(dtype), copy=True))
    out = np.empty((B, H, L, Dv), dtype=dtype)
    for t in range(L):
        out[:, :, t], M = complex_beta_step(M, tk[:, :, t], np.asarray(theta_q)[:, :, t],
                                            np.asarray(v)[:, :, t], np.asarray(phi)[:, :, t], dtype)
    return out, M


def rel_l2(a, b):
    """Relative L2 error ||a - b|| / ||b|| (complex arrays compare as real pairs)."""
    a = np.asarray(a)
    b = np.asarray(b)
    if np.iscomplexobj(a) or np.iscomplexobj(b):
        a = np.stack([np.real(a), np.imag(a)], -1)
        b = np.stack([np.real(b), np.imag(b)], -1)
    a = a.astype(np.float64)
    b = b.astype(np.float64)
    den = np.linalg.norm(b.ravel())
    num = np.linalg.norm((a - b).ravel())
    return float(num / den) if den > 0 else float(num)
