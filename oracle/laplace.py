"""Oracle (test infrastructure): LaplacePhaseCore, restated in numpy.

Reference: mcarbonell/delta-phase v1.3.0, delta_phase/layers.py.

* :func:`project`            -- ``LaplacePhaseCore._project`` (layers.py:462-479)
* :func:`laplace_chunkwise`  -- the chunk loop of ``LaplacePhaseCore.forward``
                                (layers.py:481-561), fed the projected phasors
* :func:`laplace_sequential` -- ``LaplacePhaseCore.forward_sequential``
                                (layers.py:563-583), the token-loop oracle

Inputs: K, Q complex (B,H,L,D) (magnitude r = e^sigma, phase theta); v (B,H,L,Dv);
beta (B,H,L); r (B,H,L,Dv) per-row decay in (0,1]; M0 (B,H,Dv,D) complex.
"""
from __future__ import annotations

import numpy as np

LOG_FLOOR = -80.0  # layers.py:445


def _cplx(dtype):
    return np.complex128 if np.dtype(dtype) == np.float64 else np.complex64


def _softplus(x):
    return np.logaddexp(0.0, x)


def project(x, weights, n_heads, d_k, time_scale=1.0, dtype=np.float64):
    """``_project`` (layers.py:462-479).  ``weights`` maps the reference parameter
    names (w_theta_k, w_sigma_k, w_theta_q, w_sigma_q, w_v, w_beta) to (out, in)
    matrices; x (B, L, d_model).  Returns (K, Q, v, beta, r_k) in the layout above.
    """
    x = np.asarray(x, dtype=dtype)
    B, L, _ = x.shape
    dt = 1.0 / float(time_scale)

    def lin(name):
        return x @ np.asarray(weights[name], dtype=dtype).T

    def heads(y):
        return y.reshape(B, L, n_heads, d_k).transpose(0, 2, 1, 3)

    theta_k = heads(lin("w_theta_k") * dt)
    sigma_k = heads(-_softplus(lin("w_sigma_k")) * dt)
    theta_q = heads(lin("w_theta_q") * dt)
    sigma_q = heads(-_softplus(lin("w_sigma_q")) * dt)
    v = heads(lin("w_v"))
    beta = (2.0 / (1.0 + np.exp(-lin("w_beta"))) * dt).transpose(0, 2, 1)
    r_k = np.exp(sigma_k)
    K = (r_k * np.cos(theta_k) + 1j * (r_k * np.sin(theta_k))).astype(_cplx(dtype))
    r_q = np.exp(sigma_q)
    Q = (r_q * np.cos(theta_q) + 1j * (r_q * np.sin(theta_q))).astype(_cplx(dtype))
    return K, Q, v.astype(dtype), beta.astype(dtype), r_k.astype(dtype)


def laplace_chunkwise(K, Q, v, beta, r, chunk_size=32, initial_state=None,
                      dtype=np.float64):
    """Chunkwise exact solve of ``LaplacePhaseCore.forward`` (layers.py:481-561).

    Returns ``(out (B,H,L,Dv), M (B,H,Dv,D))``.  Pads the tail with r = 1,
    beta = 0 like the reference (:490-497) and undoes the (trivial) pad decay
    (:555-559).
    """
    cd = _cplx(dtype)
    K = np.asarray(K, dtype=cd)
    Q = np.asarray(Q, dtype=cd)
    v = np.asarray(v, dtype=dtype)
    beta = np.asarray(beta, dtype=dtype)
    r = np.asarray(r, dtype=dtype)
    B, H, L, dk = K.shape
    Dv = v.shape[-1]
    inv_dk = 1.0 / float(dk)
    M = (np.zeros((B, H, Dv, dk), dtype=cd) if initial_state is None
         else np.array(initial_state, dtype=cd, copy=True))

    C = min(int(chunk_size), max(L, 1))                           # :491
    pad = (C - L % C) % C
    if pad:                                                       # :492-497
        K = np.concatenate([K, np.zeros((B, H, pad, dk), cd)], 2)
        Q = np.concatenate([Q, np.zeros((B, H, pad, dk), cd)], 2)
        v = np.concatenate([v, np.zeros((B, H, pad, Dv), dtype)], 2)
        r = np.concatenate([r, np.ones((B, H, pad, Dv), dtype)], 2)
        beta = np.concatenate([beta, np.zeros((B, H, pad), dtype)], 2)
    NC = (L + pad) // C
    Kv = K.reshape(B, H, NC, C, dk)
    Qv = Q.reshape(B, H, NC, C, dk)
    vv = v.reshape(B, H, NC, C, Dv)
    rv = r.reshape(B, H, NC, C, Dv)
    bv = beta.reshape(B, H, NC, C)
    tril0 = np.tril(np.ones((C, C), dtype=bool))
    trilm1 = np.tril(np.ones((C, C), dtype=bool), -1)
    eye = np.eye(C, dtype=dtype)

    outs = []
    for ci in range(NC):                                          # :507-550
        kc, qc = Kv[:, :, ci], Qv[:, :, ci]
        vo, bc, rc = vv[:, :, ci], bv[:, :, ci], rv[:, :, ci]
        with np.errstate(divide="ignore"):
            Sr = np.cumsum(np.maximum(np.log(rc), LOG_FLOOR), axis=2)   # :512 (B,H,m,o)
        G = np.exp(Sr)
        Gprev = np.concatenate([np.ones_like(G[:, :, :1]), G[:, :, :-1]], 2)
        kH = np.conj(np.swapaxes(kc, -1, -2))
        qH = np.conj(np.swapaxes(qc, -1, -2))
        g_km = np.real(kc @ kH) * inv_dk                          # :516 [s,m]
        h_qm = np.real(kc @ qH) * inv_dk                          # :517 [s,m]
        B0k = np.real(M @ kH) * inv_dk                            # :519 (o,m)
        B0q = np.real(M @ qH) * inv_dk                            # :520
        Sro = np.swapaxes(Sr, -1, -2)                             # (o,m)
        Sro_prev = np.concatenate([np.zeros_like(Sro[..., :1]), Sro[..., :-1]], -1)
        P_oms = np.exp(Sro_prev[..., :, None] - Sro[..., None, :])  # (o,m,s)
        coef = P_oms * bc[:, :, None, None, :] * np.swapaxes(g_km, -1, -2)[:, :, None]
        Acoef = eye + np.where(trilm1, coef, 0.0)                 # :528-531
        RHS = np.swapaxes(vo - Gprev * np.swapaxes(B0k, -1, -2), -1, -2)  # (o,m) :533
        # :534 per-channel lower-triangular solve by forward substitution
        E = np.zeros_like(RHS)
        for m in range(C):
            E[..., m] = RHS[..., m] - np.einsum("...s,...s->...", Acoef[..., m, :m], E[..., :m])
        Et = np.swapaxes(E, -1, -2)                               # (m,o)
        BEt = bc[..., None] * Et
        Ointer = G * np.swapaxes(B0q, -1, -2)                     # :539
        with np.errstate(over="ignore", invalid="ignore"):
            FE = np.exp(-Sr) * BEt                                # :540
            Hl = np.swapaxes(np.where(tril0, np.swapaxes(h_qm, -1, -2), 0.0), -1, -2)
            Z = np.swapaxes(Hl, -1, -2) @ FE                      # :543
            outs.append(Ointer + G * Z)                           # :544
        Wdec = np.exp(Sr[:, :, -1:, :] - Sr)                      # :547
        WE = Wdec * BEt
        M = np.exp(Sr[:, :, -1, :])[..., None] * M + np.swapaxes(WE.astype(cd), -1, -2) @ kc

    out = np.concatenate(outs, 2)[:, :, :L]
    if pad:                                                       # :555-559
        pad_G = np.prod(rv[:, :, -1, C - pad:, :], axis=2)
        safe = np.where(pad_G > 1e-30, pad_G, 1.0)
        M = M / safe.astype(cd)[..., None]
    return out, M


def laplace_sequential(K, Q, v, beta, r, initial_state=None, dtype=np.float64):
    """Token loop ``forward_sequential`` (layers.py:563-583).

    v_old reads the pre-decay state; the decay scales rows (value channels).
    Returns ``(out (B,H,L,Dv), M)``.
    """
    cd = _cplx(dtype)
    K = np.asarray(K, dtype=cd)
    Q = np.asarray(Q, dtype=cd)
    v = np.asarray(v, dtype=dtype)
    beta = np.asarray(beta, dtype=dtype)
    r = np.asarray(r, dtype=dtype)
    B, H, L, dk = K.shape
    Dv = v.shape[-1]
    inv_dk = 1.0 / float(dk)
    M = (np.zeros((B, H, Dv, dk), dtype=cd) if initial_state is None
         else np.array(initial_state, dtype=cd, copy=True))
    out = np.empty((B, H, L, Dv), dtype=dtype)
    for t in range(L):
        kt, qt = K[:, :, t], Q[:, :, t]
        v_old = np.real(np.einsum("bhoc,bhc->bho", M, np.conj(kt))) * inv_dk
        err = v[:, :, t] - v_old
        M = M * r[:, :, t][..., None] + beta[:, :, t][..., None, None] * (
            err.astype(cd)[..., :, None] * kt[..., None, :])
        out[:, :, t] = np.real(np.einsum("bhoc,bhc->bho", M, np.conj(qt))) * inv_dk
    return out, M
