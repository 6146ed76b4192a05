"""Oracle (test infrastructure): gradients of the delta-rule core, as the reference computes
them when it trains -- PyTorch autograd through its recurrence.

Reference: mcarbonell/delta-phase v1.3.0.  The reference's training path is autograd of
its PyTorch code: ``delta_phase_chunkwise_fused`` sends gradient-enabled calls to
``_chunkwise_delta_reference`` (delta_phase/kernels/triton_chunk_delta.py:279-291,
:211-252), and ``ComplexBetaDeltaPhaseBlock.forward`` differentiates its token loop
(delta_phase/layers.py:346-360).  The functions here restate those recurrences token by
token in torch on the CPU (float64) and let autograd produce the gradients:

* :func:`core_grads`         -- real beta (the chunkwise path and its token recurrence,
  layers.py:279-285, are the same function of the inputs).
* :func:`complex_beta_grads` -- complex beta = 1 + e^{i phi} (layers.py:344, 354-360).
* :func:`laplace_grads`      -- the LaplacePhaseCore recurrence with per-row decay
  (layers.py:481-583).

core_grads and complex_beta_grads take numpy inputs and the output / final-state gradients (``dout`` (B,H,L,Dv),
``dM`` (B,H,Dv,D) complex or None) and return numpy gradients
``(d theta_k, d theta_q, d v, d beta_or_phi, d M0 or None)`` with PyTorch's complex
convention (dL/dRe + i dL/dIm).  Pinned against gradients of the reference itself in
tests/golden/grad.npz and tests/golden/laplace_grad.npz.
"""
from __future__ import annotations

import numpy as np
import torch


def _t(a, requires_grad=True):
    t = torch.from_numpy(np.asarray(a, dtype=np.float64).copy())
    return t.requires_grad_(requires_grad)


def _loop(tk, tq, v, g, M0, complex_beta):
    """The token recurrence (layers.py:279-285 for real beta, layers.py:354-360 for the
    complex beta) in torch float64: returns (out (B,H,L,Dv), M_final)."""
    B, H, L, D = tk.shape
    Dv = v.shape[-1]
    K = torch.polar(torch.ones_like(tk), tk)
    Q = torch.polar(torch.ones_like(tq), tq)
    M = torch.zeros(B, H, Dv, D, dtype=torch.complex128) if M0 is None else M0
    outs = []
    for t in range(L):
        k, q = K[:, :, t], Q[:, :, t]
        v_old = torch.matmul(M, torch.conj(k).unsqueeze(-1)).squeeze(-1).real / D
        err = (v[:, :, t] - v_old).to(M.dtype)
        bt = (1.0 + torch.polar(torch.ones_like(g[:, :, t]), g[:, :, t])) if complex_beta else g[:, :, t]
        M = M + bt.unsqueeze(-1).unsqueeze(-1) * torch.matmul(err.unsqueeze(-1), k.unsqueeze(-2))
        outs.append(torch.matmul(M, torch.conj(q).unsqueeze(-1)).squeeze(-1).real / D)
    return torch.stack(outs, 2), M


def _grads(theta_k, theta_q, v, g, dout, dM, M0, complex_beta):
    tk, tq, vv, gg = _t(theta_k), _t(theta_q), _t(v), _t(g)
    m0 = None
    if M0 is not None:
        m0 = torch.from_numpy(np.asarray(M0, dtype=np.complex128).copy()).requires_grad_(True)
    out, M = _loop(tk, tq, vv, gg, m0, complex_beta)
    outs, gos = [out], [torch.from_numpy(np.asarray(dout, dtype=np.float64))]
    if dM is not None:
        outs.append(M)
        gos.append(torch.from_numpy(np.asarray(dM, dtype=np.complex128)))
    inputs = [tk, tq, vv, gg] + ([m0] if m0 is not None else [])
    grads = torch.autograd.grad(outs, inputs, gos, allow_unused=True)
    res = [None if x is None else x.detach().numpy() for x in grads[:4]]
    res.append(grads[4].detach().numpy() if m0 is not None else None)
    return tuple(res)


def core_grads(theta_k, theta_q, v, beta, dout, dM=None, M0=None):
    """Gradients of the real-beta core (triton_chunk_delta.py:211-252)."""
    return _grads(theta_k, theta_q, v, beta, dout, dM, M0, False)


def complex_beta_grads(theta_k, theta_q, v, phi, dout, dM=None, M0=None):
    """Gradients of the complex-beta token loop (layers.py:346-360) w.r.t. phi."""
    return _grads(theta_k, theta_q, v, phi, dout, dM, M0, True)


def laplace_grads(theta_k, logmag_k, theta_q, logmag_q, v, log_decay, beta, dout, dM=None, M0=None):
    """Gradients of the LaplacePhaseCore recurrence (the token loop of
    ``forward_sequential``, layers.py:563-583, which its chunk loop layers.py:481-561
    equals) with K = exp(logmag_k) e^{i theta_k}, Q likewise, r = exp(log_decay) per
    (token, value row): returns numpy ``(d theta_k, d logmag_k, d theta_q, d logmag_q,
    d v, d log_decay, d beta, d M0 or None)``."""
    names = (theta_k, logmag_k, theta_q, logmag_q, v, log_decay, beta)
    tk, mk, tq, mq, vv, ld, bb = (_t(a) for a in names)
    m0 = None
    if M0 is not None:
        m0 = torch.from_numpy(np.asarray(M0, dtype=np.complex128).copy()).requires_grad_(True)
    B, H, L, D = tk.shape
    Dv = vv.shape[-1]
    K = torch.complex(torch.exp(mk) * torch.cos(tk), torch.exp(mk) * torch.sin(tk))
    Q = torch.complex(torch.exp(mq) * torch.cos(tq), torch.exp(mq) * torch.sin(tq))
    r = torch.exp(ld)
    M = torch.zeros(B, H, Dv, D, dtype=torch.complex128) if m0 is None else m0
    outs = []
    for t in range(L):
        k, q = K[:, :, t], Q[:, :, t]
        v_old = torch.matmul(M, torch.conj(k).unsqueeze(-1)).squeeze(-1).real / D
        err = (vv[:, :, t] - v_old).to(M.dtype)
        M = M * r[:, :, t].unsqueeze(-1) + bb[:, :, t][..., None, None] * torch.matmul(err.unsqueeze(-1),
                                                                                     k.unsqueeze(-2))
        outs.append(torch.matmul(M, torch.conj(q).unsqueeze(-1)).squeeze(-1).real / D)
    out = torch.stack(outs, 2)
    o_list, g_list = [out], [torch.from_numpy(np.asarray(dout, dtype=np.float64))]
    if dM is not None:
        o_list.append(M)
        g_list.append(torch.from_numpy(np.asarray(dM, dtype=np.complex128)))
    inputs = [tk, mk, tq, mq, vv, ld, bb] + ([m0] if m0 is not None else [])
    grads = torch.autograd.grad(o_list, inputs, g_list, allow_unused=True)
    res = [x.detach().numpy() for x in grads[:7]]
    res.append(grads[7].detach().numpy() if m0 is not None else None)
    return tuple(res)
