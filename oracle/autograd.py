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

Both take numpy inputs and the output / final-state gradients (``dout`` (B,H,L,Dv),
``dM`` (B,H,Dv,D) complex or None) and return numpy gradients
``(d theta_k, d theta_q, d v, d beta_or_phi, d M0 or None)`` with PyTorch's complex
convention (dL/dRe + i dL/dIm).  Pinned against gradients of the reference itself in
tests/golden/grad.npz.
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
