"""Functional chunkwise delta-rule core on the B200 CUDA kernels.

Drop-in for ``delta_phase.kernels.triton_chunk_delta`` (mcarbonell/delta-phase v1.3.0):

* :func:`delta_phase_chunkwise_fused` -- same signature and return contract as the
  reference dispatcher (triton_chunk_delta.py:279-291) and ``_chunkwise_delta_reference``
  (:211-252): ``(out (B,H,L,D) real, M (B,H,D,D) complex)``; ``L`` must be a multiple
  of ``chunk_size`` (the reference's ``view`` raises RuntimeError otherwise);
  ``initial_state`` is never modified.
* :class:`DeltaPhaseCudaFunction` (alias ``DeltaPhaseTritonFunction``) -- the autograd
  wrapper: forward on the fused kernels, backward on ``dp_core_bwd`` (the reference's
  Function, :255-276, raises in backward and its dispatcher sends gradient-enabled calls
  to the PyTorch path instead; here both directions run on the GPU kernels).
* :func:`gram_matrix_cuda` (alias ``gram_matrix_triton``) -- the strictly-lower phasor
  Gram of the archived Triton kernel (:32-122).
* :func:`decode_step` -- the fused single-token state update (layers.py:279-285).
* ``complex_beta=True`` on :func:`chunkwise_forward` / :func:`decode_step` -- the
  complex-beta rule of ComplexBetaDeltaPhaseBlock (layers.py:294-418), ``beta`` then
  holding phi of beta = 1 + e^{i phi}; :func:`complex_beta_chunkwise` is its chunkwise
  form over a sequence (the reference's token loop, layers.py:346-360).
* :func:`laplace_chunkwise` -- the LaplacePhaseCore chunk solve (layers.py:481-561);
  differentiable through :class:`LaplaceCudaFunction` (backward on ``dp_laplace_bwd``).
* :func:`triton_available` -- kept for API compatibility; True when the CUDA library
  is loaded and a GPU is present (the kernels it reported on are replaced here).
"""
from __future__ import annotations

import torch

from .. import _capi


def phasor(theta: torch.Tensor) -> torch.Tensor:
    """exp(i theta) as complex64 (layers.py:203-206 / triton_chunk_delta.py:220-221)."""
    _capi.require_cuda(theta)
    if theta.dtype == torch.float64:
        raise TypeError("float64 inputs are not supported by the CUDA path")
    out = torch.empty(theta.shape, device=theta.device, dtype=torch.complex64)
    _capi.phasor(theta, out)
    return out


def cuda_available() -> bool:
    """True if the deltaphase_b200 library loads and a CUDA device is present."""
    return torch.cuda.is_available() and _capi.library_available()


def triton_available() -> bool:
    """Reference name (triton_chunk_delta.py:21-23): reports whether the fused GPU path
    can run.  Here that path is the sm_100a CUDA library, not Triton."""
    return cuda_available()


def _check_phase_inputs(theta_k, theta_q, v, beta):
    if theta_k.dim() != 4 or theta_q.shape != theta_k.shape:
        raise ValueError("theta_k and theta_q must both be (B, H, L, D)")
    if v.dim() != 4 or v.shape[:3] != theta_k.shape[:3]:
        raise ValueError("v must be (B, H, L, Dv)")
    if beta.shape != theta_k.shape[:3]:
        raise ValueError("beta must be (B, H, L)")
    if theta_k.dtype == torch.float64 or v.dtype == torch.float64:
        raise TypeError("float64 inputs are not supported by the CUDA path")
    if not (theta_k.dtype == theta_q.dtype == v.dtype):
        raise TypeError("theta_k, theta_q and v must share one dtype")


def _complex_state_view(state, B, H, Dv, D, device):
    """float32 (B,H,Dv,D,2) contiguous view of a complex64 state (copied if needed)."""
    if state is None:
        return None
    if not torch.is_complex(state):
        raise TypeError("the delta-rule state must be a complex tensor")
    if state.dtype != torch.complex64:
        raise TypeError("the CUDA path keeps the state in complex64")
    if tuple(state.shape) != (B, H, Dv, D):
        raise ValueError(f"state must be (B, H, Dv, D) = {(B, H, Dv, D)}, got {tuple(state.shape)}")
    if state.device != device:
        raise RuntimeError("state must be on the same device as the inputs")
    return torch.view_as_real(state.contiguous())


def chunkwise_forward(theta_k, theta_q, v, beta, chunk_size=64, initial_state=None, out=None,
                      complex_beta=False):
    """Run the CUDA chunkwise core; ragged L is allowed (tokens past L do not exist).

    ``out`` may be a preallocated float32 (B, H, L, Dv) view (any strides with unit
    channel stride), e.g. a (B, L, H, Dv) buffer transposed.  ``complex_beta``: ``beta``
    holds phi and the write strength is 1 + e^{i phi}.  Returns ``(out, M)``.
    """
    _check_phase_inputs(theta_k, theta_q, v, beta)
    _capi.require_cuda(theta_k, theta_q, v, beta)
    B, H, L, D = theta_k.shape
    Dv = v.shape[-1]
    dev = theta_k.device
    s_in = _complex_state_view(initial_state, B, H, Dv, D, dev)
    if out is None:
        out = torch.empty(B, H, L, Dv, device=dev, dtype=torch.float32)
    M = torch.empty(B, H, Dv, D, device=dev, dtype=torch.complex64)
    _capi.core_fwd(theta_k, theta_q, v, beta, chunk_size, s_in, out, torch.view_as_real(M),
                   complex_beta=complex_beta)
    return out, M


def complex_beta_chunkwise(theta_k, theta_q, v, phi, initial_state=None):
    """Complex-beta delta rule over a sequence: the chunkwise (WY) form of the token loop
    of ComplexBetaDeltaPhaseBlock.forward (layers.py:346-360), beta = 1 + e^{i phi}.

    theta_k, theta_q, v: (B, H, L, D); phi (B, H, L); initial_state (B, H, D, D)
    complex64 or None (never modified).  Any L.  Returns ``(out (B,H,L,D) float32,
    M (B,H,D,D) complex64)``.
    """
    if torch.is_grad_enabled() and any(
            t is not None and t.requires_grad for t in (theta_k, theta_q, v, phi, initial_state)):
        return DeltaPhaseCudaFunction.apply(theta_k, theta_q, v, phi, 64, initial_state, True)
    with torch.no_grad():
        return chunkwise_forward(theta_k, theta_q, v, phi, 64, initial_state, complex_beta=True)


class DeltaPhaseCudaFunction(torch.autograd.Function):
    """Autograd wrapper of the chunkwise core: forward on dp_core_fwd (dp_core_cbeta_fwd
    when ``complex_beta``), backward on dp_core_bwd, which returns the gradients of
    theta_k, theta_q, v, beta (phi) and the initial state in the inputs' dtypes.  Same
    call signature as the reference's DeltaPhaseTritonFunction (triton_chunk_delta.py:
    255-276), whose backward raises; ``complex_beta`` is an extra trailing argument."""

    @staticmethod
    def forward(ctx, theta_k, theta_q, v, beta, chunk_size=64, initial_state=None, complex_beta=False):
        out, M = chunkwise_forward(theta_k, theta_q, v, beta, chunk_size, initial_state,
                                   complex_beta=complex_beta)
        ctx.save_for_backward(theta_k, theta_q, v, beta, initial_state)
        ctx.complex_beta = bool(complex_beta)
        return out, M

    @staticmethod
    def backward(ctx, grad_out, grad_final_state):
        tk, tq, v, beta, M0 = ctx.saved_tensors
        B, H, L, D = tk.shape
        Dv = v.shape[-1]
        dev = tk.device
        go = (torch.zeros(B, H, L, Dv, device=dev, dtype=torch.float32) if grad_out is None
              else grad_out.to(torch.float32).contiguous())
        gM = (None if grad_final_state is None
              else torch.view_as_real(grad_final_state.to(torch.complex64).contiguous()))
        s_in = None if M0 is None else torch.view_as_real(M0.detach().to(torch.complex64).contiguous())
        f32 = dict(device=dev, dtype=torch.float32)
        dtk, dtq = torch.empty(B, H, L, D, **f32), torch.empty(B, H, L, D, **f32)
        dv, db = torch.empty(B, H, L, Dv, **f32), torch.empty(B, H, L, **f32)
        need_m0 = M0 is not None and ctx.needs_input_grad[5]
        dM0 = torch.empty(B, H, Dv, D, device=dev, dtype=torch.complex64) if need_m0 else None
        _capi.core_bwd(tk, tq, v, beta, s_in, go, gM, dtk, dtq, dv, db,
                       None if dM0 is None else torch.view_as_real(dM0), complex_beta=ctx.complex_beta)
        return (dtk.to(tk.dtype), dtq.to(tq.dtype), dv.to(v.dtype), db.to(beta.dtype), None,
                None if dM0 is None else dM0.to(M0.dtype), None)


DeltaPhaseTritonFunction = DeltaPhaseCudaFunction


def delta_phase_chunkwise_fused(theta_k, theta_q, v, beta, chunk_size=64, initial_state=None):
    """Chunkwise complex delta-rule forward (reference: triton_chunk_delta.py:279-291).

    theta_k, theta_q, v: (B, H, L, D) float32/bfloat16/float16 CUDA tensors; beta (B, H, L);
    initial_state: (B, H, D, D) complex64 or None.  Returns ``(out (B,H,L,D) float32,
    M (B,H,D,D) complex64)``.  L must be a multiple of chunk_size, as in the reference.
    """
    L = theta_k.shape[2]
    if chunk_size < 1 or L % chunk_size != 0:
        raise RuntimeError(
            f"shape mismatch: L={L} is not a multiple of chunk_size={chunk_size}")
    if torch.is_grad_enabled() and any(
            t is not None and t.requires_grad for t in (theta_k, theta_q, v, beta, initial_state)):
        return DeltaPhaseCudaFunction.apply(theta_k, theta_q, v, beta, chunk_size, initial_state)
    with torch.no_grad():
        return chunkwise_forward(theta_k, theta_q, v, beta, chunk_size, initial_state)


def gram_matrix_cuda(theta_k: torch.Tensor, beta: torch.Tensor) -> torch.Tensor:
    """Strictly-lower row-beta-scaled phasor Gram (N, C, C) float32
    (contract of gram_matrix_reference, triton_chunk_delta.py:192-208)."""
    if theta_k.dim() != 3 or beta.shape != theta_k.shape[:2]:
        raise ValueError("theta_k must be (N, C, D) and beta (N, C)")
    _capi.require_cuda(theta_k, beta)
    th = theta_k.contiguous()
    b = beta.contiguous()
    N, C, _ = th.shape
    out = torch.empty(N, C, C, device=th.device, dtype=torch.float32)
    _capi.gram(th, b, out)
    return out


gram_matrix_triton = gram_matrix_cuda


def decode_step(memory_state, theta_k, theta_q, v, beta, out=None, state_out=None, complex_beta=False,
                gate_mode=None):
    """Fused decode step (layers.py:279-285).  memory_state (B,H,Dv,D) complex64;
    theta_k/theta_q (B,H,D); v (B,H,Dv); beta (B,H).  Returns ``(out (B,H,Dv) float32,
    new_state)``.  ``state_out=memory_state`` updates the state in place.
    ``complex_beta``: ``beta`` holds phi, the step of ComplexBetaDeltaPhaseBlock
    (layers.py:402-407).  ``gate_mode`` (``_capi.DP_GATE_*``): ``beta`` is the write
    gate's raw projection and the kernel forms beta from it (2 sigmoid(g), 1, or
    1 + e^{i g})."""
    B, H, D = theta_k.shape
    Dv = v.shape[-1]
    _capi.require_cuda(memory_state, theta_k, theta_q, v, beta)
    s_in = _complex_state_view(memory_state, B, H, Dv, D, theta_k.device)
    if state_out is None:
        state_out = torch.empty(B, H, Dv, D, device=theta_k.device, dtype=torch.complex64)
    elif state_out.dtype != torch.complex64 or not state_out.is_contiguous():
        raise ValueError("state_out must be a contiguous complex64 tensor")
    if out is None:
        out = torch.empty(B, H, Dv, device=theta_k.device, dtype=torch.float32)
    _capi.core_decode(s_in, torch.view_as_real(state_out), theta_k, theta_q, v, beta, out,
                      complex_beta=complex_beta, gate_mode=gate_mode)
    return out, state_out


class LaplaceCudaFunction(torch.autograd.Function):
    """Autograd wrapper of the Laplace core: forward on dp_laplace_fwd, backward on
    dp_laplace_bwd (gradients of every input in its own dtype; None for absent
    log-magnitudes)."""

    @staticmethod
    def forward(ctx, theta_k, logmag_k, theta_q, logmag_q, v, log_decay, beta, chunk_size=32, initial_state=None):
        out, M = _laplace_forward(theta_k, logmag_k, theta_q, logmag_q, v, log_decay, beta, chunk_size,
                                  initial_state, None)
        ctx.save_for_backward(theta_k, logmag_k, theta_q, logmag_q, v, log_decay, beta, initial_state)
        return out, M

    @staticmethod
    def backward(ctx, grad_out, grad_final_state):
        tk, mk, tq, mq, v, ld, beta, M0 = ctx.saved_tensors
        B, H, L, D = tk.shape
        Dv = v.shape[-1]
        dev = tk.device
        f32 = dict(device=dev, dtype=torch.float32)
        go = (torch.zeros(B, H, L, Dv, **f32) if grad_out is None else grad_out.to(torch.float32).contiguous())
        gM = (None if grad_final_state is None
              else torch.view_as_real(grad_final_state.to(torch.complex64).contiguous()))
        s_in = None if M0 is None else torch.view_as_real(M0.detach().to(torch.complex64).contiguous())
        grads = (torch.empty(B, H, L, D, **f32), torch.empty(B, H, L, D, **f32), torch.empty(B, H, L, D, **f32),
                 torch.empty(B, H, L, D, **f32), torch.empty(B, H, L, Dv, **f32), torch.empty(B, H, L, Dv, **f32),
                 torch.empty(B, H, L, **f32))
        need_m0 = M0 is not None and ctx.needs_input_grad[8]
        dM0 = torch.empty(B, H, Dv, D, device=dev, dtype=torch.complex64) if need_m0 else None
        _capi.laplace_bwd(tk, mk, tq, mq, v, ld, beta, s_in, go, gM, grads,
                          None if dM0 is None else torch.view_as_real(dM0))
        like = (tk, mk, tq, mq, v, ld, beta)
        res = [None if x is None else g.to(x.dtype) for g, x in zip(grads, like)]
        return (*res, None, None if dM0 is None else dM0.to(M0.dtype))


def laplace_chunkwise(theta_k, logmag_k, theta_q, logmag_q, v, log_decay, beta, chunk_size=32,
                      initial_state=None, out=None):
    """LaplacePhaseCore chunk solve (layers.py:481-561) on the CUDA kernel.

    K = exp(logmag_k) e^{i theta_k}, Q = exp(logmag_q) e^{i theta_q} ((B,H,L,D); the
    log-magnitudes may be None = unit phasors); log_decay (B,H,L,Dv) is log r per value
    channel (clamped at -80 per step like the reference); beta (B,H,L).
    Returns ``(out (B,H,L,Dv) float32, M (B,H,Dv,D) complex64)``.  Differentiable (through
    LaplaceCudaFunction) when autograd records and an input requires grad; ``out`` must
    then be None.
    """
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in (
            theta_k, logmag_k, theta_q, logmag_q, v, log_decay, beta, initial_state)):
        if out is not None:
            raise ValueError("out= is not supported when gradients are recorded")
        return LaplaceCudaFunction.apply(theta_k, logmag_k, theta_q, logmag_q, v, log_decay, beta, chunk_size,
                                         initial_state)
    return _laplace_forward(theta_k, logmag_k, theta_q, logmag_q, v, log_decay, beta, chunk_size, initial_state,
                            out)


def _laplace_forward(theta_k, logmag_k, theta_q, logmag_q, v, log_decay, beta, chunk_size, initial_state, out):
    B, H, L, D = theta_k.shape
    Dv = v.shape[-1]
    _capi.require_cuda(theta_k, theta_q, v, log_decay, beta)
    for t in (logmag_k, logmag_q):
        if t is not None and t.shape != theta_k.shape:
            raise ValueError("log-magnitudes must match theta's shape")
    if log_decay.shape != v.shape:
        raise ValueError("log_decay must be (B, H, L, Dv)")
    dt = theta_k.dtype
    for t in (theta_q, v, log_decay, logmag_k, logmag_q):
        if t is not None and t.dtype != dt:
            raise TypeError("phase, magnitude, value and decay inputs must share one dtype")
    if dt == torch.float64:
        raise TypeError("float64 inputs are not supported by the CUDA path")
    s_in = _complex_state_view(initial_state, B, H, Dv, D, theta_k.device)
    if out is None:
        out = torch.empty(B, H, L, Dv, device=theta_k.device, dtype=torch.float32)
    M = torch.empty(B, H, Dv, D, device=theta_k.device, dtype=torch.complex64)
    _capi.laplace_fwd(theta_k, logmag_k, theta_q, logmag_q, v, log_decay, beta, chunk_size, s_in,
                      out, torch.view_as_real(M))
    return out, M
