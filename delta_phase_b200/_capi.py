"""ctypes binding of the deltaphase_b200 C ABI (include/deltaphase_b200.h).

torch is used only for device memory, the current stream and dtype bookkeeping; every
computation on the hot path runs in the CUDA library.  There is no CPU fallback: if
the library is missing or a tensor is not on a CUDA device, these functions raise.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libdeltaphase_b200.so")

DP_F32, DP_BF16, DP_F16 = 0, 1, 2
_DTYPE_CODES = {torch.float32: DP_F32, torch.bfloat16: DP_BF16, torch.float16: DP_F16}

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64P = ctypes.POINTER(ctypes.c_int64)
_SIG = {
    "dp_version": (ctypes.c_char_p, []),
    "dp_last_error": (ctypes.c_char_p, []),
    "dp_status_string": (ctypes.c_char_p, [_I]),
    "dp_device_error": (_I, [_I]),
    "dp_core_fwd": (_I, [_P, _P, _P, _P, _I, _I, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I64P, _P]),
    "dp_core_decode": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _P, _I, _I, _I, _I, _I64P, _P]),
    "dp_core_cbeta_fwd": (_I, [_P, _P, _P, _P, _I, _I, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I64P, _P]),
    "dp_core_cbeta_decode": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _P, _I, _I, _I, _I, _I64P, _P]),
    "dp_core_decode_gated": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _P, _I, _I, _I, _I, _I64P, _P]),
    "dp_core_bwd_workspace_size": (ctypes.c_size_t, [_I, _I, _I, _I]),
    "dp_core_bwd": (_I, [_P, _P, _P, _P, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I64P,
                         _P, ctypes.c_size_t, _P]),
    "dp_gram": (_I, [_P, _P, _I, _I, _P, _I, _I, _I, _P]),
    "dp_phasor": (_I, [_P, _I, ctypes.c_int64, _P, _P]),
    "dp_laplace_fwd": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I, _P, _P, _P, _I, _I, _I, _I, _I,
                            _I, _I64P, _P]),
    "dp_laplace_bwd_workspace_size": (ctypes.c_size_t, [_I, _I, _I, _I, _I]),
    "dp_laplace_bwd": (_I, [_P] * 7 + [_I, _I] + [_P] * 11 + [_I] * 5 + [_I64P, _P, ctypes.c_size_t, _P]),
    "dp_ffn_fold": (_I, [_P, _P, _P, _P, _P, _I, _I, _P]),
    "dp_ffn_workspace_size": (ctypes.c_size_t, [_I, _I, _I]),
    "dp_ffn_fwd": (_I, [_P, _I, _P, _P, _P, _I, _I, _P, ctypes.c_size_t, _P]),
    "dp_ffn_fwd_residual": (_I, [_P, _I, _P, _P, _P, _I, _I, _P, ctypes.c_size_t, _P]),
    "dp_ffn_features": (_I, [_P, _I, _P, _P, _I, _I, _P]),
    "dp_gemm_skinny": (_I, [_P, ctypes.c_int64, _P, _P, _I, _P, _I, ctypes.c_int64, _I, _I, _I, _I, _P]),
    "dp_ffn_fwd_noalloc": (_I, [_P, _I, _P, _P, _P, _I, _I, _P]),
    "dp_ffn_noalloc_max_tokens": (ctypes.c_size_t, [_I, _I]),
    "dp_ln_conv_silu": (_I, [_P, _I, _P, _P, ctypes.c_float, _P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "dp_ln_conv_step": (_I, [_P, _I, _P, _P, ctypes.c_float, _P, _P, _P, _P, _I, _I, _I, _I, _P]),
    "dp_layernorm": (_I, [_P, _I, _P, _P, _P, ctypes.c_float, _P, _P, _I, ctypes.c_int64, _I, _P]),
}

_lib = None
_lock = threading.Lock()


class DeltaPhaseCudaError(RuntimeError):
    """A deltaphase_b200 entry point returned a non-zero status."""

    def __init__(self, fn, status, msg):
        super().__init__(f"{fn} failed with status {status}: {msg}")
        self.status = status


def lib():
    """Load the CUDA library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"deltaphase_b200 CUDA library not found at {LIB_PATH}; build it with "
                        "`python -m delta_phase_b200.build` (nvcc, sm_100a)")
                L = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in _SIG.items():
                    f = getattr(L, name)
                    f.restype = res
                    f.argtypes = args
                _lib = L
    return _lib


def exported_symbols():
    return list(_SIG)


def version():
    return lib().dp_version().decode()


def device_error(clear=True):
    """Synchronise the current device and return (optionally clear) the device-side
    error word: 0, or 5 (DP_ERR_TIMEOUT) if a kernel's bounded wait expired."""
    return int(lib().dp_device_error(1 if clear else 0))


def library_available():
    try:
        lib()
        return True
    except (RuntimeError, OSError):
        return False


def _check(fn, status):
    if status != 0:
        L = lib()
        msg = L.dp_last_error().decode()
        if status == 1:
            raise ValueError(f"{fn}: {msg}")
        raise DeltaPhaseCudaError(fn, status, msg)


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPE_CODES[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype} (the CUDA path takes float32, bfloat16 "
                        "or float16; float64 is not supported)") from None


def require_cuda(*tensors):
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("deltaphase_b200 kernels require CUDA tensors")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError("all tensors must be on the same CUDA device")
    return dev


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def strides_array(values):
    arr = (ctypes.c_int64 * len(values))(*[int(x) for x in values])
    return arr


def seq_strides(t: torch.Tensor):
    """(sb, sh, st) of a (B, H, L, C) view with unit channel stride."""
    if t.dim() != 4:
        raise ValueError("expected a 4-D (B, H, L, C) tensor")
    if t.shape[-1] > 1 and t.stride(-1) != 1:
        raise ValueError("the channel dimension must have unit stride")
    return t.stride(0), t.stride(1), t.stride(2)


def core_fwd(theta_k, theta_q, v, beta, chunk_size, state_in, out, state_out, complex_beta=False):
    """dp_core_fwd on (B,H,L,D) views.  state_in/state_out are float32 views of the
    interleaved complex64 state (B,H,Dv,D,2), contiguous.  complex_beta: ``beta`` holds
    phi of beta = 1 + e^{i phi} (dp_core_cbeta_fwd)."""
    dev = require_cuda(theta_k, theta_q, v, beta, state_in, out, state_out)
    B, H, L, D = theta_k.shape
    Dv = v.shape[-1]
    st = []
    for t in (theta_k, theta_q, v):
        st += seq_strides(t)
    st += (beta.stride(0), beta.stride(1), beta.stride(2))
    st += seq_strides(out)
    arr = strides_array(st)
    name = "dp_core_cbeta_fwd" if complex_beta else "dp_core_fwd"
    with torch.cuda.device(dev):
        rc = getattr(lib(), name)(ptr(theta_k), ptr(theta_q), ptr(v), ptr(beta), dtype_code(theta_k),
                                  dtype_code(beta), ptr(state_in), ptr(out), ptr(state_out), B, H, L, D,
                                  Dv, int(chunk_size), arr, stream_of(dev))
    _check(name, rc)


DP_GATE_BETA, DP_GATE_SIGMOID2, DP_GATE_ONE, DP_GATE_PHI = 0, 1, 2, 3


def core_decode(state_in, state_out, theta_k, theta_q, v, beta, out, complex_beta=False, gate_mode=None):
    """dp_core_decode; theta_k/theta_q (B,H,D), v (B,H,Dv), beta (B,H), out (B,H,Dv).
    complex_beta: ``beta`` holds phi of beta = 1 + e^{i phi} (dp_core_cbeta_decode).
    gate_mode (one of DP_GATE_*): ``beta`` is the raw gate that dp_core_decode_gated maps
    to the write strength itself."""
    dev = require_cuda(state_in, state_out, theta_k, theta_q, v, beta, out)
    B, H, D = theta_k.shape
    Dv = v.shape[-1]
    for t in (theta_k, theta_q, v, out):
        if t.shape[-1] > 1 and t.stride(-1) != 1:
            raise ValueError("the channel dimension must have unit stride")
    st = []
    for t in (theta_k, theta_q, v, beta, out):
        st += (t.stride(0), t.stride(1))
    with torch.cuda.device(dev):
        if gate_mode is not None:
            name = "dp_core_decode_gated"
            rc = lib().dp_core_decode_gated(ptr(state_in), ptr(state_out), ptr(theta_k), ptr(theta_q), ptr(v),
                                            ptr(beta), dtype_code(theta_k), dtype_code(beta), int(gate_mode),
                                            ptr(out), B, H, D, Dv, strides_array(st), stream_of(dev))
        else:
            name = "dp_core_cbeta_decode" if complex_beta else "dp_core_decode"
            rc = getattr(lib(), name)(ptr(state_in), ptr(state_out), ptr(theta_k), ptr(theta_q), ptr(v),
                                      ptr(beta), dtype_code(theta_k), dtype_code(beta), ptr(out), B, H, D,
                                      Dv, strides_array(st), stream_of(dev))
    _check(name, rc)


def core_bwd(theta_k, theta_q, v, beta, state_in, grad_out, grad_state_out, grad_theta_k, grad_theta_q,
             grad_v, grad_beta, grad_state_in, complex_beta=False):
    """dp_core_bwd.  theta_k/theta_q/v/beta as core_fwd; state tensors are float32 views of
    complex64 states (B,H,Dv,D,2) or None; gradient outputs float32 contiguous."""
    dev = require_cuda(theta_k, theta_q, v, beta, grad_out, grad_theta_k, grad_theta_q, grad_v, grad_beta)
    B, H, L, D = theta_k.shape
    Dv = v.shape[-1]
    for t in (grad_out, grad_theta_k, grad_theta_q, grad_v, grad_beta):
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise ValueError("gradient tensors must be contiguous float32")
    st = []
    for t in (theta_k, theta_q, v):
        st += seq_strides(t)
    st += (beta.stride(0), beta.stride(1), beta.stride(2))
    ws = torch.empty(max(1, int(lib().dp_core_bwd_workspace_size(B, H, L, Dv))), device=dev, dtype=torch.uint8)
    with torch.cuda.device(dev):
        rc = lib().dp_core_bwd(ptr(theta_k), ptr(theta_q), ptr(v), ptr(beta), dtype_code(theta_k), dtype_code(beta),
                               1 if complex_beta else 0, ptr(state_in), ptr(grad_out), ptr(grad_state_out),
                               ptr(grad_theta_k), ptr(grad_theta_q), ptr(grad_v), ptr(grad_beta), ptr(grad_state_in),
                               B, H, L, D, Dv, strides_array(st), ptr(ws), ws.numel(), stream_of(dev))
    _check("dp_core_bwd", rc)


def gram(theta, beta, out):
    dev = require_cuda(theta, beta, out)
    N, C, D = theta.shape
    with torch.cuda.device(dev):
        rc = lib().dp_gram(ptr(theta), ptr(beta), dtype_code(theta), dtype_code(beta), ptr(out), N, C,
                           D, stream_of(dev))
    _check("dp_gram", rc)


def phasor(theta, out):
    """dp_phasor: out (complex64, same shape as theta) = exp(i theta)."""
    dev = require_cuda(theta, out)
    th = theta.contiguous()
    with torch.cuda.device(dev):
        rc = lib().dp_phasor(ptr(th), dtype_code(th), th.numel(), ptr(torch.view_as_real(out)),
                             stream_of(dev))
    _check("dp_phasor", rc)


def laplace_fwd(theta_k, logmag_k, theta_q, logmag_q, v, log_decay, beta, chunk_size, state_in,
                out, state_out):
    dev = require_cuda(theta_k, logmag_k, theta_q, logmag_q, v, log_decay, beta, state_in, out,
                       state_out)
    B, H, L, D = theta_k.shape
    Dv = v.shape[-1]
    st = []
    for t in (theta_k, logmag_k, theta_q, logmag_q, v, log_decay):
        st += (0, 0, 0) if t is None else seq_strides(t)
    st += (beta.stride(0), beta.stride(1), beta.stride(2))
    st += seq_strides(out)
    with torch.cuda.device(dev):
        rc = lib().dp_laplace_fwd(ptr(theta_k), ptr(logmag_k), ptr(theta_q), ptr(logmag_q), ptr(v),
                                  ptr(log_decay), ptr(beta), dtype_code(theta_k), dtype_code(beta),
                                  ptr(state_in), ptr(out), ptr(state_out), B, H, L, D, Dv,
                                  int(chunk_size), strides_array(st), stream_of(dev))
    _check("dp_laplace_fwd", rc)


def laplace_bwd(theta_k, logmag_k, theta_q, logmag_q, v, log_decay, beta, state_in, grad_out, grad_state_out,
                grads, grad_state_in):
    """dp_laplace_bwd.  ``grads`` = (theta_k, logmag_k, theta_q, logmag_q, v, log_decay, beta)
    gradient outputs, float32 contiguous; state tensors are float32 views of complex64
    states or None."""
    dev = require_cuda(theta_k, theta_q, v, log_decay, beta, grad_out, *grads)
    B, H, L, D = theta_k.shape
    Dv = v.shape[-1]
    for t in (grad_out,) + tuple(grads):
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise ValueError("gradient tensors must be contiguous float32")
    st = []
    for t in (theta_k, logmag_k, theta_q, logmag_q, v, log_decay):
        st += (0, 0, 0) if t is None else seq_strides(t)
    st += (beta.stride(0), beta.stride(1), beta.stride(2))
    ws = torch.empty(max(1, int(lib().dp_laplace_bwd_workspace_size(B, H, L, D, Dv))), device=dev, dtype=torch.uint8)
    with torch.cuda.device(dev):
        rc = lib().dp_laplace_bwd(ptr(theta_k), ptr(logmag_k), ptr(theta_q), ptr(logmag_q), ptr(v), ptr(log_decay),
                                  ptr(beta), dtype_code(theta_k), dtype_code(beta), ptr(state_in), ptr(grad_out),
                                  ptr(grad_state_out), *[ptr(g) for g in grads], ptr(grad_state_in), B, H, L, D, Dv,
                                  strides_array(st), ptr(ws), ws.numel(), stream_of(dev))
    _check("dp_laplace_bwd", rc)


def ffn_fold(logits, mats, banks, combine, F, d, nb):
    dev = require_cuda(logits, mats, banks, combine, F)
    with torch.cuda.device(dev):
        rc = lib().dp_ffn_fold(ptr(logits), ptr(mats), ptr(banks), ptr(combine), ptr(F), d, nb,
                               stream_of(dev))
    _check("dp_ffn_fold", rc)


def ffn_workspace_size(tokens, d, dtype):
    return int(lib().dp_ffn_workspace_size(tokens, d, _DTYPE_CODES[dtype]))


def ffn_fwd(x, dct, F, y, workspace):
    dev = require_cuda(x, dct, F, y, workspace)
    tokens, d = x.shape
    with torch.cuda.device(dev):
        rc = lib().dp_ffn_fwd(ptr(x), dtype_code(x), ptr(dct), ptr(F), ptr(y), tokens, d,
                              ptr(workspace), workspace.numel() * workspace.element_size(),
                              stream_of(dev))
    _check("dp_ffn_fwd", rc)


def ffn_fwd_residual(x, dct, F, y, workspace):
    """dp_ffn_fwd_residual: y (tokens, d) float32 += FFN(x)."""
    dev = require_cuda(x, dct, F, y, workspace)
    tokens, d = x.shape
    if y.dtype != torch.float32 or not y.is_contiguous() or tuple(y.shape) != (tokens, d):
        raise ValueError("y must be a contiguous float32 (tokens, d) tensor")
    with torch.cuda.device(dev):
        rc = lib().dp_ffn_fwd_residual(ptr(x), dtype_code(x), ptr(dct), ptr(F), ptr(y), tokens, d,
                                       ptr(workspace), workspace.numel() * workspace.element_size(),
                                       stream_of(dev))
    _check("dp_ffn_fwd_residual", rc)


def ffn_features(x, hdct, z):
    """dp_ffn_features: z (tokens, 6d) from x (tokens, d) and hdct = x mat_dct^T (float32)."""
    dev = require_cuda(x, hdct, z)
    tokens, d = x.shape
    for t in (x, hdct, z):
        if not t.is_contiguous():
            raise ValueError("dp_ffn_features takes contiguous tensors")
    if hdct.dtype != torch.float32 or z.dtype != x.dtype or tuple(z.shape) != (tokens, 6 * d):
        raise ValueError("hdct must be float32 (tokens, d) and z (tokens, 6d) of x's dtype")
    with torch.cuda.device(dev):
        rc = lib().dp_ffn_features(ptr(x), dtype_code(x), ptr(hdct), ptr(z), tokens, d, stream_of(dev))
    _check("dp_ffn_features", rc)


SKINNY_MAX_ROWS = 16


def gemm_skinny(x, w, bias, y, accumulate=False):
    """dp_gemm_skinny: y (M, N) = x (M, K) w^T (+ bias) (+ y); x, w bf16, M <= 16."""
    dev = require_cuda(x, w, y)
    M, K = x.shape
    N = w.shape[0]
    if x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
        raise ValueError("dp_gemm_skinny takes bf16 x and w")
    if x.stride(1) != 1 or not w.is_contiguous() or y.stride(1) != 1 or tuple(y.shape) != (M, N):
        raise ValueError("x, y need unit column stride, w must be contiguous (N, K)")
    with torch.cuda.device(dev):
        rc = lib().dp_gemm_skinny(ptr(x), x.stride(0), ptr(w), None if bias is None else ptr(bias),
                                  DP_F32 if bias is None else dtype_code(bias), ptr(y), dtype_code(y),
                                  y.stride(0), int(bool(accumulate)), M, N, K, stream_of(dev))
    _check("dp_gemm_skinny", rc)


def ffn_fwd_noalloc(x, dct, F, y):
    """dp_ffn_fwd_noalloc: the FFN forward with the library's fixed device scratch
    instead of a workspace (for callers that cannot allocate; see the header)."""
    dev = require_cuda(x, dct, F, y)
    tokens, d = x.shape
    with torch.cuda.device(dev):
        rc = lib().dp_ffn_fwd_noalloc(ptr(x), dtype_code(x), ptr(dct), ptr(F), ptr(y), tokens, d,
                                      stream_of(dev))
    _check("dp_ffn_fwd_noalloc", rc)


def ffn_noalloc_max_tokens(d, dtype):
    return int(lib().dp_ffn_noalloc_max_tokens(d, _DTYPE_CODES[dtype]))


def ln_conv_silu(x, ln_w, ln_b, eps, conv_w, conv_b, out):
    """dp_ln_conv_silu: out = n + SiLU(causal depthwise conv(n)), n = LayerNorm(x); x, out
    (B, L, d) contiguous; conv_w (d, k) float32."""
    dev = require_cuda(x, ln_w, ln_b, conv_w, out)
    B, L, d = x.shape
    k = conv_w.shape[-1]
    with torch.cuda.device(dev):
        rc = lib().dp_ln_conv_silu(ptr(x), dtype_code(x), ptr(ln_w), ptr(ln_b), float(eps), ptr(conv_w),
                                   ptr(conv_b) if conv_b is not None else None, ptr(out), dtype_code(out),
                                   B, L, d, k, stream_of(dev))
    _check("dp_ln_conv_silu", rc)


def layernorm(x, ln_w, ln_b, eps, y, residual=None, sum_out=None):
    """dp_layernorm: s = x (+ residual) (written to sum_out if given); y = LayerNorm(s).
    x, y, residual, sum_out are (rows, d) contiguous."""
    dev = require_cuda(x, ln_w, ln_b, y)
    rows, d = x.shape
    with torch.cuda.device(dev):
        rc = lib().dp_layernorm(ptr(x), dtype_code(x), ptr(residual) if residual is not None else None,
                                ptr(ln_w), ptr(ln_b), float(eps), ptr(sum_out) if sum_out is not None else None,
                                ptr(y), dtype_code(y), rows, d, stream_of(dev))
    _check("dp_layernorm", rc)


def ln_conv_step(x, ln_w, ln_b, eps, conv_w, conv_b, conv_state, out):
    """dp_ln_conv_step: one decode token; x, out (B, d) contiguous; conv_state (B, d, k-1)
    float32 contiguous, updated in place."""
    dev = require_cuda(x, ln_w, ln_b, conv_w, conv_state, out)
    B, d = x.shape
    k = conv_w.shape[-1]
    if conv_state.dtype != torch.float32 or not conv_state.is_contiguous() or \
            tuple(conv_state.shape) != (B, d, k - 1):
        raise ValueError(f"conv_state must be a contiguous float32 ({B}, {d}, {k - 1}) tensor")
    with torch.cuda.device(dev):
        rc = lib().dp_ln_conv_step(ptr(x), dtype_code(x), ptr(ln_w), ptr(ln_b), float(eps), ptr(conv_w),
                                   ptr(conv_b) if conv_b is not None else None, ptr(conv_state), ptr(out),
                                   dtype_code(out), B, d, k, stream_of(dev))
    _check("dp_ln_conv_step", rc)
