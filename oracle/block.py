"""Oracle (test infrastructure): the DeltaPhaseHolographicBlock glue in numpy.

Reference: mcarbonell/delta-phase v1.3.0, delta_phase/layers.py.

* :func:`block_forward` -- ``DeltaPhaseHolographicBlock.forward`` (layers.py:177-244)
* :func:`block_step`    -- ``DeltaPhaseHolographicBlock.step``    (layers.py:246-291)
* :func:`cb_block_forward`, :func:`cb_block_step` -- ``ComplexBetaDeltaPhaseBlock``
  forward / step (layers.py:324-418)

Parameters are a dict keyed by the reference ``state_dict`` names (norm1.weight,
causal_conv.conv.weight, w_k.weight, ..., ffn.combine.weight, ffn.mat_dct, ...).
The core and FFN are the oracle functions of :mod:`oracle.core` and
:mod:`oracle.spectral`.
"""
from __future__ import annotations

import numpy as np

from . import core, spectral


def _p(params, name, dtype):
    return np.asarray(params[name], dtype=dtype)


def layer_norm(x, w, b, eps=1e-5):
    mu = x.mean(-1, keepdims=True)
    var = ((x - mu) ** 2).mean(-1, keepdims=True)
    return (x - mu) / np.sqrt(var + eps) * w + b


def silu(x):
    return x / (1.0 + np.exp(-x))


def linear(x, params, name, dtype):
    y = x @ _p(params, f"{name}.weight", dtype).T
    bname = f"{name}.bias"
    if bname in params:
        y = y + _p(params, bname, dtype)
    return y


def causal_conv(x, params, dtype):
    """``ShortCausalConv1D.forward`` (layers.py:74-78): depthwise causal conv,
    SiLU, residual.  conv weight (d, 1, k), bias (d,)."""
    w = _p(params, "causal_conv.conv.weight", dtype)[:, 0, :]     # (d, k)
    bias = _p(params, "causal_conv.conv.bias", dtype)
    B, L, d = x.shape
    k = w.shape[-1]
    xp = np.concatenate([np.zeros((B, k - 1, d), dtype), x], 1)
    out = np.zeros_like(x) + bias
    for j in range(k):
        out = out + xp[:, j:j + L, :] * w[:, j]
    return x + silu(out)


def causal_conv_step(x_t, conv_state, params, dtype):
    """``ShortCausalConv1D.step`` (layers.py:80-88).  conv_state (B, d, k-1)."""
    w = _p(params, "causal_conv.conv.weight", dtype)[:, 0, :]
    bias = _p(params, "causal_conv.conv.bias", dtype)
    B, _, d = x_t.shape
    k = w.shape[-1]
    if conv_state is None:
        conv_state = np.zeros((B, d, k - 1), dtype)
    inputs = np.concatenate([conv_state, np.swapaxes(x_t, 1, 2)], 2)   # (B, d, k)
    new_state = inputs[:, :, 1:]
    conv = (inputs * w[None]).sum(-1) + bias
    return x_t + silu(conv)[:, None, :], new_state


def ffn_params(params):
    out = {}
    for k, v in params.items():
        if k.startswith("ffn."):
            out[k[4:]] = v
    return out


def _heads(y, B, L, H, dk):
    return y.reshape(B, L, H, dk).transpose(0, 2, 1, 3)


def block_forward(x, params, n_heads, chunk_size, beta_mode="learned",
                  memory_state=None, dtype=np.float64):
    """layers.py:177-244.  Returns ``(x_out, M_state)``."""
    x = np.asarray(x, dtype=dtype)
    B, L, d = x.shape
    dk = d // n_heads
    C = chunk_size
    normed = layer_norm(x, _p(params, "norm1.weight", dtype), _p(params, "norm1.bias", dtype))
    conv_x = causal_conv(normed, params, dtype)
    pad = (C - L % C) % C                                          # :185-190
    if pad:
        conv_x = np.concatenate([conv_x, np.zeros((B, pad, d), dtype)], 1)
    Lp = L + pad
    tk = _heads(linear(conv_x, params, "w_k", dtype), B, Lp, n_heads, dk)
    tq = _heads(linear(conv_x, params, "w_q", dtype), B, Lp, n_heads, dk)
    v = _heads(linear(conv_x, params, "w_v", dtype), B, Lp, n_heads, dk)
    beta = (2.0 / (1.0 + np.exp(-linear(conv_x, params, "w_beta", dtype)))).transpose(0, 2, 1)
    if beta_mode == "fixed":
        beta = np.ones_like(beta)
    if pad:
        beta[:, :, L:] = 0.0                                       # :198-201
    out, M = core.chunkwise_delta(tk, tq, v, beta, C, memory_state, dtype)
    retrieved = out[:, :, :L].transpose(0, 2, 1, 3).reshape(B, L, d)
    rn = layer_norm(retrieved, _p(params, "norm_retrieved.weight", dtype),
                    _p(params, "norm_retrieved.bias", dtype))
    x1 = x + linear(rn, params, "out_proj", dtype)
    n2 = layer_norm(x1, _p(params, "norm2.weight", dtype), _p(params, "norm2.bias", dtype))
    return x1 + spectral.lerp_ffn(n2, ffn_params(params), dtype), M


def block_step(x_t, params, n_heads, state=None, beta_mode="learned", dtype=np.float64):
    """layers.py:246-291.  x_t (B, 1, d); state = (conv_state, M) or None.
    Returns ``(x_out, (conv_state, M))``."""
    x_t = np.asarray(x_t, dtype=dtype)
    B, _, d = x_t.shape
    dk = d // n_heads
    conv_state, M = (None, None) if state is None else state
    normed = layer_norm(x_t, _p(params, "norm1.weight", dtype), _p(params, "norm1.bias", dtype))
    conv_x, new_conv = causal_conv_step(normed, conv_state, params, dtype)
    tk = _heads(linear(conv_x, params, "w_k", dtype), B, 1, n_heads, dk)[:, :, 0]
    tq = _heads(linear(conv_x, params, "w_q", dtype), B, 1, n_heads, dk)[:, :, 0]
    v = _heads(linear(conv_x, params, "w_v", dtype), B, 1, n_heads, dk)[:, :, 0]
    beta = (2.0 / (1.0 + np.exp(-linear(conv_x, params, "w_beta", dtype))))[:, 0, :]
    if beta_mode == "fixed":
        beta = np.ones_like(beta)
    if M is None:
        M = np.zeros((B, n_heads, dk, dk), dtype=core._cplx(dtype))
    out, M = core.decode_step(M, tk, tq, v, beta, dtype)
    rn = layer_norm(out.reshape(B, 1, d), _p(params, "norm_retrieved.weight", dtype),
                    _p(params, "norm_retrieved.bias", dtype))
    x1 = x_t + linear(rn, params, "out_proj", dtype)
    n2 = layer_norm(x1, _p(params, "norm2.weight", dtype), _p(params, "norm2.bias", dtype))
    return x1 + spectral.lerp_ffn(n2, ffn_params(params), dtype), (new_conv, M)


def cb_block_forward(x, params, n_heads, memory_state=None, dtype=np.float64):
    """``ComplexBetaDeltaPhaseBlock.forward`` (layers.py:324-366): LayerNorm, causal conv,
    projections, phi = w_phi(conv_x), the complex-beta token loop, output projection and
    FFN.  Returns ``(x_out, M_state)``."""
    x = np.asarray(x, dtype=dtype)
    B, L, d = x.shape
    dk = d // n_heads
    normed = layer_norm(x, _p(params, "norm1.weight", dtype), _p(params, "norm1.bias", dtype))
    conv_x = causal_conv(normed, params, dtype)
    tk = _heads(linear(conv_x, params, "w_k", dtype), B, L, n_heads, dk)
    tq = _heads(linear(conv_x, params, "w_q", dtype), B, L, n_heads, dk)
    v = _heads(linear(conv_x, params, "w_v", dtype), B, L, n_heads, dk)
    phi = linear(conv_x, params, "w_phi", dtype).transpose(0, 2, 1)     # :336
    out, M = core.complex_beta_recurrent(tk, tq, v, phi, memory_state, dtype)
    retrieved = out.transpose(0, 2, 1, 3).reshape(B, L, d)
    rn = layer_norm(retrieved, _p(params, "norm_retrieved.weight", dtype),
                    _p(params, "norm_retrieved.bias", dtype))
    x1 = x + linear(rn, params, "out_proj", dtype)
    n2 = layer_norm(x1, _p(params, "norm2.weight", dtype), _p(params, "norm2.bias", dtype))
    return x1 + spectral.lerp_ffn(n2, ffn_params(params), dtype), M


def cb_block_step(x_t, params, n_heads, state=None, dtype=np.float64):
    """``ComplexBetaDeltaPhaseBlock.step`` (layers.py:368-418).  x_t (B, 1, d);
    state = (conv_state, M) or None.  Returns ``(x_out, (conv_state, M))``."""
    x_t = np.asarray(x_t, dtype=dtype)
    B, _, d = x_t.shape
    dk = d // n_heads
    conv_state, M = (None, None) if state is None else state
    normed = layer_norm(x_t, _p(params, "norm1.weight", dtype), _p(params, "norm1.bias", dtype))
    conv_x, new_conv = causal_conv_step(normed, conv_state, params, dtype)
    tk = _heads(linear(conv_x, params, "w_k", dtype), B, 1, n_heads, dk)[:, :, 0]
    tq = _heads(linear(conv_x, params, "w_q", dtype), B, 1, n_heads, dk)[:, :, 0]
    v = _heads(linear(conv_x, params, "w_v", dtype), B, 1, n_heads, dk)[:, :, 0]
    phi = linear(conv_x, params, "w_phi", dtype)[:, 0, :]
    if M is None:
        M = np.zeros((B, n_heads, dk, dk), dtype=core._cplx(dtype))
    out, M = core.complex_beta_step(M, tk, tq, v, phi, dtype)
    rn = layer_norm(out.reshape(B, 1, d), _p(params, "norm_retrieved.weight", dtype),
                    _p(params, "norm_retrieved.bias", dtype))
    x1 = x_t + linear(rn, params, "out_proj", dtype)
    n2 = layer_norm(x1, _p(params, "norm2.weight", dtype), _p(params, "norm2.bias", dtype))
    return x1 + spectral.lerp_ffn(n2, ffn_params(params), dtype), (new_conv, M)
