"""Drop-in modules of the DeltaPhase hot path, running on the B200 CUDA kernels.

Same class names, constructor arguments, parameter and buffer names as
``delta_phase/layers.py`` (mcarbonell/delta-phase v1.3.0), so ``state_dict`` files
load in both directions:

* :class:`ShortCausalConv1D`            -- layers.py:60-88 (torch glue, unchanged math)
* :class:`LearnableSubstrateLerpFFN`    -- layers.py:90-145 (CUDA: dp_ffn_fold/dp_ffn_fwd)
* :class:`DeltaPhaseHolographicBlock`   -- layers.py:147-291 (CUDA: dp_core_fwd/dp_core_decode)
* :class:`ComplexBetaDeltaPhaseBlock`   -- layers.py:294-418 (CUDA: dp_core_cbeta_fwd/dp_core_cbeta_decode)
* :class:`LaplacePhaseCore`             -- layers.py:422-583 (CUDA: dp_laplace_fwd)

The delta-rule core, its decode step, the block glue and the spectral FFN run in the
CUDA library, with no CPU fallback.  Training: when autograd is recording (grad enabled
and an input or parameter requires grad -- the reference dispatcher's rule,
triton_chunk_delta.py:279-291), the two delta-rule blocks run their glue and the FFN as
differentiable torch ops and the core through DeltaPhaseCudaFunction (backward on the
dp_core_bwd kernel); LaplacePhaseCore through LaplaceCudaFunction (dp_laplace_bwd).
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _capi
from .kernels.chunk_delta import DeltaPhaseCudaFunction, chunkwise_forward, decode_step, laplace_chunkwise
from .spectral import create_dct2_matrix, create_haar_matrix, create_hadamard_matrix

_BRANCHES = ("fwht", "dct", "haar")


def _records_autograd(module: nn.Module, *tensors) -> bool:
    """True when autograd would record this call: grad enabled and an input or a
    parameter of ``module`` requires grad."""
    if not torch.is_grad_enabled():
        return False
    return any(t is not None and t.requires_grad for t in tensors) or \
        any(p.requires_grad for p in module.parameters())


class ShortCausalConv1D(nn.Module):
    """Depthwise causal conv (kernel_size 4) + SiLU + residual (layers.py:60-88)."""

    def __init__(self, d_model: int, kernel_size: int = 4):
        super().__init__()
        self.kernel_size = kernel_size
        self.conv = nn.Conv1d(d_model, d_model, kernel_size, padding=kernel_size - 1, groups=d_model)
        self.act = nn.SiLU()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, L, D = x.shape
        conv_out = self.conv(x.transpose(1, 2))[:, :, :L].transpose(1, 2)
        return x + self.act(conv_out)

    def step(self, x_t: torch.Tensor, conv_state=None):
        B, L, D = x_t.shape
        if conv_state is None:
            conv_state = torch.zeros(B, D, self.kernel_size - 1, device=x_t.device, dtype=x_t.dtype)
        inputs = torch.cat([conv_state, x_t.transpose(1, 2)], dim=2)
        new_conv_state = inputs[:, :, 1:]
        conv_out = F.conv1d(inputs, self.conv.weight, self.conv.bias, groups=D)[:, :, -1:]
        return x_t + self.act(conv_out.transpose(1, 2)), new_conv_state


class LearnableSubstrateLerpFFN(nn.Module):
    """Spectral Lerp FFN (layers.py:90-145) on the folded CUDA path.

    The three branch activations are linear in z = [cos h_b, sin h_b] (angle addition),
    so the parameters are folded once into F (6d x d, float64 accumulation) and each
    call runs the fast transforms, 6d sincos per token and one GEMM.  F is rebuilt
    whenever a parameter or buffer changes (tracked by tensor version counters).
    """

    def __init__(self, d_model: int, num_banks: int = 4):
        super().__init__()
        self.d_model = d_model
        self.num_banks = num_banks
        self.substrate_logits = nn.Parameter(torch.tensor([0.0, 0.0, 0.0]))
        self.register_buffer("mat_fwht", create_hadamard_matrix(d_model))
        self.register_buffer("mat_dct", create_dct2_matrix(d_model))
        self.register_buffer("mat_haar", create_haar_matrix(d_model))
        for b in _BRANCHES:
            setattr(self, f"phi1_{b}", nn.Parameter(torch.zeros(num_banks, d_model)))
            setattr(self, f"phi2_{b}", nn.Parameter(torch.zeros(num_banks, d_model)))
            setattr(self, f"w1_{b}", nn.Parameter(torch.ones(num_banks, d_model)))
            setattr(self, f"w2_{b}", nn.Parameter(torch.ones(num_banks, d_model)))
        self.combine = nn.Linear(num_banks * d_model, d_model, bias=False)
        self._fold_key = None
        self._fold = {}

    def _state_key(self):
        ts = [self.substrate_logits, self.mat_fwht, self.mat_dct, self.mat_haar, self.combine.weight]
        for b in _BRANCHES:
            ts += [getattr(self, f"{n}_{b}") for n in ("phi1", "phi2", "w1", "w2")]
        return tuple((t.data_ptr(), t._version, t.device) for t in ts)

    @torch.no_grad()
    def folded(self, dtype):
        """F (6d x d) and the DCT matrix in ``dtype`` (float32 or bfloat16), cached."""
        key = self._state_key()
        if key != self._fold_key:
            d, nb = self.d_model, self.num_banks
            dev = self.mat_dct.device
            f32 = lambda t: t.detach().to(device=dev, dtype=torch.float32).contiguous()  # noqa: E731
            mats = torch.stack([f32(self.mat_fwht), f32(self.mat_dct), f32(self.mat_haar)])
            banks = torch.stack([torch.stack([f32(getattr(self, f"{n}_{b}"))
                                              for n in ("phi1", "phi2", "w1", "w2")])
                                 for b in _BRANCHES])
            Fm = torch.empty(6 * d, d, device=dev, dtype=torch.float32)
            _capi.ffn_fold(f32(self.substrate_logits), mats, banks, f32(self.combine.weight), Fm, d, nb)
            self._fold = {torch.float32: (Fm, f32(self.mat_dct))}
            self._fold_key = key
        if dtype not in self._fold:
            Fm, dct = self._fold[torch.float32]
            self._fold[dtype] = (Fm.to(dtype), dct.to(dtype))
        return self._fold[dtype]

    @torch.no_grad()
    def folded_t(self):
        """F^T (d x 6d) in bf16, contiguous: the combine matrix in nn.Linear layout for
        dp_gemm_skinny, cached with the fold."""
        Fm, _ = self.folded(torch.bfloat16)
        if self._fold.get("t") is None or self._fold["t"][0] is not Fm:
            self._fold["t"] = (Fm, Fm.t().contiguous())
        return self._fold["t"][1]

    def _forward_autograd(self, x: torch.Tensor) -> torch.Tensor:
        """The reference's formula (layers.py:119-141) as differentiable torch ops, for
        training (the folded CUDA path has no backward)."""
        weights = F.softmax(self.substrate_logits, dim=0)
        out = 0.0
        for i, b in enumerate(_BRANCHES):
            mat = getattr(self, f"mat_{b}")
            h = F.linear(x, mat).unsqueeze(-2)
            a = (torch.cos(h + getattr(self, f"phi1_{b}")) * getattr(self, f"w1_{b}") +
                 torch.sin(h + getattr(self, f"phi2_{b}")) * getattr(self, f"w2_{b}")).flatten(-2)
            out = out + weights[i] * F.linear(self.combine(a), mat.t())
        return out

    def _compute_dtype(self, x: torch.Tensor):
        """(GEMM operand dtype, output dtype) of the CUDA path for input ``x``."""
        cdt = torch.bfloat16 if x.dtype == torch.bfloat16 else torch.float32
        out_dt = x.dtype
        if cdt == torch.float32 and torch.is_autocast_enabled(x.device.type):
            # the reference's transforms and combine are matmuls, which autocast runs in
            # its lower precision: take the bf16 path and return bf16 like they would
            if torch.get_autocast_dtype(x.device.type) == torch.bfloat16:
                cdt = out_dt = torch.bfloat16
        return cdt, out_dt

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.shape[-1] != self.d_model:
            raise ValueError(f"expected last dim {self.d_model}, got {x.shape[-1]}")
        if x.dtype == torch.float64:
            raise TypeError("float64 inputs are not supported by the CUDA path")
        if _records_autograd(self, x):
            _capi.require_cuda(x, self.mat_dct)
            return self._forward_autograd(x)
        _capi.require_cuda(x, self.mat_dct)
        cdt, out_dt = self._compute_dtype(x)
        x2 = x.reshape(-1, self.d_model).to(cdt).contiguous()
        Fm, dct = self.folded(cdt)
        y = torch.empty_like(x2)
        ws = torch.empty(_capi.ffn_workspace_size(x2.shape[0], self.d_model, cdt),
                         device=x.device, dtype=torch.uint8)
        _capi.ffn_fwd(x2, dct, Fm, y, ws)
        return y.view(x.shape).to(out_dt)

    def add_to(self, residual: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
        """``residual += ffn(x)`` in place for a contiguous float32 ``residual`` shaped like
        ``x``, the block's ``x + self.ffn(self.norm2(x))`` (layers.py:243, 290) with the add
        in the combine GEMM's epilogue (dp_ffn_fwd_residual).  Inference path only."""
        _capi.require_cuda(x, residual, self.mat_dct)
        cdt, _ = self._compute_dtype(x)
        x2 = x.reshape(-1, self.d_model).to(cdt).contiguous()
        Fm, dct = self.folded(cdt)
        tokens, d = x2.shape
        ws = torch.empty(_capi.ffn_workspace_size(tokens, d, cdt), device=x.device, dtype=torch.uint8)
        if cdt == torch.bfloat16 and tokens <= _capi.SKINNY_MAX_ROWS and d % 32 == 0:
            # decode batch: DCT projection and folded combine through dp_gemm_skinny (F^T
            # is the (d, 6d) weight in nn.Linear layout), features in between
            hdct = ws[:tokens * d * 4].view(torch.float32).view(tokens, d)
            z = ws[tokens * d * 4:tokens * d * 16].view(torch.bfloat16).view(tokens, 6 * d)
            _capi.gemm_skinny(x2, dct, None, hdct)
            _capi.ffn_features(x2, hdct, z)
            _capi.gemm_skinny(z, self.folded_t(), None, residual.view(-1, d), accumulate=True)
            return residual
        _capi.ffn_fwd_residual(x2, dct, Fm, residual.view(-1, self.d_model), ws)
        return residual

    def get_substrate_probabilities(self):
        probs = F.softmax(self.substrate_logits, dim=0)
        return probs[0].item(), probs[1].item(), probs[2].item()


class _DeltaRuleBlock(nn.Module):
    """Forward and step shared by the two delta-rule blocks: LayerNorm -> causal conv ->
    projections -> the delta-rule core -> norm_retrieved -> out_proj -> norm2 -> FFN.
    Subclasses name the write-gate projection (``_gate_linear``), map its output to the
    kernel's gate (``_write_gate``) and to ``last_beta``, and set ``_complex_beta``."""

    _complex_beta = False

    def _gate_linear(self) -> nn.Linear:
        raise NotImplementedError

    def _write_gate(self, g: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError

    def _last_beta(self, gate: torch.Tensor) -> torch.Tensor:
        return gate.detach()

    def _decode_gate_mode(self) -> int:
        """How dp_core_decode_gated forms beta from the raw gate projection."""
        raise NotImplementedError

    @property
    def last_beta(self):
        """The write strengths of the last forward or step, as the reference records them
        (layers.py:240, 268, 346, 400).  After a step it is formed on access from the raw
        gate the decode kernel read, so the step launches no gate kernels of its own."""
        raw = self.__dict__.get("_last_gate_raw")
        if raw is not None:
            with torch.no_grad():
                return self._last_beta(self._write_gate(raw).unsqueeze(-1))
        return self.__dict__.get("_last_beta_value")

    @last_beta.setter
    def last_beta(self, value):
        self.__dict__["_last_beta_value"] = value
        self.__dict__["_last_gate_raw"] = None

    def _proj_weights(self, dtype):
        """[w_k; w_q; w_v; gate] weights (and biases, when the layers have them)
        concatenated in ``dtype`` (one GEMM for the four input projections), rebuilt when
        any of them changes."""
        lins = (self.w_k, self.w_q, self.w_v, self._gate_linear())
        biases = [m.bias for m in lins if m.bias is not None]
        if biases and len(biases) != len(lins):
            raise ValueError("the input projections must all have biases or none")
        ts = tuple(m.weight for m in lins) + tuple(biases)
        key = (dtype,) + tuple((t.data_ptr(), t._version) for t in ts)
        if getattr(self, "_proj_key", None) != key:
            with torch.no_grad():
                W = torch.cat([t.detach() for t in ts[:4]], 0).to(dtype).contiguous()
                bvec = torch.cat([t.detach() for t in ts[4:]], 0).to(dtype).contiguous() if biases else None
            self._proj_cache = (W, bvec)
            self._proj_key = key
        return self._proj_cache

    def _forward_autograd(self, x: torch.Tensor, memory_state=None):
        """Differentiable block forward for training: the reference's sequence of torch
        ops around the core (layers.py:177-244 / 324-366) with the core through
        DeltaPhaseCudaFunction (CUDA forward and backward)."""
        B, L, D = x.shape
        H, dk = self.n_heads, self.d_k
        conv_x = self.causal_conv(self.norm1(x))
        tk = self.w_k(conv_x).view(B, L, H, dk).transpose(1, 2)
        tq = self.w_q(conv_x).view(B, L, H, dk).transpose(1, 2)
        v = self.w_v(conv_x).view(B, L, H, dk).transpose(1, 2)
        beta = self._write_gate(self._gate_linear()(conv_x)).transpose(1, 2)   # (B, H, L)
        if tk.dtype != tq.dtype or tk.dtype != v.dtype:
            tq, v = tq.to(tk.dtype), v.to(tk.dtype)
        out, M_state = DeltaPhaseCudaFunction.apply(tk, tq, v, beta, self.chunk_size, memory_state,
                                                    self._complex_beta)
        self.last_beta = self._last_beta(beta)
        retrieved = out.transpose(1, 2).reshape(B, L, D)
        x = x + self.out_proj(self.norm_retrieved(retrieved))
        return x + self.ffn(self.norm2(x)), M_state

    def forward(self, x: torch.Tensor, memory_state=None):
        """Block forward (layers.py:177-244); see ``_forward``."""
        return self._forward(x, memory_state)

    def _forward(self, x: torch.Tensor, memory_state=None, keep_fp32: bool = False):
        """Block forward (layers.py:177-244) on fused kernels: LayerNorm + causal conv +
        SiLU + residual in one pass, the four input projections as one GEMM, the
        delta-rule core, LayerNorm -> output projection, and the residual add fused into
        norm2.  GEMM operands are bf16 under bf16 autocast (like the reference's autocast
        matmuls) and float32 otherwise; the residual stream stays float32.  When autograd
        records (training), the differentiable path above runs instead.  ``keep_fp32``
        returns the float32 residual stream instead of casting it back to x's dtype (the
        model's layer loop passes it between blocks that way)."""
        if x.dtype == torch.float64:
            raise TypeError("float64 inputs are not supported by the CUDA path")
        _capi.require_cuda(x)
        if _records_autograd(self, x, memory_state):
            return self._forward_autograd(x, memory_state)
        B, L, D = x.shape
        H, dk = self.n_heads, self.d_k
        bf16_ac = torch.is_autocast_enabled(x.device.type) and \
            torch.get_autocast_dtype(x.device.type) == torch.bfloat16
        gdt = torch.bfloat16 if (bf16_ac or x.dtype == torch.bfloat16) else torch.float32
        xc = x.contiguous()
        conv = self.causal_conv.conv
        conv_x = torch.empty(B, L, D, device=x.device, dtype=gdt)
        _capi.ln_conv_silu(xc, self.norm1.weight.float(), self.norm1.bias.float(), self.norm1.eps,
                           conv.weight.detach().float().reshape(D, -1).contiguous(),
                           None if conv.bias is None else conv.bias.detach().float(), conv_x)
        W, bvec = self._proj_weights(gdt)
        with torch.autocast(x.device.type, enabled=False):
            proj = F.linear(conv_x, W, bvec)                      # (B, L, 3D + H)
        # (B, L, H, dk) slices of the projection viewed as (B, H, L, dk): the kernel reads
        # them in place and writes the retrieved values straight into (B, L, D)
        tk = proj[..., :D].view(B, L, H, dk).transpose(1, 2)
        tq = proj[..., D:2 * D].view(B, L, H, dk).transpose(1, 2)
        v = proj[..., 2 * D:3 * D].view(B, L, H, dk).transpose(1, 2)
        beta = self._write_gate(proj[..., 3 * D:]).transpose(1, 2)   # (B, H, L)
        retrieved = torch.empty(B, L, D, device=x.device, dtype=torch.float32)
        _, M_state = chunkwise_forward(tk, tq, v, beta, self.chunk_size, memory_state,
                                       out=retrieved.view(B, L, H, dk).transpose(1, 2),
                                       complex_beta=self._complex_beta)
        self.last_beta = self._last_beta(beta)
        nr = self.norm_retrieved
        rn = torch.empty(B * L, D, device=x.device, dtype=gdt)
        _capi.layernorm(retrieved.view(B * L, D), nr.weight.float(), nr.bias.float(), nr.eps, rn)
        o = self.out_proj(rn)
        # s = x + out_proj(...) (float32), n2 = norm2(s) in the FFN's operand dtype
        res = xc.view(B * L, D)
        res32 = res if res.dtype == torch.float32 else res.float()
        s_sum = torch.empty(B * L, D, device=x.device, dtype=torch.float32)
        n2 = torch.empty(B * L, D, device=x.device, dtype=gdt)
        _capi.layernorm(o.contiguous(), self.norm2.weight.float(), self.norm2.bias.float(), self.norm2.eps, n2,
                        residual=res32, sum_out=s_sum)
        out = self.ffn.add_to(s_sum, n2).view(B, L, D)
        return (out if (keep_fp32 or x.dtype == torch.float32) else out.to(x.dtype)), M_state

    def _out_proj_weights(self, dtype):
        """out_proj weight and bias in ``dtype``, rebuilt when either changes."""
        ts = (self.out_proj.weight, self.out_proj.bias)
        key = (dtype,) + tuple((t.data_ptr(), t._version) for t in ts)
        if getattr(self, "_oproj_key", None) != key:
            with torch.no_grad():
                self._oproj_cache = tuple(t.detach().to(dtype).contiguous() for t in ts)
            self._oproj_key = key
        return self._oproj_cache

    def _step_inplace(self, x_t: torch.Tensor, conv_state: torch.Tensor, memory_state: torch.Tensor,
                      keep_fp32: bool = False):
        """One decode token (layers.py:246-291) with the state updated in place:
        ``conv_state`` (B, d, k-1) float32 and ``memory_state`` (B, H, d_k, d_k) complex64
        are overwritten, so their addresses stay fixed (what a captured CUDA graph needs).
        norm1 + the conv step in one kernel, the projections as one GEMM on cached
        weights (no per-call casts), the fused decode kernel (which forms the write gate
        from its raw projection), norm_retrieved, and norm2 with the residual add fused
        in.  Returns x (B, 1, d)."""
        if x_t.dtype == torch.float64:
            raise TypeError("float64 inputs are not supported by the CUDA path")
        B, _, D = x_t.shape
        H, dk = self.n_heads, self.d_k
        bf16_ac = torch.is_autocast_enabled(x_t.device.type) and \
            torch.get_autocast_dtype(x_t.device.type) == torch.bfloat16
        gdt = torch.bfloat16 if (bf16_ac or x_t.dtype == torch.bfloat16) else torch.float32
        xc = x_t.reshape(B, D).contiguous()
        conv = self.causal_conv.conv
        conv_x = torch.empty(B, D, device=x_t.device, dtype=gdt)
        _capi.ln_conv_step(xc, self.norm1.weight.float(), self.norm1.bias.float(), self.norm1.eps,
                           conv.weight.detach().float().reshape(D, -1).contiguous(),
                           None if conv.bias is None else conv.bias.detach().float(), conv_state, conv_x)
        W, bvec = self._proj_weights(gdt)
        Wo, bo = self._out_proj_weights(gdt)
        # decode batches of bf16 rows: the weights stream through dp_gemm_skinny
        skinny = gdt == torch.bfloat16 and B <= _capi.SKINNY_MAX_ROWS and D % 32 == 0
        with torch.autocast(x_t.device.type, enabled=False):
            if skinny:
                proj = torch.empty(B, W.shape[0], device=x_t.device, dtype=gdt)
                _capi.gemm_skinny(conv_x, W, bvec, proj)
            else:
                proj = F.linear(conv_x, W, bvec)                  # (B, 3D + H)
            tk = proj[:, :D].view(B, H, dk)
            tq = proj[:, D:2 * D].view(B, H, dk)
            v = proj[:, 2 * D:3 * D].view(B, H, dk)
            gate = proj[:, 3 * D:]                                 # raw (B, H) gate
            self.last_beta = None
            self.__dict__["_last_gate_raw"] = gate
            out, _ = decode_step(memory_state, tk, tq, v, gate, state_out=memory_state,
                                 gate_mode=self._decode_gate_mode())
            nr = self.norm_retrieved
            rn = torch.empty(B, D, device=x_t.device, dtype=gdt)
            _capi.layernorm(out.view(B, D), nr.weight.float(), nr.bias.float(), nr.eps, rn)
            if skinny:
                o = torch.empty(B, D, device=x_t.device, dtype=gdt)
                _capi.gemm_skinny(rn, Wo, bo, o)
            else:
                o = F.linear(rn, Wo, bo)
            res32 = xc if xc.dtype == torch.float32 else xc.float()
            s_sum = torch.empty(B, D, device=x_t.device, dtype=torch.float32)
            n2 = torch.empty(B, D, device=x_t.device, dtype=gdt)
            _capi.layernorm(o, self.norm2.weight.float(), self.norm2.bias.float(), self.norm2.eps, n2,
                            residual=res32, sum_out=s_sum)
        y = self.ffn.add_to(s_sum, n2).view(B, 1, D)
        return y if (keep_fp32 or x_t.dtype == torch.float32) else y.to(x_t.dtype)

    def step(self, x_t: torch.Tensor, state=None):
        """Single-token step (layers.py:246-291); returns ``(x, (conv_state, M))``.
        The input state is not modified: the new conv state (float32, (B, d, k-1)) and
        memory state are fresh tensors."""
        return self._step_fresh(x_t, state)

    def _step_fresh(self, x_t: torch.Tensor, state=None, keep_fp32: bool = False):
        """``step`` on fresh state tensors; ``keep_fp32`` returns the float32 residual
        stream instead of casting it back to x_t's dtype (the model's decode loop passes it
        between blocks that way)."""
        B, _, D = x_t.shape
        H, dk = self.n_heads, self.d_k
        if state is None:
            conv_state, memory_state = None, None
        elif isinstance(state, tuple):
            conv_state, memory_state = state
        else:
            conv_state, memory_state = None, state
        k = self.causal_conv.kernel_size
        if conv_state is None:
            conv_new = torch.zeros(B, D, k - 1, device=x_t.device, dtype=torch.float32)
        else:
            conv_new = conv_state.detach().to(torch.float32).clone().contiguous()
        if memory_state is None:
            mem_new = torch.zeros(B, H, dk, dk, dtype=torch.complex64, device=x_t.device)
        else:
            mem_new = memory_state.detach().to(torch.complex64).clone().contiguous()
        x = self._step_inplace(x_t, conv_new, mem_new, keep_fp32=keep_fp32)
        return x, (conv_new, mem_new)


class DeltaPhaseHolographicBlock(_DeltaRuleBlock):
    """Chunkwise complex delta-phase memory block (layers.py:147-291)."""

    def __init__(self, d_model: int, n_heads: int = 8, conv_kernel_size: int = 4,
                 chunk_size: int = 64, num_banks: int = 4, beta_mode: str = "learned"):
        super().__init__()
        if beta_mode not in ("learned", "fixed"):
            raise ValueError(f"beta_mode must be 'learned' or 'fixed', got {beta_mode!r}")
        self.d_model = d_model
        self.n_heads = n_heads
        self.d_k = d_model // n_heads
        self.inv_dk = 1.0 / float(self.d_k)
        self.chunk_size = chunk_size
        self.beta_mode = beta_mode
        self.last_beta = None
        self.norm1 = nn.LayerNorm(d_model)
        self.norm2 = nn.LayerNorm(d_model)
        self.norm_retrieved = nn.LayerNorm(d_model)
        self.causal_conv = ShortCausalConv1D(d_model, kernel_size=conv_kernel_size)
        self.w_k = nn.Linear(d_model, d_model)
        self.w_q = nn.Linear(d_model, d_model)
        self.w_v = nn.Linear(d_model, d_model)
        self.w_beta = nn.Linear(d_model, n_heads)
        self.out_proj = nn.Linear(d_model, d_model)
        self.ffn = LearnableSubstrateLerpFFN(d_model, num_banks=num_banks)

    def _gate_linear(self):
        return self.w_beta

    def _write_gate(self, g):
        """beta = 2 sigmoid(w_beta(conv_x)) (layers.py:195), or 1 in "fixed" mode (:196-197)."""
        if self.beta_mode == "fixed":
            return torch.ones(g.shape, device=g.device, dtype=torch.float32)
        return 2.0 * torch.sigmoid(g.float())

    def _decode_gate_mode(self):
        return _capi.DP_GATE_ONE if self.beta_mode == "fixed" else _capi.DP_GATE_SIGMOID2


class ComplexBetaDeltaPhaseBlock(_DeltaRuleBlock):
    """Complex-beta Householder block (layers.py:294-418): beta_t = 1 + e^{i phi_t} with
    phi = w_phi(conv_x), update M += beta (v - Re(M conj k) / d_k) k^T.  The reference
    runs a token loop (layers.py:346-360); here the sequence goes through the chunkwise
    (WY) form of the same recurrence on the tensor-core kernel (dp_core_cbeta_fwd) and
    ``step`` through dp_core_cbeta_decode.  ``chunk_size`` is kept for the constructor's
    signature; like the reference's loop, the result does not depend on it."""

    _complex_beta = True

    def __init__(self, d_model: int, n_heads: int = 4, conv_kernel_size: int = 4,
                 chunk_size: int = 32, num_banks: int = 2):
        super().__init__()
        self.d_model = d_model
        self.n_heads = n_heads
        self.d_k = d_model // n_heads
        self.inv_dk = 1.0 / float(self.d_k)
        self.chunk_size = chunk_size
        self.beta_mode = "complex"
        self.norm1 = nn.LayerNorm(d_model)
        self.norm2 = nn.LayerNorm(d_model)
        self.norm_retrieved = nn.LayerNorm(d_model)
        self.causal_conv = ShortCausalConv1D(d_model, kernel_size=conv_kernel_size)
        self.w_k = nn.Linear(d_model, d_model, bias=False)
        self.w_q = nn.Linear(d_model, d_model, bias=False)
        self.w_v = nn.Linear(d_model, d_model, bias=False)
        self.w_phi = nn.Linear(d_model, n_heads, bias=False)
        self.out_proj = nn.Linear(d_model, d_model)
        self.ffn = LearnableSubstrateLerpFFN(d_model, num_banks=num_banks)
        self.last_beta = None

    def _gate_linear(self):
        return self.w_phi

    def _write_gate(self, g):
        """phi (float32); the kernels form beta = 1 + e^{i phi} (layers.py:344, 397)."""
        return g.float()

    def _last_beta(self, phi):
        """beta_complex = 1 + polar(1, phi), as the reference records it (layers.py:346, 400)."""
        with torch.no_grad():
            return 1.0 + torch.polar(torch.ones_like(phi), phi)

    def _decode_gate_mode(self):
        return _capi.DP_GATE_PHI


class LaplacePhaseCore(nn.Module):
    """Gated (Laplace) phase memory core (layers.py:422-583) on the CUDA kernel.

    Recurrence: v_old = Re(M k^H)/d_k; M = diag(r_t) M + beta_t (v_t - v_old) k_t^T;
    out_t = Re(M q^H)/d_k with K = r_k e^{i theta_k}, r_t = r_k (both from sigma_k).
    """

    LOG_FLOOR = -80.0

    def __init__(self, d_model=64, n_heads=4, d_k=16, chunk_size=32):
        super().__init__()
        self.d_model = d_model
        self.n_heads = n_heads
        self.d_k = d_k
        self.inv_dk = 1.0 / float(d_k)
        self.chunk_size = int(chunk_size)
        self.w_theta_k = nn.Linear(d_model, d_model, bias=False)
        self.w_sigma_k = nn.Linear(d_model, d_model, bias=False)
        self.w_theta_q = nn.Linear(d_model, d_model, bias=False)
        self.w_sigma_q = nn.Linear(d_model, d_model, bias=False)
        self.w_v = nn.Linear(d_model, d_model, bias=False)
        self.w_beta = nn.Linear(d_model, n_heads, bias=False)

    def _proj(self, x, time_scale):
        """Real projections (layers.py:462-479 before the phasor is formed), float32."""
        B, L, _ = x.shape
        dt = 1.0 / float(time_scale)
        if x.dtype == torch.float64:
            raise TypeError("float64 inputs are not supported by the CUDA path")
        hv = lambda y: y.view(B, L, self.n_heads, self.d_k).transpose(1, 2)  # noqa: E731
        theta_k = hv(self.w_theta_k(x).float() * dt)
        sigma_k = hv(-F.softplus(self.w_sigma_k(x).float()) * dt)
        theta_q = hv(self.w_theta_q(x).float() * dt)
        sigma_q = hv(-F.softplus(self.w_sigma_q(x).float()) * dt)
        v = hv(self.w_v(x).float())
        beta = (2.0 * torch.sigmoid(self.w_beta(x).float()) * dt).transpose(1, 2)
        return theta_k, sigma_k, theta_q, sigma_q, v, beta

    def _project(self, x: torch.Tensor, time_scale: float):
        """Reference API (layers.py:462-479): returns (K, Q, v, beta, r_k)."""
        theta_k, sigma_k, theta_q, sigma_q, v, beta = self._proj(x, time_scale)
        r_k = torch.exp(sigma_k)
        r_q = torch.exp(sigma_q)
        K = torch.complex(r_k * torch.cos(theta_k), r_k * torch.sin(theta_k))
        Q = torch.complex(r_q * torch.cos(theta_q), r_q * torch.sin(theta_q))
        return K, Q, v, beta, r_k

    def forward(self, x: torch.Tensor, memory_state=None, time_scale: float = 1.0):
        theta_k, sigma_k, theta_q, sigma_q, v, beta = self._proj(x, time_scale)
        B, H, L, dk = theta_k.shape
        if _records_autograd(self, x, memory_state):
            # training: sigma_k is both the key's log-magnitude and the row decay; autograd
            # adds the two gradients
            out, M = laplace_chunkwise(theta_k, sigma_k, theta_q, sigma_q, v, sigma_k, beta, self.chunk_size,
                                       memory_state)
            return out.transpose(1, 2).reshape(B, L, H * dk), M
        retrieved = torch.empty(B, L, H * dk, device=x.device, dtype=torch.float32)
        _, M = laplace_chunkwise(theta_k, sigma_k, theta_q, sigma_q, v, sigma_k, beta,
                                 self.chunk_size, memory_state,
                                 out=retrieved.view(B, L, H, dk).transpose(1, 2))
        return retrieved, M

    def forward_sequential(self, x: torch.Tensor, memory_state=None, time_scale: float = 1.0):
        """Literal token loop (layers.py:563-583), kept as the module's reference API for
        equivalence tests; it is not used by ``forward``."""
        K, Q, v, beta, r_k = self._project(x, time_scale)
        B, H, L, dk = K.shape
        M = (torch.zeros(B, H, dk, dk, dtype=torch.complex64, device=x.device)
             if memory_state is None else memory_state)
        outs = []
        for t in range(L):
            kt, qt, vt, bt = K[:, :, t], Q[:, :, t], v[:, :, t], beta[:, :, t]
            v_old = torch.matmul(M, torch.conj(kt).unsqueeze(-1)).squeeze(-1).real * self.inv_dk
            err = vt - v_old
            M = M * r_k[:, :, t].unsqueeze(-1) + bt[..., None, None] * torch.matmul(
                err.to(M.dtype).unsqueeze(-1), kt.unsqueeze(-2))
            outs.append(torch.matmul(M, torch.conj(qt).unsqueeze(-1)).squeeze(-1).real * self.inv_dk)
        retrieved = torch.stack(outs, 2).transpose(1, 2).reshape(B, L, self.d_model)
        return retrieved, M
