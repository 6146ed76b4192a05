"""DeltaPhase language model on the B200 blocks (drop-in for delta_phase/model.py:9-140).

Same config fields, module names and weight init, so reference checkpoints load.
``beta_mode="complex"`` / ``"complex_householder"`` builds ComplexBetaDeltaPhaseBlock
layers (model.py:38-45 of the reference), the others DeltaPhaseHolographicBlock.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _capi
from .layers import ComplexBetaDeltaPhaseBlock, DeltaPhaseHolographicBlock


@dataclass
class DeltaPhaseConfig:
    dim: int = 512
    emb_dim: int = 128
    n_layers: int = 6
    n_heads: int = 8
    vocab_size: int = 32768
    max_seq_len: int = 2048
    chunk_size: int = 128
    conv_kernel_size: int = 4
    num_banks: int = 4
    weight_tying: bool = True
    beta_mode: str = "learned"


class DeltaPhaseModel(nn.Module):
    """Embedding (optionally factorised), N holographic blocks, final norm, tied head."""

    def __init__(self, config: DeltaPhaseConfig):
        super().__init__()
        self.config = config
        if config.emb_dim and config.emb_dim > 0:
            self.embed = nn.Embedding(config.vocab_size, config.emb_dim)
            self.embed_proj = nn.Linear(config.emb_dim, config.dim, bias=False)
            self.use_factorized = True
        else:
            self.embed = nn.Embedding(config.vocab_size, config.dim)
            self.embed_proj = None
            self.use_factorized = False
        if config.beta_mode in ("complex", "complex_householder"):
            make = lambda: ComplexBetaDeltaPhaseBlock(  # noqa: E731
                d_model=config.dim, n_heads=config.n_heads, conv_kernel_size=config.conv_kernel_size,
                chunk_size=config.chunk_size, num_banks=config.num_banks)
        else:
            make = lambda: DeltaPhaseHolographicBlock(  # noqa: E731
                d_model=config.dim, n_heads=config.n_heads, conv_kernel_size=config.conv_kernel_size,
                chunk_size=config.chunk_size, num_banks=config.num_banks, beta_mode=config.beta_mode)
        self.blocks = nn.ModuleList([make() for _ in range(config.n_layers)])
        self.norm_f = nn.LayerNorm(config.dim)
        if self.use_factorized:
            self.head_proj = nn.Linear(config.dim, config.emb_dim, bias=False)
            self.head = nn.Linear(config.emb_dim, config.vocab_size, bias=False)
        else:
            self.head_proj = None
            self.head = nn.Linear(config.dim, config.vocab_size, bias=False)
        if config.weight_tying:
            self.head.weight = self.embed.weight
        self._init_weights()

    def _init_weights(self):
        for m in self.modules():
            if isinstance(m, nn.Linear):
                nn.init.normal_(m.weight, std=0.02)
                if m.bias is not None:
                    nn.init.zeros_(m.bias)
            elif isinstance(m, nn.Embedding):
                nn.init.normal_(m.weight, std=0.02)

    def _embed(self, ids):
        e = self.embed(ids)
        return self.embed_proj(e) if self.use_factorized else e

    def _head(self, h):
        h = self.norm_f(h)
        if self.head_proj is not None:
            h = self.head_proj(h)
        return self.head(h)

    # ---- decode step: embedding and head of a few bf16 rows on the library's kernels
    def _bf16_weight(self, lin):
        """bf16 copy of a Linear's / Embedding's weight, rebuilt when it changes."""
        cache = self.__dict__.setdefault("_bf16_cache", {})
        w = lin.weight
        key = (w.data_ptr(), w._version, w.device)
        hit = cache.get(id(w))  # per parameter: the tied embedding / head share one copy
        if hit is None or hit[0] != key:
            with torch.no_grad():
                hit = (key, w.detach().to(torch.bfloat16).contiguous())
            cache[id(w)] = hit
        return hit[1]

    def _step_fast(self, rows: int, dev) -> bool:
        """Decode rows under bf16 autocast go through dp_layernorm / dp_gemm_skinny with
        cached bf16 weights (no per-token weight casts)."""
        if not (dev.type == "cuda" and torch.is_autocast_enabled("cuda")
                and torch.get_autocast_dtype("cuda") == torch.bfloat16):
            return False
        if rows > _capi.SKINNY_MAX_ROWS or torch.is_grad_enabled():
            return False
        dims = [self.config.dim] + ([self.config.emb_dim] if self.use_factorized else [])
        return all(d % 32 == 0 for d in dims) and self.head.bias is None and \
            (self.embed_proj is None or self.embed_proj.bias is None) and \
            (self.head_proj is None or self.head_proj.bias is None)

    def _embed_step(self, ids):
        """_embed for one token per sequence; (B, 1, dim), float32 on the fast path."""
        B = ids.shape[0]
        if not self._step_fast(B, ids.device):
            return self._embed(ids)
        e = F.embedding(ids.reshape(B), self._bf16_weight(self.embed))
        if not self.use_factorized:
            return e.view(B, 1, -1)
        h = torch.empty(B, self.config.dim, device=ids.device, dtype=torch.float32)
        _capi.gemm_skinny(e, self._bf16_weight(self.embed_proj), None, h)
        return h.view(B, 1, -1)

    def _head_step(self, h):
        """_head for one token per sequence; bf16 logits on the fast path, like the
        autocast matmul of the reference's head."""
        B = h.shape[0]
        if not self._step_fast(B, h.device):
            return self._head(h)
        d = self.config.dim
        x = h.reshape(B, d)
        n = torch.empty(B, d, device=h.device, dtype=torch.bfloat16)
        nf = self.norm_f
        _capi.layernorm(x.contiguous(), nf.weight.float(), nf.bias.float(), nf.eps, n)
        if self.head_proj is not None:
            p = torch.empty(B, self.config.emb_dim, device=h.device, dtype=torch.bfloat16)
            _capi.gemm_skinny(n, self._bf16_weight(self.head_proj), None, p)
            n = p
        out = torch.empty(B, self.config.vocab_size, device=h.device, dtype=torch.bfloat16)
        _capi.gemm_skinny(n, self._bf16_weight(self.head), None, out)
        return out.view(B, 1, -1)

    def forward(self, input_ids: torch.Tensor, states: Optional[List[torch.Tensor]] = None):
        """Prefill over a whole sequence (model.py:82-103); returns logits."""
        h = self._embed(input_ids)
        if states is None:
            states = [None] * len(self.blocks)
        for i, block in enumerate(self.blocks):
            # the residual stream stays float32 between blocks (no bf16 round trip per layer)
            h, _ = block._forward(h, states[i], keep_fp32=True)
        return self._head(h)

    def forward_with_states(self, input_ids: torch.Tensor, states=None):
        """Prefill that also returns each block's final memory state, for decode."""
        h = self._embed(input_ids)
        if states is None:
            states = [None] * len(self.blocks)
        out_states = []
        for i, block in enumerate(self.blocks):
            h, M = block._forward(h, states[i], keep_fp32=True)
            out_states.append(M)
        return self._head(h), out_states

    def step(self, input_id_t: torch.Tensor, states=None) -> Tuple[torch.Tensor, list]:
        """One decode step (model.py:105-128); returns (logits, new_states)."""
        h = self._embed_step(input_id_t)
        if states is None:
            states = [None] * len(self.blocks)
        new_states = []
        for i, block in enumerate(self.blocks):
            # the residual stream stays float32 between blocks (no bf16 round trip per layer)
            h, s = block._step_fresh(h, states[i], keep_fp32=True)
            new_states.append(s)
        return self._head_step(h), new_states

    def print_substrate_report(self):
        print("=" * 72)
        print(f"{'Layer':<10} | {'% FWHT':>10} | {'% DCT-II':>10} | {'% Haar':>10}")
        print("-" * 72)
        for idx, block in enumerate(self.blocks):
            p = block.ffn.get_substrate_probabilities()
            print(f"{idx + 1:<10} | {p[0] * 100:>10.2f} | {p[1] * 100:>10.2f} | {p[2] * 100:>10.2f}")
        print("=" * 72)
