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

    def forward(self, input_ids: torch.Tensor, states: Optional[List[torch.Tensor]] = None):
        """Prefill over a whole sequence (model.py:82-103); returns logits."""
        h = self._embed(input_ids)
        if states is None:
            states = [None] * len(self.blocks)
        for i, block in enumerate(self.blocks):
            h, _ = block(h, states[i])
        return self._head(h)

    def forward_with_states(self, input_ids: torch.Tensor, states=None):
        """Prefill that also returns each block's final memory state, for decode."""
        h = self._embed(input_ids)
        if states is None:
            states = [None] * len(self.blocks)
        out_states = []
        for i, block in enumerate(self.blocks):
            h, M = block(h, states[i])
            out_states.append(M)
        return self._head(h), out_states

    def step(self, input_id_t: torch.Tensor, states=None) -> Tuple[torch.Tensor, list]:
        """One decode step (model.py:105-128); returns (logits, new_states)."""
        h = self._embed(input_id_t)
        if states is None:
            states = [None] * len(self.blocks)
        new_states = []
        for i, block in enumerate(self.blocks):
            # the residual stream stays float32 between blocks (no bf16 round trip per layer)
            h, s = block._step_fresh(h, states[i], keep_fp32=True)
            new_states.append(s)
        return self._head(h), new_states

    def print_substrate_report(self):
        print("=" * 72)
        print(f"{'Layer':<10} | {'% FWHT':>10} | {'% DCT-II':>10} | {'% Haar':>10}")
        print("-" * 72)
        for idx, block in enumerate(self.blocks):
            p = block.ffn.get_substrate_probabilities()
            print(f"{idx + 1:<10} | {p[0] * 100:>10.2f} | {p[1] * 100:>10.2f} | {p[2] * 100:>10.2f}")
        print("=" * 72)
