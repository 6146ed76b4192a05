"""Full-model decode step as one CUDA graph.

``DeltaPhaseModel.step`` (model.py:105-128) runs, per token and per layer, three
LayerNorms, the causal-conv step, four projections, the fused decode kernel, the output
projection and the spectral FFN (DCT GEMM, feature kernel, folded GEMM): a few hundred
small launches per token, so eager decoding is bound by launch and Python overhead.
``DecodeGraph`` captures one whole step once, with the token ids, the per-layer conv
states and the per-layer memory states in static buffers that the step updates in
place, and replays it per token.

The arithmetic is exactly ``DeltaPhaseModel.step``'s (the same module calls, through
the blocks' ``_step_inplace``, for both block kinds).  The buffers belong to the graph: the
states returned by :meth:`states` alias them and change on the next :meth:`step`.
"""
from __future__ import annotations

import torch


class DecodeGraph:
    """Captured decode step of ``model`` for a fixed batch size.

    ``states``: per-layer ``(conv_state or None, M or None)`` to start from (e.g. the
    memory states of ``forward_with_states``); missing entries start at zero.
    ``autocast_dtype``: the dtype of ``torch.autocast`` inside the step (None: off).
    """

    def __init__(self, model, batch: int, states=None, autocast_dtype=torch.bfloat16, warmup: int = 2):
        self.model = model
        self.autocast_dtype = autocast_dtype
        dev = next(model.parameters()).device
        self.ids = torch.zeros(batch, 1, dtype=torch.long, device=dev)
        self.conv, self.mem = [], []
        for i, blk in enumerate(model.blocks):
            d, k = blk.d_model, blk.causal_conv.kernel_size
            conv = torch.zeros(batch, d, k - 1, device=dev, dtype=torch.float32)
            mem = torch.zeros(batch, blk.n_heads, blk.d_k, blk.d_k, device=dev, dtype=torch.complex64)
            if states is not None and states[i] is not None:
                c0, m0 = states[i] if isinstance(states[i], tuple) else (None, states[i])
                if c0 is not None:
                    conv.copy_(c0)
                if m0 is not None:
                    mem.copy_(m0)
            self.conv.append(conv)
            self.mem.append(mem)
        # warm-up on a side stream: library handles, the FFN fold cache and lazily sized
        # workspaces exist before capture; the states are restored afterwards
        saved = [t.clone() for t in self.conv + self.mem]
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(max(1, warmup)):
                self._run()
        torch.cuda.current_stream(dev).wait_stream(side)
        for t, s in zip(self.conv + self.mem, saved):
            t.copy_(s)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.logits = self._run()

    def _run(self):
        m = self.model
        with torch.no_grad(), torch.autocast("cuda", dtype=self.autocast_dtype or torch.float32,
                                             enabled=self.autocast_dtype is not None):
            h = m._embed_step(self.ids)
            for blk, conv, mem in zip(m.blocks, self.conv, self.mem):
                h = blk._step_inplace(h, conv, mem, keep_fp32=True)
            return m._head_step(h)

    def step(self, input_id_t: torch.Tensor) -> torch.Tensor:
        """One token per sequence, ids (B, 1); returns the logits (a static buffer)."""
        self.ids.copy_(input_id_t)
        self.graph.replay()
        return self.logits

    def states(self):
        """Current per-layer ``(conv_state, M)`` (the graph's buffers)."""
        return list(zip(self.conv, self.mem))
