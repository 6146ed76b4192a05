"""The full-model decode step captured as a CUDA graph (delta_phase_b200.decode_graph)
against eager DeltaPhaseModel.step (model.py:105-128) and against prefill."""
import pytest
import torch

import delta_phase_b200 as dp
from delta_phase_b200.decode_graph import DecodeGraph

from helpers import TOL_F32, rel_l2

pytestmark = pytest.mark.gpu


def _model(dim=256, heads=4, layers=2, vocab=300, seed=0):
    torch.manual_seed(seed)
    cfg = dp.DeltaPhaseConfig(dim=dim, n_heads=heads, n_layers=layers, vocab_size=vocab, chunk_size=32)
    return dp.DeltaPhaseModel(cfg).cuda().eval()


@pytest.mark.parametrize("autocast", [None, torch.bfloat16])
def test_graph_matches_eager_steps(autocast):
    model = _model()
    B, L = 3, 40
    ids = torch.randint(0, 300, (B, L + 6), device="cuda")
    with torch.no_grad():
        _, Ms = model.forward_with_states(ids[:, :L])
    g = DecodeGraph(model, B, states=[(None, M) for M in Ms], autocast_dtype=autocast)
    st = [(None, M.clone()) for M in Ms]
    for t in range(L, L + 6):
        with torch.no_grad(), torch.autocast("cuda", dtype=autocast or torch.float32, enabled=autocast is not None):
            le, st = model.step(ids[:, t:t + 1], st)
        lg = g.step(ids[:, t:t + 1])
        assert rel_l2(lg.float(), le.float()) < 1e-5, t
    for (ce, Me), (cg, Mg) in zip(st, g.states()):
        assert rel_l2(Mg, Me) < 1e-5
        assert rel_l2(cg, ce.float()) < 1e-5


def test_graph_decode_reproduces_prefill():
    """Decoding a sequence token by token through the graph gives prefill's last logits."""
    model = _model(dim=128, heads=2, vocab=500, seed=1)
    B, L = 2, 40
    ids = torch.randint(0, 500, (B, L), device="cuda")
    with torch.no_grad():
        logits = model(ids)
    g = DecodeGraph(model, B, autocast_dtype=None)
    for t in range(L):
        lt = g.step(ids[:, t:t + 1])
    assert rel_l2(lt[:, 0], logits[:, -1]) < TOL_F32


def test_step_fast_embedding_and_head(monkeypatch):
    """Under bf16 autocast, model.step's embedding and head run on dp_gemm_skinny /
    dp_layernorm with cached bf16 weights; they agree with the module path (torch
    embedding, nn.LayerNorm, autocast matmuls) to bf16 precision."""
    model = _model(dim=256, heads=4, layers=2, vocab=300, seed=3)
    B = 5
    ids = torch.randint(0, 300, (B, 6), device="cuda")
    outs = {}
    for fast in (True, False):
        if not fast:
            monkeypatch.setattr(type(model), "_step_fast", lambda self, rows, dev: False)
        st = None
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
            for t in range(6):
                lg, st = model.step(ids[:, t:t + 1], st)
        outs[fast] = lg.float()
    assert outs[True].shape == (B, 1, 300)
    assert rel_l2(outs[True], outs[False]) < 2e-2
