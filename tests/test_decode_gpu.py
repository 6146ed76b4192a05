"""GPU parity of the decode step (dp_core_decode) against the fp64 oracle
(the step of DeltaPhaseHolographicBlock.step, layers.py:279-285)."""
import numpy as np
import pytest
import torch

import delta_phase_b200 as dp
from oracle import core as ocore

from helpers import TOL_BF16, TOL_F32, rel_l2, round_bf16, to_dev

pytestmark = pytest.mark.gpu


def _inputs(seed, B, H, D):
    rng = np.random.default_rng(seed)
    M = (rng.standard_normal((B, H, D, D)) + 1j * rng.standard_normal((B, H, D, D))).astype(np.complex64)
    k = rng.uniform(0, 2 * np.pi, (B, H, D)).astype(np.float32)
    q = rng.uniform(0, 2 * np.pi, (B, H, D)).astype(np.float32)
    v = rng.standard_normal((B, H, D)).astype(np.float32)
    b = rng.uniform(0, 2, (B, H)).astype(np.float32)
    return M, k, q, v, b


@pytest.mark.parametrize("B,H,D", [(2, 4, 64), (1, 1, 1), (3, 2, 33), (2, 2, 128), (1, 3, 300), (8, 16, 64)])
def test_decode_fp32(B, H, D):
    M, k, q, v, b = _inputs(D, B, H, D)
    Md = to_dev(M)
    out, Mn = dp.decode_step(Md, to_dev(k), to_dev(q), to_dev(v), to_dev(b))
    ro, rM = ocore.decode_step(M, k, q, v, b)
    assert rel_l2(out, ro) < TOL_F32
    assert rel_l2(Mn, rM) < TOL_F32
    assert torch.equal(Md, to_dev(M))  # input state untouched (fresh output)


def test_decode_in_place_and_bf16():
    M, k, q, v, b = _inputs(1, 2, 4, 64)
    k, q, v, b = (round_bf16(a) for a in (k, q, v, b))
    Md = to_dev(M)
    out, Mn = dp.decode_step(Md, to_dev(k, torch.bfloat16), to_dev(q, torch.bfloat16),
                             to_dev(v, torch.bfloat16), to_dev(b, torch.bfloat16), state_out=Md)
    assert Mn.data_ptr() == Md.data_ptr()
    ro, rM = ocore.decode_step(M, k, q, v, b)
    assert rel_l2(out, ro) < TOL_BF16 and rel_l2(Md, rM) < TOL_BF16


def test_decode_loop_matches_chunkwise():
    """256 decode steps from a prefill state == one chunkwise pass over the whole sequence."""
    rng = np.random.default_rng(3)
    B, H, D, L0, L1 = 2, 3, 64, 128, 256
    tk = rng.uniform(0, 2 * np.pi, (B, H, L0 + L1, D)).astype(np.float32)
    tq = rng.uniform(0, 2 * np.pi, (B, H, L0 + L1, D)).astype(np.float32)
    v = rng.standard_normal((B, H, L0 + L1, D)).astype(np.float32)
    b = rng.uniform(0, 2, (B, H, L0 + L1)).astype(np.float32)
    full, Mfull = dp.delta_phase_chunkwise_fused(to_dev(tk), to_dev(tq), to_dev(v), to_dev(b), 64)
    _, M = dp.delta_phase_chunkwise_fused(to_dev(tk[:, :, :L0]), to_dev(tq[:, :, :L0]),
                                          to_dev(v[:, :, :L0]), to_dev(b[:, :, :L0]), 64)
    outs = []
    for t in range(L0, L0 + L1):
        o, M = dp.decode_step(M, to_dev(tk[:, :, t]), to_dev(tq[:, :, t]), to_dev(v[:, :, t]),
                              to_dev(b[:, :, t]), state_out=M)
        outs.append(o)
    assert rel_l2(torch.stack(outs, 2), full[:, :, L0:]) < TOL_F32
    assert rel_l2(M, Mfull) < TOL_F32


@pytest.mark.parametrize("mode", ["sigmoid2", "one", "phi", "beta"])
@pytest.mark.parametrize("D,gdt", [(64, torch.float32), (33, torch.float32), (128, torch.bfloat16),
                                   (32, torch.bfloat16)])
def test_decode_gated(mode, D, gdt):
    """dp_core_decode_gated reads the raw gate from a strided (B, H) slice of the block's
    projection row and forms beta itself: 2 sigmoid(g) (layers.py:265), 1 (beta_mode
    "fixed", :266-267), 1 + e^{i g} (layers.py:397-398), or g as given."""
    B, H = 3, 4
    M, k, q, v, _ = _inputs(D + 7, B, H, D)
    rng = np.random.default_rng(D)
    proj = rng.standard_normal((B, 3 * H * D + H)).astype(np.float32) * 2.0
    proj = round_bf16(proj) if gdt == torch.bfloat16 else proj
    g = proj[:, 3 * H * D:]
    gate = to_dev(proj, gdt)[:, 3 * H * D:]
    code = {"beta": dp._capi.DP_GATE_BETA, "sigmoid2": dp._capi.DP_GATE_SIGMOID2,
            "one": dp._capi.DP_GATE_ONE, "phi": dp._capi.DP_GATE_PHI}[mode]
    out, Mn = dp.decode_step(to_dev(M), to_dev(k), to_dev(q), to_dev(v), gate, gate_mode=code)
    if mode == "phi":
        ro, rM = ocore.complex_beta_step(M, k, q, v, g)
    else:
        b = {"beta": g, "sigmoid2": 2.0 / (1.0 + np.exp(-g.astype(np.float64))), "one": np.ones_like(g)}[mode]
        ro, rM = ocore.decode_step(M, k, q, v, b)
    assert rel_l2(out, ro) < TOL_F32
    assert rel_l2(Mn, rM) < TOL_F32
