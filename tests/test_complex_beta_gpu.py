"""GPU parity of the complex-beta rule (ComplexBetaDeltaPhaseBlock, beta = 1 + e^{i phi})
against the reference's token loop in fp64.

Golden vectors come from the reference's own block (tests/golden/make_golden.py, forward
hooks record the phases, values and phi its loop consumed and what it returned); the numpy
oracle (pinned to them on CPU) covers the other seeded cases.  The chunkwise kernels
(dp_core_cbeta_fwd: tensor cores for d_k = 64 bf16, CUDA cores otherwise) and the decode
step (dp_core_cbeta_decode) are called through the C ABI.
Tolerances (relative L2 vs fp64): 2e-3 for float32 inputs, 1e-2 for bfloat16 inputs.
"""
import numpy as np
import pytest
import torch

import delta_phase_b200 as dp
from delta_phase_b200.kernels import chunkwise_forward, complex_beta_chunkwise, decode_step
from oracle import block as oblock
from oracle import core as ocore

from helpers import TOL_BF16, TOL_F32, load_golden, rel_l2, report, round_bf16, to_dev

pytestmark = pytest.mark.gpu


def cb_inputs(seed, B, H, L, D, phi_scale=2.0):
    rng = np.random.default_rng(seed)
    tk = rng.uniform(0.0, 2 * np.pi, (B, H, L, D)).astype(np.float32)
    tq = rng.uniform(0.0, 2 * np.pi, (B, H, L, D)).astype(np.float32)
    v = rng.standard_normal((B, H, L, D)).astype(np.float32)
    phi = (phi_scale * rng.standard_normal((B, H, L))).astype(np.float32)
    return tk, tq, v, phi


def rand_state(seed, B, H, D):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((B, H, D, D)) + 1j * rng.standard_normal((B, H, D, D))).astype(np.complex64)


def golden_params(g, i):
    p = f"c{i}_p_"
    return {k[len(p):]: g[k] for k in g.files if k.startswith(p)}


def test_golden_core_fp32():
    """The phases, values and phi the reference's loop consumed -> what it returned."""
    g = load_golden("complex_beta")
    for i in range(int(g["n_cases"])):
        p = f"c{i}_"
        M0 = to_dev(g[p + "M0"].astype(np.complex64)) if p + "M0" in g.files else None
        out, M = complex_beta_chunkwise(to_dev(g[p + "theta_k"], torch.float32), to_dev(g[p + "theta_q"], torch.float32),
                                        to_dev(g[p + "v"], torch.float32), to_dev(g[p + "phi"], torch.float32), M0)
        torch.cuda.synchronize()
        assert rel_l2(out, g[p + "retrieved"]) < TOL_F32
        assert rel_l2(M, g[p + "M"]) < TOL_F32
        if M0 is not None:
            assert torch.equal(M0, to_dev(g[p + "M0"].astype(np.complex64)))


@pytest.mark.parametrize("L,init", [(1, False), (63, True), (64, False), (65, True), (200, False),
                                    (1000, True), (4096, False)])
def test_tensor_core_bf16(L, init):
    """d_k = 64 bf16 inputs: the tcgen05 kernel on fp16 operand tiles (the isometric update
    does not damp rounding errors, which grow like sqrt(L): 1000 and 4096 tokens)."""
    B, H, D = 2, 3, 64
    tk, tq, v, phi = (round_bf16(a) for a in cb_inputs(11 + L, B, H, L, D))
    M0 = rand_state(L, B, H, D) if init else None
    out, M = chunkwise_forward(to_dev(tk, torch.bfloat16), to_dev(tq, torch.bfloat16), to_dev(v, torch.bfloat16),
                               to_dev(phi), 64, None if M0 is None else to_dev(M0), complex_beta=True)
    ref_out, ref_M = ocore.complex_beta_recurrent(tk, tq, v, phi, M0)
    assert rel_l2(out, ref_out) < TOL_BF16
    assert rel_l2(M, ref_M) < TOL_BF16


def test_tensor_core_bf16_full_length():
    """One (b, h) unit at the headline length (L = 8192, d_k = 64, bf16, phi ~ N(0, 1) as in
    the block) against the fp64 token loop (layers.py:346-360).  The isometric update lets
    rounding errors add up along the sequence, so this is the longest-path check."""
    B, H, L, D = 1, 1, 8192, 64
    tk, tq, v, phi = (round_bf16(a) for a in cb_inputs(8192, B, H, L, D, phi_scale=1.0))
    out, M = chunkwise_forward(to_dev(tk, torch.bfloat16), to_dev(tq, torch.bfloat16), to_dev(v, torch.bfloat16),
                               to_dev(phi), 64, None, complex_beta=True)
    ref_out, ref_M = ocore.complex_beta_recurrent(tk, tq, v, phi)
    e_out, e_M = rel_l2(out, ref_out), rel_l2(M, ref_M)
    report("cbeta_bf16_L8192", out=e_out, M=e_M)
    assert e_out < TOL_BF16
    assert e_M < TOL_BF16


def test_tensor_core_bf16_phi():
    """phi given in bfloat16 (the projection's dtype under autocast)."""
    B, H, L, D = 1, 4, 300, 64
    tk, tq, v, phi = (round_bf16(a) for a in cb_inputs(5, B, H, L, D))
    out, M = chunkwise_forward(to_dev(tk, torch.bfloat16), to_dev(tq, torch.bfloat16), to_dev(v, torch.bfloat16),
                               to_dev(phi, torch.bfloat16), 64, None, complex_beta=True)
    ref_out, ref_M = ocore.complex_beta_recurrent(tk, tq, v, phi)
    assert rel_l2(out, ref_out) < TOL_BF16
    assert rel_l2(M, ref_M) < TOL_BF16


@pytest.mark.parametrize("D,L", [(64, 130), (16, 77), (32, 33), (128, 40), (5, 9)])
def test_cuda_core_fp32(D, L):
    """float32 inputs and other head sizes: the CUDA-core kernel."""
    B, H = 2, 2
    tk, tq, v, phi = cb_inputs(3 * D + L, B, H, L, D)
    M0 = rand_state(D, B, H, D)
    out, M = complex_beta_chunkwise(to_dev(tk), to_dev(tq), to_dev(v), to_dev(phi), to_dev(M0))
    ref_out, ref_M = ocore.complex_beta_recurrent(tk, tq, v, phi, M0)
    assert rel_l2(out, ref_out) < TOL_F32
    assert rel_l2(M, ref_M) < TOL_F32


def test_out_of_range_values_are_reported():
    """Values past the fp16 range of the operand tiles set DP_ERR_RANGE (7) in the device
    error word instead of passing silently."""
    from delta_phase_b200 import _capi
    B, H, L, D = 1, 2, 128, 64
    tk, tq, v, phi = cb_inputs(1, B, H, L, D)
    _capi.device_error(clear=True)
    chunkwise_forward(to_dev(tk, torch.bfloat16), to_dev(tq, torch.bfloat16), to_dev(v * 1e6, torch.bfloat16),
                      to_dev(phi), 64, None, complex_beta=True)
    assert _capi.device_error(clear=True) == 7
    chunkwise_forward(to_dev(tk, torch.bfloat16), to_dev(tq, torch.bfloat16), to_dev(v, torch.bfloat16),
                      to_dev(phi), 64, None, complex_beta=True)
    assert _capi.device_error(clear=True) == 0


def test_real_beta_limit():
    """phi = 0 gives beta = 2: the complex-beta kernel then follows the real-beta rule's
    oracle (the holographic block's recurrence at beta = 2)."""
    B, H, L, D = 2, 2, 256, 64
    tk, tq, v, _ = (round_bf16(a) for a in cb_inputs(9, B, H, L, D))
    args = [to_dev(a, torch.bfloat16) for a in (tk, tq, v)]
    out_c, M_c = chunkwise_forward(*args, torch.zeros(B, H, L, device="cuda"), 64, None, complex_beta=True)
    ref_out, ref_M = ocore.recurrent_delta(tk, tq, v, np.full((B, H, L), 2.0, np.float32))
    assert rel_l2(out_c, ref_out) < TOL_BF16
    assert rel_l2(M_c, ref_M) < TOL_BF16


def test_split_sequence_matches_whole():
    """Size-independent property at a long length: two halves with the state carried equal
    the whole sequence (B=2, H=4, L=8192, d_k=64, bf16)."""
    B, H, L, D = 2, 4, 8192, 64
    g = torch.Generator(device="cuda").manual_seed(0)
    tk = (torch.rand(B, H, L, D, device="cuda", generator=g) * 6.2832).bfloat16()
    tq = (torch.rand(B, H, L, D, device="cuda", generator=g) * 6.2832).bfloat16()
    v = torch.randn(B, H, L, D, device="cuda", generator=g).bfloat16()
    phi = torch.randn(B, H, L, device="cuda", generator=g) * 2
    out, M = chunkwise_forward(tk, tq, v, phi, 64, None, complex_beta=True)
    h = 3000  # not a chunk multiple
    o1, M1 = chunkwise_forward(tk[:, :, :h], tq[:, :, :h], v[:, :, :h], phi[:, :, :h], 64, None, complex_beta=True)
    o2, M2 = chunkwise_forward(tk[:, :, h:], tq[:, :, h:], v[:, :, h:], phi[:, :, h:], 64, M1, complex_beta=True)
    assert rel_l2(torch.cat([o1, o2], 2), out) < 1e-2
    assert rel_l2(M2, M) < 1e-2
    assert torch.isfinite(out).all()


@pytest.mark.parametrize("D", [64, 16, 96, 7])
def test_decode_step(D):
    B, H = 3, 4
    tk, tq, v, phi = cb_inputs(D, B, H, 1, D)
    tk, tq, v, phi = tk[:, :, 0], tq[:, :, 0], v[:, :, 0], phi[:, :, 0]
    M0 = rand_state(D + 1, B, H, D)
    Md = to_dev(M0)
    out, Mn = decode_step(Md, to_dev(tk), to_dev(tq), to_dev(v), to_dev(phi), complex_beta=True)
    ref_out, ref_M = ocore.complex_beta_step(M0, tk, tq, v, phi)
    assert rel_l2(out, ref_out) < 1e-5
    assert rel_l2(Mn, ref_M) < 1e-5
    assert torch.equal(Md, to_dev(M0))  # not in place unless asked
    decode_step(Md, to_dev(tk), to_dev(tq), to_dev(v), to_dev(phi), state_out=Md, complex_beta=True)
    assert rel_l2(Md, ref_M) < 1e-5


def test_block_golden_forward_and_step():
    """ComplexBetaDeltaPhaseBlock with the reference's weights: forward and step loop."""
    g = load_golden("complex_beta")
    H = int(g["n_heads"])
    for i in range(int(g["n_cases"])):
        p = f"c{i}_"
        blk = dp.ComplexBetaDeltaPhaseBlock(d_model=64, n_heads=H).cuda().eval()
        sd = {k: torch.from_numpy(np.asarray(v)) for k, v in golden_params(g, i).items()}
        blk.load_state_dict({k: v.float() for k, v in sd.items()})
        x = to_dev(g[p + "x"], torch.float32)
        M0 = to_dev(g[p + "M0"].astype(np.complex64)) if p + "M0" in g.files else None
        with torch.no_grad():
            out, M = blk(x, memory_state=M0)
            st = None if M0 is None else (None, M0)
            outs = []
            for t in range(x.shape[1]):
                o, st = blk.step(x[:, t:t + 1], st)
                outs.append(o)
        assert rel_l2(out, g[p + "out"]) < TOL_F32
        assert rel_l2(M, g[p + "M"]) < TOL_F32
        assert rel_l2(torch.cat(outs, 1), g[p + "out_step"]) < TOL_F32
        assert rel_l2(st[1], g[p + "M_step"]) < TOL_F32
        assert blk.last_beta.dtype == torch.complex64 and blk.last_beta.shape == (2, H, 1)


def test_block_bf16_autocast_head64():
    """d_model 512, 8 heads of 64 under bf16 autocast: the tensor-core path inside the
    block (the projection rows, 3 * 512 + 8 values, keep 16-byte alignment), against the
    oracle block on the same weights."""
    torch.manual_seed(3)
    blk = dp.ComplexBetaDeltaPhaseBlock(d_model=512, n_heads=8).cuda().eval()
    x = torch.randn(2, 150, 512, device="cuda")
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        out, M = blk(x)
    params = {k: v.detach().double().cpu().numpy() for k, v in blk.state_dict().items()}
    ref_out, ref_M = oblock.cb_block_forward(x.cpu().numpy(), params, n_heads=8)
    assert rel_l2(out, ref_out) < 2e-2
    assert rel_l2(M, ref_M) < 5e-2


def test_model_complex_beta_prefill_matches_steps():
    """DeltaPhaseModel(beta_mode="complex"): prefill logits equal the step loop's."""
    cfg = dp.DeltaPhaseConfig(dim=128, emb_dim=32, n_layers=2, n_heads=2, vocab_size=300, chunk_size=32,
                              beta_mode="complex")
    torch.manual_seed(0)
    model = dp.DeltaPhaseModel(cfg).cuda().eval()
    assert all(isinstance(b, dp.ComplexBetaDeltaPhaseBlock) for b in model.blocks)
    ids = torch.randint(0, 300, (2, 40), device="cuda")
    with torch.no_grad():
        logits = model(ids)
        st = None
        outs = []
        for t in range(ids.shape[1]):
            lg, st = model.step(ids[:, t:t + 1], st)
            outs.append(lg)
    assert rel_l2(torch.cat(outs, 1), logits) < 1e-3


def test_decode_graph_complex_beta():
    """The CUDA-graph decode loop on complex-beta layers equals the eager step loop."""
    cfg = dp.DeltaPhaseConfig(dim=128, emb_dim=32, n_layers=2, n_heads=2, vocab_size=300, beta_mode="complex")
    torch.manual_seed(1)
    model = dp.DeltaPhaseModel(cfg).cuda().eval()
    ids = torch.randint(0, 300, (2, 12), device="cuda")
    with torch.no_grad():
        st = None
        ref = []
        for t in range(ids.shape[1]):
            lg, st = model.step(ids[:, t:t + 1], st)
            ref.append(lg)
        graph = dp.DecodeGraph(model, batch=2, autocast_dtype=None)
        got = [graph.step(ids[:, t:t + 1]).clone() for t in range(ids.shape[1])]
    assert rel_l2(torch.cat(got, 1), torch.cat(ref, 1)) < 1e-4
