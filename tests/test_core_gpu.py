"""GPU parity of the chunkwise core (dp_core_fwd) against the reference's fp64 path.

Golden vectors come from the reference itself (tests/golden/make_golden.py); the
numpy oracle (pinned to those vectors on CPU) covers the other seeded cases.
Tolerances (relative L2 vs fp64): 2e-3 for float32 inputs, 1e-2 for bfloat16 inputs.
"""
import numpy as np
import pytest
import torch

import delta_phase_b200 as dp
from delta_phase_b200.kernels import chunkwise_forward
from oracle import core as ocore

from helpers import TOL_BF16, TOL_F32, core_inputs, load_golden, rel_l2, report, round_bf16, to_dev

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case", ["core_cfg1"] + [f"core_case{i}" for i in range(6)])
def test_golden_fp32(case):
    g = load_golden(case)
    M0 = to_dev(g["M0"]) if "M0" in g else None
    with torch.no_grad():
        out, M = dp.delta_phase_chunkwise_fused(to_dev(g["theta_k"]), to_dev(g["theta_q"]),
                                                to_dev(g["v"]), to_dev(g["beta"]),
                                                int(g["chunk_size"]), M0)
    torch.cuda.synchronize()
    assert out.dtype == torch.float32 and M.dtype == torch.complex64
    assert rel_l2(out, g["out"]) < TOL_F32
    assert rel_l2(M, g["M"]) < TOL_F32
    # the recurrent (token-by-token) definition of the same outputs
    assert rel_l2(out, g["out_rec"]) < TOL_F32
    if M0 is not None:  # the caller's initial state is not modified
        assert torch.equal(M0, to_dev(g["M0"]))


def test_config1_both_oracles():
    """B=2, H=4, L=256, d_k=32, C=32, fp32, seed 0: vs chunkwise and recurrent paths."""
    tk, tq, v, beta = core_inputs(0, 2, 4, 256, 32)
    out, M = dp.delta_phase_chunkwise_fused(to_dev(tk), to_dev(tq), to_dev(v), to_dev(beta), 32)
    ref_out, ref_M = ocore.chunkwise_delta(tk, tq, v, beta, 32)
    rec_out, rec_M = ocore.recurrent_delta(tk, tq, v, beta)
    assert rel_l2(out, ref_out) < TOL_F32 and rel_l2(M, ref_M) < TOL_F32
    assert rel_l2(out, rec_out) < TOL_F32 and rel_l2(M, rec_M) < TOL_F32


@pytest.mark.parametrize("D,C,L", [(64, 64, 512), (64, 64, 1000), (32, 32, 96), (16, 8, 40),
                                   (128, 64, 128), (48, 16, 77), (1, 4, 9)])
def test_bf16_inputs(D, C, L):
    tk, tq, v, beta = core_inputs(7 + D + L, 2, 3, L, D)
    tk, tq, v, beta = (round_bf16(a) for a in (tk, tq, v, beta))
    out, M = chunkwise_forward(to_dev(tk, torch.bfloat16), to_dev(tq, torch.bfloat16),
                               to_dev(v, torch.bfloat16), to_dev(beta, torch.bfloat16), C)
    ref_out, ref_M = ocore.recurrent_delta(tk, tq, v, beta)
    assert rel_l2(out, ref_out) < TOL_BF16
    assert rel_l2(M, ref_M) < TOL_BF16


@pytest.mark.parametrize("L", [1, 31, 32, 33, 64, 100])
def test_ragged_lengths_and_init_state(L):
    """Any L (the block's padded tail) with a random non-zero complex initial state."""
    rng = np.random.default_rng(L)
    B, H, D = 2, 2, 32
    tk, tq, v, beta = core_inputs(L, B, H, L, D)
    M0 = (rng.standard_normal((B, H, D, D)) + 1j * rng.standard_normal((B, H, D, D))).astype(np.complex64)
    out, M = chunkwise_forward(to_dev(tk), to_dev(tq), to_dev(v), to_dev(beta), 32, to_dev(M0))
    ref_out, ref_M = ocore.recurrent_delta(tk, tq, v, beta, M0)
    assert rel_l2(out, ref_out) < TOL_F32
    assert rel_l2(M, ref_M) < TOL_F32


def test_zero_length_returns_initial_state():
    M0 = torch.randn(1, 2, 8, 8, dtype=torch.complex64, device="cuda")
    z = torch.zeros(1, 2, 0, 8, device="cuda")
    out, M = chunkwise_forward(z, z, z, torch.zeros(1, 2, 0, device="cuda"), 4, M0)
    assert out.shape == (1, 2, 0, 8)
    assert torch.equal(M, M0)


def test_beta_zero_leaves_state_unchanged():
    tk, tq, v, beta = core_inputs(3, 1, 2, 64, 16)
    beta[:] = 0
    M0 = torch.randn(1, 2, 16, 16, dtype=torch.complex64, device="cuda")
    out, M = chunkwise_forward(to_dev(tk), to_dev(tq), to_dev(v), to_dev(beta), 16, M0)
    assert torch.allclose(M, M0)
    ref_out, _ = ocore.recurrent_delta(tk, tq, v, beta, M0.cpu().numpy())
    assert rel_l2(out, ref_out) < TOL_F32


def test_strided_block_layout():
    """(B, L, H, D) projections viewed as (B, H, L, D), output written into (B, L, H*D)."""
    B, L, H, D = 2, 70, 4, 16
    rng = np.random.default_rng(5)
    tk = to_dev(rng.uniform(0, 6.28, (B, L, H, D)).astype(np.float32))
    tq = to_dev(rng.uniform(0, 6.28, (B, L, H, D)).astype(np.float32))
    v = to_dev(rng.standard_normal((B, L, H, D)).astype(np.float32))
    beta = to_dev(rng.uniform(0, 2, (B, L, H)).astype(np.float32))
    buf = torch.empty(B, L, H * D, device="cuda")
    chunkwise_forward(tk.transpose(1, 2), tq.transpose(1, 2), v.transpose(1, 2),
                      beta.transpose(1, 2), 16, out=buf.view(B, L, H, D).transpose(1, 2))
    ref, _ = ocore.recurrent_delta(tk.transpose(1, 2).cpu().numpy(), tq.transpose(1, 2).cpu().numpy(),
                                   v.transpose(1, 2).cpu().numpy(), beta.transpose(1, 2).cpu().numpy())
    assert rel_l2(buf.view(B, L, H, D).transpose(1, 2), ref) < TOL_F32


@pytest.mark.parametrize("L", [64, 200, 256])
def test_strided_projection_views_tensor_core(L):
    """bf16 d_k = 64 inputs as column slices of one (B, L, 3 H 64 + H) projection (the
    block's layout): the tensor-core kernel loads them through TMA tensor maps; the result
    equals the same inputs made contiguous (identical arithmetic) and the oracle."""
    B, H, D = 2, 8, 64  # row width 3 H 64 + H = 1544: token stride a multiple of 8 (tensor-core path)
    rng = np.random.default_rng(L)
    proj = np.concatenate([rng.uniform(0, 6.28, (B, L, 2 * H * D)), rng.standard_normal((B, L, H * D)),
                           rng.standard_normal((B, L, H))], -1)
    proj = round_bf16(proj.astype(np.float32))
    pd = to_dev(proj, torch.bfloat16)
    views = [pd[..., i * H * D:(i + 1) * H * D].view(B, L, H, D).transpose(1, 2) for i in range(3)]
    beta = to_dev(rng.uniform(0, 2, (B, H, L)).astype(np.float32))
    out_s, M_s = chunkwise_forward(*views, beta, 64)
    out_c, M_c = chunkwise_forward(*[t.contiguous() for t in views], beta, 64)
    assert torch.equal(out_s, out_c) and torch.equal(M_s, M_c)
    ref, _ = ocore.recurrent_delta(*[t.float().cpu().numpy() for t in views], beta.cpu().numpy())
    assert rel_l2(out_s, ref) < TOL_BF16


@pytest.mark.parametrize("L", [64, 200, 1000])
def test_tensor_core_output_layouts(L):
    """The pipelined tensor-core kernel (real beta, d_k = 64, bf16) writes its outputs with
    bulk tensor stores (tokens past L clipped by the tensor map): a transposed (B, L, H, Dv)
    output and one with padded rows give the same bits as a contiguous output, with a random
    initial state, and leave the padding alone; an output whose rows are not 16-byte
    multiples goes to the CUDA-core kernel.  All match the oracle."""
    B, H, D = 2, 3, 64
    rng = np.random.default_rng(100 + L)
    tk, tq, v, beta = core_inputs(40 + L, B, H, L, D)
    tk, tq, v, beta = (round_bf16(a) for a in (tk, tq, v, beta))
    M0 = (0.3 * (rng.standard_normal((B, H, D, D)) + 1j * rng.standard_normal((B, H, D, D)))).astype(np.complex64)
    args = [to_dev(a, torch.bfloat16) for a in (tk, tq, v)] + [to_dev(beta)]
    out_c, M_c = chunkwise_forward(*args, 64, to_dev(M0))
    # (B, L, H, Dv) buffer viewed as (B, H, L, Dv): token stride H * 64 floats (tensor map)
    buf = torch.empty(B, L, H, D, device="cuda")
    out_t, M_t = chunkwise_forward(*args, 64, to_dev(M0), out=buf.transpose(1, 2))
    # token stride 68 floats: padded rows, still a tensor map; the padding is never written
    pad = torch.full((B, H, L, D + 4), float("nan"), device="cuda")
    out_p, M_p = chunkwise_forward(*args, 64, to_dev(M0), out=pad[..., :D])
    # token stride 65 floats (not 16-byte rows): the CUDA-core kernel takes the call
    odd = torch.full((B, H, L, D + 1), float("nan"), device="cuda")
    out_o, M_o = chunkwise_forward(*args, 64, to_dev(M0), out=odd[..., :D])
    assert torch.equal(out_t, out_c) and torch.equal(M_t, M_c)
    assert torch.equal(out_p, out_c) and torch.equal(M_p, M_c)
    assert torch.isnan(pad[..., D:]).all() and torch.isnan(odd[..., D]).all()
    ref_out, ref_M = ocore.recurrent_delta(tk, tq, v, beta, M0)
    for o, m in ((out_c, M_c), (out_o, M_o)):
        assert rel_l2(o, ref_out) < TOL_BF16 and rel_l2(m, ref_M) < TOL_BF16


def test_dispatcher_contract():
    tk, tq, v, beta = core_inputs(1, 1, 2, 30, 8)
    with pytest.raises(RuntimeError):  # L not a multiple of chunk_size, as in the reference
        dp.delta_phase_chunkwise_fused(to_dev(tk), to_dev(tq), to_dev(v), to_dev(beta), 16)
    with pytest.raises(RuntimeError):  # CPU tensors are rejected: no CPU fallback
        dp.delta_phase_chunkwise_fused(torch.from_numpy(tk), torch.from_numpy(tq),
                                       torch.from_numpy(v), torch.from_numpy(beta), 10)
    with pytest.raises(TypeError):
        dp.delta_phase_chunkwise_fused(to_dev(tk).double(), to_dev(tq).double(),
                                       to_dev(v).double(), to_dev(beta).double(), 10)
    x = to_dev(tk).requires_grad_(True)
    out, _ = dp.delta_phase_chunkwise_fused(x, to_dev(tq), to_dev(v), to_dev(beta), 10)
    out.sum().backward()  # the backward kernel (tests/test_backward_gpu.py checks its values)
    assert x.grad is not None and x.grad.shape == x.shape and torch.isfinite(x.grad).all()


def test_full_length_slice_parity_bf16():
    """Full-length (L = 8192, d_k = 64) units of the B=8, H=16 workload vs the fp64 oracle."""
    tk, tq, v, beta = core_inputs(0, 1, 2, 8192, 64)
    tk, tq, v, beta = (round_bf16(a) for a in (tk, tq, v, beta))
    out, M = chunkwise_forward(to_dev(tk, torch.bfloat16), to_dev(tq, torch.bfloat16),
                               to_dev(v, torch.bfloat16), to_dev(beta, torch.bfloat16), 64)
    ref_out, ref_M = ocore.chunkwise_delta(tk, tq, v, beta, 64)
    e_out, e_M = rel_l2(out, ref_out), rel_l2(M, ref_M)
    report("core_bf16_L8192", out=e_out, M=e_M)
    assert e_out < TOL_BF16
    assert e_M < TOL_BF16


def _b8h16_l8192_inputs(seed=0, B=8, H=16, L=8192, D=64):
    g = torch.Generator(device="cuda").manual_seed(seed)
    tk = (torch.rand(B, H, L, D, device="cuda", generator=g) * 2 * np.pi).to(torch.bfloat16)
    tq = (torch.rand(B, H, L, D, device="cuda", generator=g) * 2 * np.pi).to(torch.bfloat16)
    v = torch.randn(B, H, L, D, device="cuda", generator=g).to(torch.bfloat16)
    beta = (2 * torch.sigmoid(torch.randn(B, H, L, device="cuda", generator=g))).to(torch.bfloat16)
    return tk, tq, v, beta


def test_b8h16_l8192_properties():
    """Size-independent checks at the full B=8, H=16, L=8192, d_k=64 workload:
    (b, h) units are independent, the result is linear in v (zero initial state), and
    a split sequence with state hand-off equals the single pass."""
    tk, tq, v, beta = _b8h16_l8192_inputs()
    out, M = chunkwise_forward(tk, tq, v, beta, 64)
    assert torch.isfinite(out).all() and torch.isfinite(torch.view_as_real(M)).all()
    for (b, h) in [(0, 0), (3, 7), (7, 15)]:
        o1, M1 = chunkwise_forward(tk[b:b + 1, h:h + 1], tq[b:b + 1, h:h + 1],
                                   v[b:b + 1, h:h + 1], beta[b:b + 1, h:h + 1], 64)
        assert rel_l2(o1[0, 0], out[b, h]) < 1e-6
        assert rel_l2(M1[0, 0], M[b, h]) < 1e-6
    # linearity: out(v1 + v2) = out(v1) + out(v2)  (phases and beta fixed, M0 = 0)
    v2 = torch.roll(v, 1, dims=2)
    o_a, _ = chunkwise_forward(tk, tq, v, beta, 64)
    o_b, _ = chunkwise_forward(tk, tq, v2, beta, 64)
    v_sum = (v.float() + v2.float())
    o_ab, _ = chunkwise_forward(tk.float(), tq.float(), v_sum, beta.float(), 64)
    assert rel_l2(o_ab, o_a + o_b) < TOL_BF16
    # split hand-off
    h = 4096
    o_1, M_1 = chunkwise_forward(tk[:, :, :h], tq[:, :, :h], v[:, :, :h], beta[:, :, :h], 64)
    o_2, M_2 = chunkwise_forward(tk[:, :, h:], tq[:, :, h:], v[:, :, h:], beta[:, :, h:], 64, M_1)
    assert rel_l2(torch.cat([o_1, o_2], 2), out) < 1e-3
    assert rel_l2(M_2, M) < 1e-3


@pytest.mark.parametrize("N,C,D", [(3, 8, 16), (4, 16, 16), (4, 32, 48), (2, 64, 64), (2, 64, 96)])
def test_gram_golden(N, C, D):
    g = load_golden("gram")
    i = [(3, 8, 16), (4, 16, 16), (4, 32, 48), (2, 64, 64), (2, 64, 96)].index((N, C, D))
    G = dp.gram_matrix_cuda(to_dev(g[f"theta{i}"]), to_dev(g[f"beta{i}"]))
    assert float((G.cpu() - torch.from_numpy(g[f"gram{i}"]).float()).abs().max()) < 1e-3
    assert float(torch.triu(G, 0).abs().max()) == 0.0


def test_no_device_side_timeouts_recorded():
    from delta_phase_b200 import _capi
    assert _capi.device_error(clear=True) == 0


def test_phasor_matches_cuda_sincos():
    """The FMA-pipe sin/cos (Cody-Waite + Taylor) against CUDA's own sin/cos."""
    from delta_phase_b200.kernels import phasor
    x = torch.linspace(-20, 20, 400001, device="cuda")
    z = phasor(x)
    assert float((z.real - torch.cos(x)).abs().max()) < 4e-6
    assert float((z.imag - torch.sin(x)).abs().max()) < 4e-6
    xb = (torch.rand(1 << 16, device="cuda") * 2 * np.pi).to(torch.bfloat16)
    zb = phasor(xb)
    assert float((zb.real - torch.cos(xb.float())).abs().max()) < 1e-6
