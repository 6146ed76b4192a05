"""GPU parity of the training path: dp_core_bwd (through DeltaPhaseCudaFunction) and the
blocks' backward against gradients of the reference.

Golden gradients come from the reference itself (tests/golden/grad.npz: autograd of its
chunkwise path and of both blocks in float64); oracle.autograd (pinned to them on CPU)
gives the other seeded cases.  Tolerances (relative L2 vs float64): 2e-3 for float32
inputs, 1e-2 for bfloat16 inputs (the forward then runs on the tensor-core kernel).
"""
import numpy as np
import pytest
import torch

import delta_phase_b200 as dp
from delta_phase_b200.kernels import DeltaPhaseCudaFunction, delta_phase_chunkwise_fused
from oracle import autograd as oag

from helpers import TOL_BF16, TOL_F32, load_golden, rel_l2, round_bf16, to_dev

pytestmark = pytest.mark.gpu


def _req(a, dtype=torch.float32):
    return to_dev(np.asarray(a), dtype).requires_grad_(True)


def _cplx(a):
    return to_dev(np.asarray(a).astype(np.complex64))


def run_core_bwd(tk, tq, v, g, dout, dM=None, M0=None, dtype=torch.float32, complex_beta=False, C=64):
    ins = [_req(a, dtype) for a in (tk, tq, v)] + [_req(g)]
    m0 = None if M0 is None else _cplx(M0).requires_grad_(True)
    out, M = DeltaPhaseCudaFunction.apply(*ins, C, m0, complex_beta)
    outs, gos = [out], [to_dev(np.asarray(dout), torch.float32)]
    if dM is not None:
        outs.append(M)
        gos.append(_cplx(dM))
    grads = torch.autograd.grad(outs, ins + ([m0] if m0 is not None else []), gos)
    torch.cuda.synchronize()
    return grads


def test_golden_real_beta():
    g = load_golden("grad")
    for i in range(int(g["n_cases"])):
        p = f"c{i}_"
        M0 = g[p + "M0"] if p + "M0" in g.files else None
        dM = g[p + "dM"] if p + "dM" in g.files else None
        grads = run_core_bwd(g[p + "theta_k"], g[p + "theta_q"], g[p + "v"], g[p + "beta"], g[p + "dout"], dM, M0,
                             C=int(g[p + "C"]))
        for k, name in enumerate(("d_theta_k", "d_theta_q", "d_v", "d_beta")):
            assert rel_l2(grads[k], g[p + name]) < TOL_F32, (i, name)
        if M0 is not None:
            assert rel_l2(grads[4], g[p + "d_M0"]) < TOL_F32


def test_golden_block_cores():
    """The cores inside the reference's two blocks: their recorded inputs and output
    gradients in, the recorded input gradients out."""
    g = load_golden("grad")
    L = int(g["hb_L"])
    raw = g["hb_gate_raw"]
    sig = 1.0 / (1.0 + np.exp(-raw))
    beta = 2.0 * sig
    beta[:, :, L:] = 0.0
    grads = run_core_bwd(g["hb_theta_k"], g["hb_theta_q"], g["hb_v"], beta, g["hb_dout"], g["hb_dM"], g["hb_M0"])
    for k, name in enumerate(("d_theta_k", "d_theta_q", "d_v")):
        assert rel_l2(grads[k], g["hb_" + name]) < TOL_F32, name
    dbeta = 2.0 * sig * (1.0 - sig)
    dbeta[:, :, L:] = 0.0
    assert rel_l2(grads[3].cpu().numpy() * dbeta, g["hb_d_gate_raw"]) < TOL_F32
    assert rel_l2(grads[4], g["hb_d_M0"]) < TOL_F32
    grads = run_core_bwd(g["cb_theta_k"], g["cb_theta_q"], g["cb_v"], g["cb_gate_raw"], g["cb_dout"], g["cb_dM"],
                         g["cb_M0"], complex_beta=True)
    for k, name in enumerate(("d_theta_k", "d_theta_q", "d_v", "d_gate_raw")):
        assert rel_l2(grads[k], g["cb_" + name]) < TOL_F32, name
    assert rel_l2(grads[4], g["cb_d_M0"]) < TOL_F32


def _inputs(seed, B, H, L, D, complex_beta):
    rng = np.random.default_rng(seed)
    tk = rng.uniform(0, 2 * np.pi, (B, H, L, D)).astype(np.float32)
    tq = rng.uniform(0, 2 * np.pi, (B, H, L, D)).astype(np.float32)
    v = rng.standard_normal((B, H, L, D)).astype(np.float32)
    g = (rng.standard_normal((B, H, L)) if complex_beta
         else 2.0 / (1.0 + np.exp(-rng.standard_normal((B, H, L))))).astype(np.float32)
    dout = rng.standard_normal((B, H, L, D)).astype(np.float32)
    M0 = (rng.standard_normal((B, H, D, D)) + 1j * rng.standard_normal((B, H, D, D))).astype(np.complex64)
    dM = (rng.standard_normal((B, H, D, D)) + 1j * rng.standard_normal((B, H, D, D))).astype(np.complex64)
    return tk, tq, v, g, dout, M0, dM


@pytest.mark.parametrize("complex_beta", [False, True])
@pytest.mark.parametrize("D,L", [(64, 150), (32, 64), (5, 13)])
def test_fp32_vs_autograd_oracle(complex_beta, D, L):
    tk, tq, v, g, dout, M0, dM = _inputs(D + L, 2, 2, L, D, complex_beta)
    grads = run_core_bwd(tk, tq, v, g, dout, dM, M0, complex_beta=complex_beta)
    ref = (oag.complex_beta_grads if complex_beta else oag.core_grads)(tk, tq, v, g, dout, dM, M0)
    for k in range(5):
        assert rel_l2(grads[k], ref[k]) < TOL_F32, k


@pytest.mark.parametrize("complex_beta", [False, True])
def test_bf16_inputs(complex_beta):
    """bf16 phases and values (tensor-core forward, fp32 backward) at d_k = 64."""
    tk, tq, v, g, dout, M0, dM = _inputs(7, 1, 3, 300, 64, complex_beta)
    tk, tq, v = (round_bf16(a) for a in (tk, tq, v))
    grads = run_core_bwd(tk, tq, v, g, dout, dM, None, dtype=torch.bfloat16, complex_beta=complex_beta)
    ref = (oag.complex_beta_grads if complex_beta else oag.core_grads)(tk, tq, v, g, dout, dM, None)
    assert grads[0].dtype == torch.bfloat16
    for k in range(4):
        assert rel_l2(grads[k].float(), ref[k]) < TOL_BF16, k


def test_directional_derivative_long_sequence():
    """Size-independent check at L = 2048: <grad, delta> equals the central difference of
    the loss along a random direction delta (float64 loss of the float32 forward)."""
    B, H, L, D = 1, 2, 2048, 64
    tk, tq, v, g, dout, M0, _ = _inputs(3, B, H, L, D, False)
    dirs = [np.random.default_rng(9 + k).standard_normal(a.shape).astype(np.float32) for k, a in
            enumerate((tk, tq, v))]
    grads = run_core_bwd(tk, tq, v, g, dout, None, M0)
    pred = sum(float((gr.double().cpu().numpy() * d).sum()) for gr, d in zip(grads[:3], dirs))
    eps = 1e-3

    def loss(s):
        args = [to_dev(a + s * d) for a, d in zip((tk, tq, v), dirs)]
        with torch.no_grad():
            out, _ = delta_phase_chunkwise_fused(*args, to_dev(g), 64, _cplx(M0))
        return float((out.double() * to_dev(dout).double()).sum())

    fd = (loss(eps) - loss(-eps)) / (2 * eps)
    assert abs(fd - pred) / abs(pred) < 1e-2


def test_dispatcher_and_no_initial_state():
    """delta_phase_chunkwise_fused with requires_grad inputs returns a differentiable result."""
    tk, tq, v, g, dout, _, _ = _inputs(11, 1, 2, 64, 16, False)
    ins = [_req(a) for a in (tk, tq, v, g)]
    out, M = delta_phase_chunkwise_fused(*ins, chunk_size=16)
    (out * to_dev(dout)).sum().backward()
    ref = oag.core_grads(tk, tq, v, g, dout)
    for t, r in zip(ins, ref):
        assert rel_l2(t.grad, r) < TOL_F32


@pytest.mark.parametrize("kind", ["hb", "cb"])
def test_block_parameter_gradients(kind):
    """Training step of the block: every parameter's gradient against the reference's."""
    g = load_golden("grad")
    p = kind + "_"
    if kind == "hb":
        blk = dp.DeltaPhaseHolographicBlock(d_model=32, n_heads=2, chunk_size=8)
    else:
        blk = dp.ComplexBetaDeltaPhaseBlock(d_model=32, n_heads=2)
    sd = {k[len(p) + 2:]: torch.from_numpy(np.asarray(g[k])).float() for k in g.files if k.startswith(p + "p_")}
    blk.load_state_dict(sd)
    blk = blk.cuda().train()
    x = to_dev(g[p + "x"], torch.float32)
    M0 = _cplx(g[p + "M0"]).requires_grad_(True)
    out, M = blk(x, memory_state=M0)
    loss = (out * to_dev(g[p + "R"], torch.float32)).sum() + (torch.conj(_cplx(g[p + "dM"])) * M).real.sum()
    loss.backward()
    assert rel_l2(out, g[p + "out"]) < TOL_F32
    assert rel_l2(M, g[p + "M"]) < TOL_F32
    assert rel_l2(M0.grad, g[p + "d_M0"]) < TOL_F32
    for name, prm in blk.named_parameters():
        ref = g[p + "g_" + name]
        if np.linalg.norm(ref) == 0:
            assert float(prm.grad.abs().max()) < 1e-6, name
        else:
            assert rel_l2(prm.grad, ref) < TOL_F32, name


def test_model_training_step():
    """DeltaPhaseModel: a training step produces finite gradients for every parameter, and
    one SGD step lowers the loss on a repeated batch."""
    cfg = dp.DeltaPhaseConfig(dim=128, emb_dim=32, n_layers=2, n_heads=2, vocab_size=200, chunk_size=32)
    torch.manual_seed(0)
    model = dp.DeltaPhaseModel(cfg).cuda().train()
    ids = torch.randint(0, 200, (2, 65), device="cuda")
    opt = torch.optim.SGD(model.parameters(), lr=0.5)
    losses = []
    for _ in range(3):
        logits = model(ids[:, :-1])
        loss = torch.nn.functional.cross_entropy(logits.reshape(-1, 200), ids[:, 1:].reshape(-1))
        opt.zero_grad()
        loss.backward()
        for n_, prm in model.named_parameters():
            assert prm.grad is not None and torch.isfinite(prm.grad).all(), n_
        opt.step()
        losses.append(float(loss.detach()))
    assert losses[-1] < losses[0]


@pytest.mark.parametrize("kind", ["hb", "cb"])
def test_block_training_under_bf16_autocast(kind):
    """As the reference's AMP test (tests/test_amp_dtypes.py:31-97): forward and backward
    under bf16 autocast stay finite, and the forward agrees with the float32 step loop
    (the projections run in bf16 there, the core on its tensor-core kernel)."""
    torch.manual_seed(5)
    if kind == "hb":
        blk = dp.DeltaPhaseHolographicBlock(d_model=512, n_heads=8, chunk_size=64)
    else:
        blk = dp.ComplexBetaDeltaPhaseBlock(d_model=512, n_heads=8)
    blk = blk.cuda().train()
    x = torch.randn(2, 130, 512, device="cuda", requires_grad=True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out, M = blk(x)
        loss = out.float().pow(2).mean() + M.abs().pow(2).mean()
    loss.backward()
    assert torch.isfinite(out.float()).all() and torch.isfinite(x.grad).all()
    for name, prm in blk.named_parameters():
        assert prm.grad is not None and torch.isfinite(prm.grad).all(), name
    with torch.no_grad():
        st = None
        outs = []
        for t in range(x.shape[1]):
            o, st = blk.step(x[:, t:t + 1].detach(), st)
            outs.append(o)
    assert rel_l2(out.float(), torch.cat(outs, 1)) < 5e-2
