"""GPU parity of the LaplacePhaseCore training path: dp_laplace_bwd (through
LaplaceCudaFunction) and the module's parameter gradients against gradients of the reference.

Golden gradients come from the reference itself (tests/golden/laplace_grad.npz: autograd
of its chunk loop in float64, with _project patched to build K, Q, v, beta and r from
leaf tensors, and every parameter of a LaplacePhaseCore for a seeded loss);
oracle.autograd.laplace_grads (pinned to them on CPU) gives the other seeded cases.
Tolerances (relative L2 vs float64): 2e-3 for float32 inputs, 1e-2 for bfloat16 inputs.
"""
import numpy as np
import pytest
import torch

import delta_phase_b200 as dp
from delta_phase_b200.kernels import LaplaceCudaFunction, laplace_chunkwise
from oracle import autograd as oag

from helpers import TOL_BF16, TOL_F32, load_golden, rel_l2, round_bf16, to_dev

pytestmark = pytest.mark.gpu

NAMES = ("theta_k", "logmag_k", "theta_q", "logmag_q", "v", "log_decay", "beta")


def run_bwd(inputs, dout, dM=None, M0=None, dtype=torch.float32, C=32):
    ins = [to_dev(np.asarray(a), torch.float32 if n == "beta" else dtype).requires_grad_(True)
           for n, a in zip(NAMES, inputs)]
    m0 = None if M0 is None else to_dev(np.asarray(M0).astype(np.complex64)).requires_grad_(True)
    out, M = LaplaceCudaFunction.apply(*ins, C, m0)
    outs, gos = [out], [to_dev(np.asarray(dout), torch.float32)]
    if dM is not None:
        outs.append(M)
        gos.append(to_dev(np.asarray(dM).astype(np.complex64)))
    grads = torch.autograd.grad(outs, ins + ([m0] if m0 is not None else []), gos)
    torch.cuda.synchronize()
    return grads


def test_golden_core_gradients():
    g = load_golden("laplace_grad")
    for i in range(int(g["n_cases"])):
        p = f"c{i}_"
        M0 = g[p + "M0"] if p + "M0" in g.files else None
        grads = run_bwd([g[p + n] for n in NAMES], g[p + "dout"], g[p + "dM"], M0, C=int(g[p + "C"]))
        for k, n in enumerate(NAMES):
            assert rel_l2(grads[k], g[p + "d_" + n]) < TOL_F32, (i, n)
        if M0 is not None:
            assert rel_l2(grads[7], g[p + "d_M0"]) < TOL_F32


def _inputs(seed, B, H, L, D, strong=False):
    rng = np.random.default_rng(seed)
    ld = -np.log1p(np.exp(rng.standard_normal((B, H, L, D)) * (3.0 if strong else 1.0)))
    return [rng.uniform(0, 2 * np.pi, (B, H, L, D)), -0.5 * rng.random((B, H, L, D)),
            rng.uniform(0, 2 * np.pi, (B, H, L, D)), -0.5 * rng.random((B, H, L, D)),
            rng.standard_normal((B, H, L, D)), ld, 2.0 / (1.0 + np.exp(-rng.standard_normal((B, H, L))))]


@pytest.mark.parametrize("D,L,strong", [(64, 100, False), (16, 77, True), (5, 9, False)])
def test_fp32_vs_autograd_oracle(D, L, strong):
    B, H = 2, 2
    ins = [a.astype(np.float32) for a in _inputs(D + L, B, H, L, D, strong)]
    rng = np.random.default_rng(1)
    dout = rng.standard_normal((B, H, L, D)).astype(np.float32)
    M0 = (rng.standard_normal((B, H, D, D)) + 1j * rng.standard_normal((B, H, D, D))).astype(np.complex64)
    dM = (rng.standard_normal((B, H, D, D)) + 1j * rng.standard_normal((B, H, D, D))).astype(np.complex64)
    grads = run_bwd(ins, dout, dM, M0)
    ref = oag.laplace_grads(*ins, dout, dM, M0)
    for k in range(8):
        assert rel_l2(grads[k], ref[k]) < TOL_F32, k


def test_bf16_inputs_tensor_core_forward():
    """bf16 inputs at d_k = 64: the forward runs on the tensor-core kernel, the backward in fp32."""
    B, H, L, D = 1, 2, 200, 64
    ins = _inputs(3, B, H, L, D)
    ins = [round_bf16(a) if n != "beta" else a.astype(np.float32) for n, a in zip(NAMES, ins)]
    dout = np.random.default_rng(2).standard_normal((B, H, L, D)).astype(np.float32)
    grads = run_bwd(ins, dout, None, None, dtype=torch.bfloat16, C=64)
    ref = oag.laplace_grads(*ins, dout)
    for k in range(7):
        assert rel_l2(grads[k].float(), ref[k]) < TOL_BF16, k


def test_functional_api_records_gradients():
    ins = [to_dev(a.astype(np.float32)).requires_grad_(True) for a in _inputs(5, 1, 2, 40, 16)]
    out, M = laplace_chunkwise(*ins, chunk_size=16)
    out.sum().backward()
    for t in ins:
        assert t.grad is not None and torch.isfinite(t.grad).all()


def test_module_parameter_gradients():
    """LaplacePhaseCore training step: every parameter's gradient against the reference's
    (w_sigma_k scaled by 3 to stress the decay, as the reference's own test does)."""
    g = load_golden("laplace_grad")
    core = dp.LaplacePhaseCore(d_model=32, n_heads=2, d_k=16, chunk_size=8)
    core.load_state_dict({k[len("mod_p_"):]: torch.from_numpy(np.asarray(g[k])).float()
                          for k in g.files if k.startswith("mod_p_")})
    core = core.cuda().train()
    x = to_dev(g["mod_x"], torch.float32)
    M0 = to_dev(g["mod_M0"].astype(np.complex64)).requires_grad_(True)
    out, M = core(x, memory_state=M0)
    loss = (out * to_dev(g["mod_R"], torch.float32)).sum() + \
        (torch.conj(to_dev(g["mod_dM"].astype(np.complex64))) * M).real.sum()
    loss.backward()
    assert rel_l2(out, g["mod_out"]) < TOL_F32
    assert rel_l2(M, g["mod_M"]) < TOL_F32
    assert rel_l2(M0.grad, g["mod_d_M0"]) < TOL_F32
    for name, prm in core.named_parameters():
        assert rel_l2(prm.grad, g["mod_g_" + name]) < TOL_F32, name
