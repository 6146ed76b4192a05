"""GPU parity of the LaplacePhaseCore kernel (dp_laplace_fwd) against the reference
(golden vectors of LaplacePhaseCore.forward / forward_sequential, layers.py:481-583)
and the fp64 oracle."""
import numpy as np
import pytest
import torch

import delta_phase_b200 as dp
from delta_phase_b200 import _capi
from oracle import laplace as olap

from helpers import TOL_BF16, TOL_F32, load_golden, rel_l2, report, round_bf16, to_dev

pytestmark = pytest.mark.gpu


def test_golden_cases():
    g = load_golden("laplace")
    for i in range(int(g["n_cases"])):
        p = f"c{i}_"
        K, Q, r = g[p + "K"], g[p + "Q"], g[p + "r"]
        f32 = lambda a: to_dev(np.ascontiguousarray(a, dtype=np.float32))  # noqa: E731
        M0 = to_dev(g[p + "M0"].astype(np.complex64)) if p + "M0" in g else None
        out, M = dp.laplace_chunkwise(f32(np.angle(K)), f32(np.log(np.abs(K))), f32(np.angle(Q)),
                                      f32(np.log(np.abs(Q))), f32(g[p + "v"]), f32(np.log(r)),
                                      f32(g[p + "beta"]), int(g[p + "C"]), M0)
        assert rel_l2(out, g[p + "out"]) < TOL_F32, i
        assert rel_l2(M, g[p + "M"]) < TOL_F32, i
        assert rel_l2(out, g[p + "out_seq"]) < TOL_F32, i


def test_module_golden():
    g = load_golden("laplace")
    for i in (5, 21):
        p = f"c{i}_"
        core = dp.LaplacePhaseCore(d_model=32, n_heads=2, d_k=16, chunk_size=int(g[p + "C"])).cuda()
        with torch.no_grad():
            for n in ("w_theta_k", "w_sigma_k", "w_theta_q", "w_sigma_q", "w_v", "w_beta"):
                getattr(core, n).weight.copy_(torch.from_numpy(g[p + n]).float())
        x = to_dev(g[p + "x"].astype(np.float32))
        M0 = to_dev(g[p + "M0"].astype(np.complex64)) if p + "M0" in g else None
        with torch.no_grad():
            out, M = core(x, memory_state=M0)
        B, L, _ = x.shape
        ref = g[p + "out"].transpose(0, 2, 1, 3).reshape(B, L, 32)
        assert rel_l2(out, ref) < TOL_F32
        assert rel_l2(M, g[p + "M"]) < TOL_F32


@pytest.mark.parametrize("L,D", [(1000, 64), (333, 16), (64, 128)])
def test_gated_unit_phasors_bf16(L, D):
    """Config-3 style inputs: unit-magnitude K, Q; log r = -softplus(N(0,1)); bf16."""
    rng = np.random.default_rng(L)
    B, H = 1, 2
    tk = round_bf16(rng.uniform(0, 2 * np.pi, (B, H, L, D)))
    tq = round_bf16(rng.uniform(0, 2 * np.pi, (B, H, L, D)))
    v = round_bf16(rng.standard_normal((B, H, L, D)))
    beta = round_bf16(2 / (1 + np.exp(-rng.standard_normal((B, H, L)))))
    logr = round_bf16(-np.logaddexp(0, rng.standard_normal((B, H, L, D))))
    bf = lambda a: to_dev(a, torch.bfloat16)  # noqa: E731
    out, M = dp.laplace_chunkwise(bf(tk), None, bf(tq), None, bf(v), bf(logr), bf(beta), 64)
    K = np.exp(1j * tk.astype(np.float64))
    Q = np.exp(1j * tq.astype(np.float64))
    ref_out, ref_M = olap.laplace_chunkwise(K, Q, v, beta, np.exp(logr.astype(np.float64)), 64)
    assert rel_l2(out, ref_out) < TOL_BF16
    assert rel_l2(M, ref_M) < TOL_BF16


def test_strong_decay_is_finite():
    """Cumulative in-chunk log-decay far below -88: the reference's exp(-S) form
    overflows there; the kernel forms every decay ratio as exp(difference)."""
    rng = np.random.default_rng(0)
    B, H, L, D = 1, 1, 64, 8
    tk = rng.uniform(0, 2 * np.pi, (B, H, L, D)).astype(np.float32)
    tq = rng.uniform(0, 2 * np.pi, (B, H, L, D)).astype(np.float32)
    v = rng.standard_normal((B, H, L, D)).astype(np.float32)
    beta = rng.uniform(0, 2, (B, H, L)).astype(np.float32)
    logr = np.full((B, H, L, D), -5.0, np.float32)
    out, M = dp.laplace_chunkwise(to_dev(tk), None, to_dev(tq), None, to_dev(v), to_dev(logr),
                                  to_dev(beta), 64)
    K = np.exp(1j * tk.astype(np.float64))
    Q = np.exp(1j * tq.astype(np.float64))
    ref_out, ref_M = olap.laplace_sequential(K, Q, v, beta, np.exp(logr.astype(np.float64)))
    assert torch.isfinite(out).all()
    assert rel_l2(out, ref_out) < TOL_F32
    assert rel_l2(M, ref_M) < TOL_F32


def _lap_bf16_inputs(seed, B, H, L, D, with_mag, logr_fill=None):
    rng = np.random.default_rng(seed)
    tk = round_bf16(rng.uniform(0, 2 * np.pi, (B, H, L, D)))
    tq = round_bf16(rng.uniform(0, 2 * np.pi, (B, H, L, D)))
    mk = round_bf16(-np.logaddexp(0, rng.standard_normal((B, H, L, D))) * 0.3) if with_mag else None
    mq = round_bf16(-np.logaddexp(0, rng.standard_normal((B, H, L, D))) * 0.3) if with_mag else None
    v = round_bf16(rng.standard_normal((B, H, L, D)))
    beta = round_bf16(2 / (1 + np.exp(-rng.standard_normal((B, H, L)))))
    if logr_fill is None:
        logr = round_bf16(-np.logaddexp(0, rng.standard_normal((B, H, L, D))))
    else:
        logr = np.full((B, H, L, D), logr_fill, np.float32)
    return tk, mk, tq, mq, v, logr, beta


def _lap_ref(tk, mk, tq, mq, v, logr, beta, M0=None):
    K = np.exp((0 if mk is None else mk.astype(np.float64)) + 1j * tk.astype(np.float64))
    Q = np.exp((0 if mq is None else mq.astype(np.float64)) + 1j * tq.astype(np.float64))
    return olap.laplace_sequential(K, Q, v, beta, np.exp(logr.astype(np.float64)), M0)


@pytest.mark.parametrize("B,H,L,with_mag,with_state,layout", [
    (2, 3, 1, False, False, "bhld"),
    (1, 2, 64, True, True, "bhld"),
    (1, 2, 129, True, True, "blhd"),
    (2, 2, 700, False, True, "blhd"),
    (1, 1, 257, True, False, "bhld"),
])
def test_tensor_core_path(B, H, L, with_mag, with_state, layout):
    """bf16, d_k = d_v = 64: the tcgen05 kernel.  Ragged tails, log-magnitudes, an
    initial state and (B, L, H, D) strided views against the fp64 token loop."""
    D = 64
    tk, mk, tq, mq, v, logr, beta = _lap_bf16_inputs(B * 1000 + L, B, H, L, D, with_mag)
    rng = np.random.default_rng(7)
    M0 = ((rng.standard_normal((B, H, D, D)) + 1j * rng.standard_normal((B, H, D, D))) * 0.5
          if with_state else None)

    def dev(a):
        if a is None:
            return None
        if layout == "blhd" and a.ndim == 4:
            return to_dev(np.ascontiguousarray(a.transpose(0, 2, 1, 3)), torch.bfloat16).transpose(1, 2)
        if layout == "blhd":
            return to_dev(np.ascontiguousarray(a.transpose(0, 2, 1)), torch.bfloat16).transpose(1, 2)
        return to_dev(a, torch.bfloat16)

    M0d = to_dev(M0.astype(np.complex64)) if with_state else None
    out, M = dp.laplace_chunkwise(dev(tk), dev(mk), dev(tq), dev(mq), dev(v), dev(logr), dev(beta), 64, M0d)
    ref_out, ref_M = _lap_ref(tk, mk, tq, mq, v, logr, beta, M0)
    assert rel_l2(out, ref_out) < TOL_BF16
    assert rel_l2(M, ref_M) < TOL_BF16
    assert _capi.device_error(clear=True) == 0


def test_tensor_core_matches_fp32_path():
    """The bf16 tcgen05 kernel and the fp32 CUDA-core kernel on the same values."""
    B, H, L, D = 1, 2, 300, 64
    tk, mk, tq, mq, v, logr, beta = _lap_bf16_inputs(5, B, H, L, D, True)
    args = (tk, mk, tq, mq, v, logr)
    out_tc, M_tc = dp.laplace_chunkwise(*[to_dev(a, torch.bfloat16) for a in args],
                                        to_dev(beta, torch.bfloat16), 64)
    out_f, M_f = dp.laplace_chunkwise(*[to_dev(a) for a in args], to_dev(beta), 64)
    assert rel_l2(out_tc, out_f) < TOL_BF16
    assert rel_l2(M_tc, M_f) < TOL_BF16


def test_tensor_core_strong_decay_is_finite():
    """log r = -5 per step (cumulative -320 per chunk) on the tcgen05 kernel."""
    B, H, L, D = 1, 2, 200, 64
    tk, mk, tq, mq, v, logr, beta = _lap_bf16_inputs(9, B, H, L, D, False, logr_fill=-5.0)
    out, M = dp.laplace_chunkwise(*[to_dev(a, torch.bfloat16) if a is not None else None
                                    for a in (tk, mk, tq, mq, v, logr, beta)], 64)
    ref_out, ref_M = _lap_ref(tk, mk, tq, mq, v, logr, beta)
    assert torch.isfinite(out).all() and torch.isfinite(torch.view_as_real(M)).all()
    assert rel_l2(out, ref_out) < TOL_BF16
    assert rel_l2(M, ref_M) < TOL_BF16


@pytest.mark.parametrize("fill", [-3.5, None])
def test_tensor_core_large_factors_and_mixed_paths(fill):
    """log r = -3.5 per step: block-relative factors up to e^56 on the factorised solve.
    None: ordinary decay with a burst of log r = -6 over tokens 100..139, so some chunks
    take the exact path and the others the factorised one."""
    B, H, L, D = 1, 2, 320, 64
    tk, mk, tq, mq, v, logr, beta = _lap_bf16_inputs(11, B, H, L, D, True, logr_fill=fill)
    if fill is None:
        logr[:, :, 100:140, :] = -6.0
    out, M = dp.laplace_chunkwise(*[to_dev(a, torch.bfloat16) for a in (tk, mk, tq, mq, v, logr, beta)], 64)
    ref_out, ref_M = _lap_ref(tk, mk, tq, mq, v, logr, beta)
    assert torch.isfinite(out).all()
    assert rel_l2(out, ref_out) < TOL_BF16
    assert rel_l2(M, ref_M) < TOL_BF16


def test_tensor_core_full_length_config3():
    """Two (b, h) units of the Laplace workload at full length: L = 32,768 (512 chunks of
    compounding decay), d_k = d_v = 64, bf16, log r = -softplus(N(0, 1)), unit phasors,
    against the fp64 chunkwise oracle (layers.py:481-561); the first 4096 tokens also
    against the fp64 token loop (layers.py:563-583)."""
    B, H, L, D = 1, 2, 32768, 64
    tk, mk, tq, mq, v, logr, beta = _lap_bf16_inputs(32768, B, H, L, D, False)
    out, M = dp.laplace_chunkwise(*[to_dev(a, torch.bfloat16) if a is not None else None
                                    for a in (tk, mk, tq, mq, v, logr, beta)], 64)
    K = np.exp(1j * tk.astype(np.float64))
    Q = np.exp(1j * tq.astype(np.float64))
    ref_out, ref_M = olap.laplace_chunkwise(K, Q, v, beta, np.exp(logr.astype(np.float64)), 64)
    e_out, e_M = rel_l2(out, ref_out), rel_l2(M, ref_M)
    n = 4096
    seq_out, _ = olap.laplace_sequential(K[:, :, :n], Q[:, :, :n], v[:, :, :n], beta[:, :, :n],
                                         np.exp(logr[:, :, :n].astype(np.float64)))
    e_seq = rel_l2(out[:, :, :n], seq_out)
    report("laplace_bf16_L32768", out=e_out, M=e_M, out_seq4096=e_seq)
    assert torch.isfinite(out).all()
    assert e_out < TOL_BF16
    assert e_M < TOL_BF16
    assert e_seq < TOL_BF16
    assert _capi.device_error(clear=True) == 0
