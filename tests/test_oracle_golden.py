"""Pin the numpy oracle against golden vectors produced by the reference itself
(tests/golden/make_golden.py).  CPU only."""
import os

import numpy as np
import pytest

from oracle import block as oblock
from oracle import core as ocore
from oracle import laplace as olap
from oracle import spectral as ospec

from conftest import GOLDEN


def load(name):
    return np.load(os.path.join(GOLDEN, name + ".npz"))


@pytest.mark.parametrize("case", ["core_cfg1"] + [f"core_case{i}" for i in range(6)])
def test_core_chunkwise_matches_reference(case):
    g = load(case)
    M0 = g["M0"] if "M0" in g else None
    out, M = ocore.chunkwise_delta(g["theta_k"], g["theta_q"], g["v"], g["beta"],
                                   int(g["chunk_size"]), M0)
    tol = 1e-6 if case == "core_cfg1" else 1e-10   # cfg1 golden stored as float32
    assert ocore.rel_l2(out, g["out"]) < tol
    assert ocore.rel_l2(M, g["M"]) < tol


@pytest.mark.parametrize("case", ["core_case0", "core_case2", "core_case4"])
def test_core_recurrent_matches_reference_steps(case):
    g = load(case)
    M0 = g["M0"] if "M0" in g else None
    out, M = ocore.recurrent_delta(g["theta_k"], g["theta_q"], g["v"], g["beta"], M0)
    assert ocore.rel_l2(out, g["out_rec"]) < 1e-10
    assert ocore.rel_l2(M, g["M_rec"]) < 1e-10
    # and the reference's own equivalence: chunkwise == recurrent
    assert ocore.rel_l2(g["out"], g["out_rec"]) < 1e-9


def test_core_L_not_multiple_of_chunk_raises():
    rng = np.random.default_rng(0)
    with pytest.raises(ValueError):
        ocore.chunkwise_delta(rng.random((1, 1, 10, 4)), rng.random((1, 1, 10, 4)),
                              rng.random((1, 1, 10, 4)), rng.random((1, 1, 10)), 4)


def test_gram_matches_reference():
    g = load("gram")
    for i in range(5):
        G = ocore.gram_matrix(g[f"theta{i}"], g[f"beta{i}"])
        np.testing.assert_allclose(G, g[f"gram{i}"], atol=1e-12)
        assert np.abs(np.triu(G)).max() == 0.0


def test_laplace_matches_reference():
    g = load("laplace")
    for i in range(int(g["n_cases"])):
        p = f"c{i}_"
        M0 = g[p + "M0"] if p + "M0" in g else None
        out, M = olap.laplace_chunkwise(g[p + "K"], g[p + "Q"], g[p + "v"], g[p + "beta"],
                                        g[p + "r"], int(g[p + "C"]), M0)
        assert ocore.rel_l2(out, g[p + "out"]) < 1e-10, i
        assert ocore.rel_l2(M, g[p + "M"]) < 1e-10, i
        out_s, M_s = olap.laplace_sequential(g[p + "K"], g[p + "Q"], g[p + "v"], g[p + "beta"],
                                             g[p + "r"], M0)
        assert ocore.rel_l2(out_s, g[p + "out_seq"]) < 1e-10, i
        assert ocore.rel_l2(M_s, g[p + "M_seq"]) < 1e-10, i


def test_laplace_project_matches_reference():
    g = load("laplace")
    for i in (5, 21):
        p = f"c{i}_"
        w = {n: g[p + n] for n in ("w_theta_k", "w_sigma_k", "w_theta_q", "w_sigma_q", "w_v", "w_beta")}
        K, Q, v, beta, r = olap.project(g[p + "x"], w, n_heads=2, d_k=16)
        for a, b in ((K, "K"), (Q, "Q"), (v, "v"), (beta, "beta"), (r, "r")):
            np.testing.assert_allclose(a, g[p + b], rtol=1e-12, atol=1e-12)


def test_spectral_matrices_match_reference():
    g = load("spectral")
    for n in (1, 2, 4, 8, 16, 64, 1024):
        np.testing.assert_array_equal(ospec.hadamard_matrix(n), g[f"fwht{n}"])
        np.testing.assert_array_equal(ospec.haar_matrix(n), g[f"haar{n}"])
        if n <= 64:
            np.testing.assert_allclose(ospec.dct2_matrix(n), g[f"dct{n}"], atol=2e-7)
        else:
            d = ospec.dct2_matrix(n)
            np.testing.assert_allclose(d[g[f"dct{n}_rows"]], g[f"dct{n}_sampled"], atol=2e-7)
            np.testing.assert_allclose(d.astype(np.float64).sum(0), g[f"dct{n}_colsum"], atol=1e-5)
    assert tuple(ospec.hadamard_matrix(768).shape) == tuple(g["fwht768_shape"])
    with pytest.raises(RuntimeError):
        ospec.haar_matrix(768)


def test_ffn_matches_reference():
    g = load("ffn")
    for i in range(int(g["n_cases"])):
        p = f"c{i}_p_"
        params = {k[len(p):]: g[k] for k in g.files if k.startswith(p)}
        y = ospec.lerp_ffn(g[f"c{i}_x"], params)
        np.testing.assert_allclose(y, g[f"c{i}_y"], rtol=1e-10, atol=1e-12)


def test_block_forward_and_step_match_reference():
    g = load("block")
    for i in range(int(g["n_cases"])):
        p = f"c{i}_"
        params = {k[len(p) + 2:]: g[k] for k in g.files if k.startswith(p + "p_")}
        mode = str(g[p + "beta_mode"])
        out, M = oblock.block_forward(g[p + "x"], params, n_heads=4, chunk_size=int(g[p + "C"]),
                                      beta_mode=mode)
        assert ocore.rel_l2(out, g[p + "out"]) < 1e-10
        assert ocore.rel_l2(M, g[p + "M"]) < 1e-10
        x = g[p + "x"]
        st = None
        outs = []
        for t in range(x.shape[1]):
            o, st = oblock.block_step(x[:, t:t + 1], params, n_heads=4, state=st, beta_mode=mode)
            outs.append(o)
        assert ocore.rel_l2(np.concatenate(outs, 1), g[p + "out_step"]) < 1e-10
        assert ocore.rel_l2(st[1], g[p + "M_step"]) < 1e-10
        np.testing.assert_allclose(st[0], g[p + "conv_state"], atol=1e-12)


def test_complex_beta_core_matches_reference():
    """The complex-beta token loop (layers.py:346-360) on the inputs the reference's own
    forward fed it, against what that loop returned."""
    g = load("complex_beta")
    for i in range(int(g["n_cases"])):
        p = f"c{i}_"
        M0 = g[p + "M0"] if p + "M0" in g.files else None
        out, M = ocore.complex_beta_recurrent(g[p + "theta_k"], g[p + "theta_q"], g[p + "v"], g[p + "phi"], M0)
        assert ocore.rel_l2(out, g[p + "retrieved"]) < 1e-12
        assert ocore.rel_l2(M, g[p + "M"]) < 1e-12


def test_complex_beta_block_forward_and_step_match_reference():
    g = load("complex_beta")
    H = int(g["n_heads"])
    for i in range(int(g["n_cases"])):
        p = f"c{i}_"
        params = {k[len(p) + 2:]: g[k] for k in g.files if k.startswith(p + "p_")}
        M0 = g[p + "M0"] if p + "M0" in g.files else None
        out, M = oblock.cb_block_forward(g[p + "x"], params, n_heads=H, memory_state=M0)
        assert ocore.rel_l2(out, g[p + "out"]) < 1e-10
        assert ocore.rel_l2(M, g[p + "M"]) < 1e-10
        x = g[p + "x"]
        st = None if M0 is None else (None, M0)
        outs = []
        for t in range(x.shape[1]):
            o, st = oblock.cb_block_step(x[:, t:t + 1], params, n_heads=H, state=st)
            outs.append(o)
        assert ocore.rel_l2(np.concatenate(outs, 1), g[p + "out_step"]) < 1e-10
        assert ocore.rel_l2(st[1], g[p + "M_step"]) < 1e-10
        np.testing.assert_allclose(st[0], g[p + "conv_state"], atol=1e-12)


def _beta_from_raw(raw, L):
    """beta as the holographic block feeds its core: 2 sigmoid(w_beta(conv_x)), 0 on the
    padded tail (layers.py:192-201); and d beta / d raw."""
    sig = 1.0 / (1.0 + np.exp(-raw))
    beta, dbeta = 2.0 * sig, 2.0 * sig * (1.0 - sig)
    beta[:, :, L:] = 0.0
    dbeta[:, :, L:] = 0.0
    return beta, dbeta


def test_autograd_oracle_matches_reference_gradients():
    """oracle.autograd (token recurrences under torch autograd) against the gradients the
    reference itself produced (chunkwise path and both blocks)."""
    from oracle import autograd as oag
    g = load("grad")
    for i in range(int(g["n_cases"])):
        p = f"c{i}_"
        M0 = g[p + "M0"] if p + "M0" in g.files else None
        dM = g[p + "dM"] if p + "dM" in g.files else None
        d = oag.core_grads(g[p + "theta_k"], g[p + "theta_q"], g[p + "v"], g[p + "beta"], g[p + "dout"], dM, M0)
        for k, name in enumerate(("d_theta_k", "d_theta_q", "d_v", "d_beta")):
            assert ocore.rel_l2(d[k], g[p + name]) < 1e-10, (i, name)
        if M0 is not None:
            assert ocore.rel_l2(d[4], g[p + "d_M0"]) < 1e-10
    # holographic block: beta = 2 sigmoid(raw) with the pad masked
    beta, dbeta = _beta_from_raw(g["hb_gate_raw"], int(g["hb_L"]))
    d = oag.core_grads(g["hb_theta_k"], g["hb_theta_q"], g["hb_v"], beta, g["hb_dout"], g["hb_dM"], g["hb_M0"])
    for k, name in enumerate(("d_theta_k", "d_theta_q", "d_v")):
        assert ocore.rel_l2(d[k], g["hb_" + name]) < 1e-10, name
    assert ocore.rel_l2(d[3] * dbeta, g["hb_d_gate_raw"]) < 1e-10
    assert ocore.rel_l2(d[4], g["hb_d_M0"]) < 1e-10
    # complex-beta block: phi is the raw gate
    d = oag.complex_beta_grads(g["cb_theta_k"], g["cb_theta_q"], g["cb_v"], g["cb_gate_raw"], g["cb_dout"],
                               g["cb_dM"], g["cb_M0"])
    for k, name in enumerate(("d_theta_k", "d_theta_q", "d_v", "d_gate_raw")):
        assert ocore.rel_l2(d[k], g["cb_" + name]) < 1e-10, name
    assert ocore.rel_l2(d[4], g["cb_d_M0"]) < 1e-10


def test_laplace_autograd_oracle_matches_reference_gradients():
    from oracle import autograd as oag
    g = load("laplace_grad")
    names = ("theta_k", "logmag_k", "theta_q", "logmag_q", "v", "log_decay", "beta")
    for i in range(int(g["n_cases"])):
        p = f"c{i}_"
        M0 = g[p + "M0"] if p + "M0" in g.files else None
        d = oag.laplace_grads(*(g[p + n] for n in names), g[p + "dout"], g[p + "dM"], M0)
        for k, n in enumerate(names):
            assert ocore.rel_l2(d[k], g[p + "d_" + n]) < 1e-10, (i, n)
        if M0 is not None:
            assert ocore.rel_l2(d[7], g[p + "d_M0"]) < 1e-10
