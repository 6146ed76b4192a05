"""Generate the golden vectors in this directory from the reference itself.

Runs the UNMODIFIED reference package (mcarbonell/delta-phase v1.3.0, imported
read-only from the directory given by the REFERENCE_ROOT environment variable, which
is required) on small seeded inputs and stores inputs + reference outputs as .npz.  The
oracle in ``oracle/`` is pinned against these files by tests/test_oracle_golden.py; the
GPU parity tests reuse them.
Usage:  REFERENCE_ROOT=<reference checkout> python tests/golden/make_golden.py [fixture ...]
(default: all of them)
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("REFERENCE_ROOT")
if not REF or not os.path.isdir(os.path.join(REF, "delta_phase")):
    sys.exit("make_golden.py: set REFERENCE_ROOT to a checkout of mcarbonell/delta-phase v1.3.0 "
             "(the directory that holds the delta_phase package)")
sys.path.insert(0, REF)

from delta_phase.kernels.triton_chunk_delta import (  # noqa: E402
    _chunkwise_delta_reference, gram_matrix_reference)
from delta_phase.layers import (  # noqa: E402
    ComplexBetaDeltaPhaseBlock, DeltaPhaseHolographicBlock, LaplacePhaseCore,
    LearnableSubstrateLerpFFN)
from delta_phase.spectral import (  # noqa: E402
    create_dct2_matrix, create_haar_matrix, create_hadamard_matrix)


def save(name, **arrays):
    path = os.path.join(HERE, name + ".npz")
    np.savez_compressed(path, **{k: np.asarray(v) for k, v in arrays.items()})
    print(f"wrote {path} ({os.path.getsize(path) / 1024:.0f} KB)")


def core_inputs(rng, B, H, L, D, Dv=None):
    Dv = D if Dv is None else Dv
    tk = rng.uniform(0.0, 2 * np.pi, (B, H, L, D)).astype(np.float32)
    tq = rng.uniform(0.0, 2 * np.pi, (B, H, L, D)).astype(np.float32)
    v = rng.standard_normal((B, H, L, Dv)).astype(np.float32)
    beta = (2.0 / (1.0 + np.exp(-rng.standard_normal((B, H, L))))).astype(np.float32)
    return tk, tq, v, beta


def run_core(tk, tq, v, beta, C, M0=None):
    t = lambda a: torch.from_numpy(np.asarray(a, np.float64))  # noqa: E731
    m0 = None if M0 is None else torch.from_numpy(M0.astype(np.complex128))
    with torch.no_grad():
        out, M = _chunkwise_delta_reference(t(tk), t(tq), t(v), t(beta), C, m0)
    return out.numpy(), M.numpy()


def run_steps(tk, tq, v, beta, M0=None):
    """The reference step recurrence (layers.py:279-285) over a whole sequence,
    executed with the reference's own block.step core arithmetic in fp64."""
    B, H, L, D = tk.shape
    M = (torch.zeros(B, H, v.shape[-1], D, dtype=torch.complex128) if M0 is None
         else torch.from_numpy(M0.astype(np.complex128)))
    outs = []
    for i in range(L):
        k = torch.polar(torch.ones(B, H, D, dtype=torch.float64), torch.from_numpy(tk[:, :, i].astype(np.float64)))
        q = torch.polar(torch.ones(B, H, D, dtype=torch.float64), torch.from_numpy(tq[:, :, i].astype(np.float64)))
        vt = torch.from_numpy(v[:, :, i].astype(np.float64))
        bt = torch.from_numpy(beta[:, :, i].astype(np.float64))
        v_old = torch.matmul(M, torch.conj(k).unsqueeze(-1)).squeeze(-1).real / D
        upd = torch.matmul((vt - v_old).to(M.dtype).unsqueeze(-1), k.unsqueeze(-2))
        M = M + bt.unsqueeze(-1).unsqueeze(-1) * upd
        outs.append((torch.matmul(M, torch.conj(q).unsqueeze(-1)).squeeze(-1).real / D).numpy())
    return np.stack(outs, 2), M.numpy()


def make_core():
    # Config "CPU-runnable core forward": B=2,H=4,L=256,d_k=32,C=32, seed 0
    rng = np.random.default_rng(0)
    tk, tq, v, beta = core_inputs(rng, 2, 4, 256, 32)
    out, M = run_core(tk, tq, v, beta, 32)
    out_s, M_s = run_steps(tk, tq, v, beta)
    save("core_cfg1", theta_k=tk, theta_q=tq, v=v, beta=beta, chunk_size=32,
         out=out.astype(np.float32), M=M.astype(np.complex64),
         out_rec=out_s.astype(np.float32), M_rec=M_s.astype(np.complex64))

    cases = [  # (B, H, L, D, Dv, C, nonzero M0)
        (1, 2, 64, 16, 16, 16, False),
        (2, 1, 96, 32, 32, 32, True),
        (1, 3, 24, 8, 8, 8, True),
        (1, 1, 128, 64, 64, 64, True),
        (2, 2, 40, 20, 20, 20, True),
        (1, 2, 100, 24, 24, 100, False),
    ]
    for idx, (B, H, L, D, Dv, C, init) in enumerate(cases):
        rng = np.random.default_rng(100 + idx)
        tk, tq, v, beta = core_inputs(rng, B, H, L, D, Dv)
        if idx == 0:
            beta[0, 0, :5] = 0.0
        M0 = None
        if init:
            M0 = (rng.standard_normal((B, H, Dv, D)) + 1j * rng.standard_normal((B, H, Dv, D))).astype(np.complex64)
        out, M = run_core(tk, tq, v, beta, C, M0)
        out_s, M_s = run_steps(tk, tq, v, beta, M0)
        kw = dict(theta_k=tk, theta_q=tq, v=v, beta=beta, chunk_size=C, out=out, M=M,
                  out_rec=out_s, M_rec=M_s)
        if M0 is not None:
            kw["M0"] = M0
        save(f"core_case{idx}", **kw)


def make_gram():
    torch.manual_seed(0)
    arrays = {}
    for i, (N, C, D) in enumerate([(3, 8, 16), (4, 16, 16), (4, 32, 48), (2, 64, 64), (2, 64, 96)]):
        th = torch.randn(N, C, D, dtype=torch.float64)
        b = torch.rand(N, C, dtype=torch.float64)
        b[0] = 0.0
        arrays[f"theta{i}"] = th.float().numpy()
        arrays[f"beta{i}"] = b.float().numpy()
        arrays[f"gram{i}"] = gram_matrix_reference(th.float().double(), b.float().double()).numpy()
    save("gram", **arrays)


def make_laplace():
    arrays = {}
    idx = 0
    for L in (1, 7, 8, 9, 17, 64):
        for init in (False, True):
            for C in (8, 32):
                torch.manual_seed(7 + idx)
                core = LaplacePhaseCore(d_model=32, n_heads=2, d_k=16, chunk_size=C).double()
                with torch.no_grad():
                    core.w_sigma_k.weight.mul_(3.0)
                    core.w_sigma_q.weight.mul_(3.0)
                x = torch.randn(2, L, 32, dtype=torch.float64)
                with torch.no_grad():
                    K, Q, v, beta, r = core._project(x, 1.0)
                M0 = (torch.randn(2, 2, 16, 16, dtype=torch.complex128) if init else None)
                with torch.no_grad():
                    out_c, Mc = core(x, memory_state=None if M0 is None else M0.clone())
                    out_s, Ms = core.forward_sequential(x, memory_state=None if M0 is None else M0.clone())
                p = f"c{idx}_"
                arrays.update({p + "K": K.numpy(), p + "Q": Q.numpy(), p + "v": v.numpy(),
                               p + "beta": beta.numpy(), p + "r": r.numpy(), p + "C": C,
                               p + "out": out_c.reshape(2, L, 2, 16).transpose(1, 2).numpy(),
                               p + "M": Mc.numpy(),
                               p + "out_seq": out_s.reshape(2, L, 2, 16).transpose(1, 2).numpy(),
                               p + "M_seq": Ms.numpy()})
                if idx in (5, 21):  # module glue (_project) pinned on two cases
                    arrays[p + "x"] = x.numpy()
                    for name in ("w_theta_k", "w_sigma_k", "w_theta_q", "w_sigma_q", "w_v", "w_beta"):
                        arrays[p + name] = getattr(core, name).weight.detach().numpy()
                if M0 is not None:
                    arrays[p + "M0"] = M0.numpy()
                idx += 1
    arrays["n_cases"] = idx
    save("laplace", **arrays)


def make_spectral():
    arrays = {}
    for n in (1, 2, 4, 8, 16, 64, 1024):
        arrays[f"fwht{n}"] = create_hadamard_matrix(n).numpy()
        arrays[f"haar{n}"] = create_haar_matrix(n).numpy()
        dct = create_dct2_matrix(n).numpy()
        if n <= 64:
            arrays[f"dct{n}"] = dct
        else:  # keep the fixture small: sampled rows + checksums
            rows = np.array([0, 1, n // 2 - 1, n - 1])
            arrays[f"dct{n}_rows"] = rows
            arrays[f"dct{n}_sampled"] = dct[rows]
            arrays[f"dct{n}_colsum"] = dct.astype(np.float64).sum(0)
    arrays["fwht768_shape"] = np.array(create_hadamard_matrix(768).shape)
    save("spectral", **arrays)


def ffn_case(d, nb, seed, tokens):
    torch.manual_seed(seed)
    ffn = LearnableSubstrateLerpFFN(d, num_banks=nb).double()
    with torch.no_grad():
        for name, p in ffn.named_parameters():
            if name == "substrate_logits":
                p.copy_(torch.randn(3, dtype=torch.float64))
            else:
                p.copy_(torch.randn_like(p) * 0.02 if name.startswith("combine")
                        else torch.randn_like(p))
    x = torch.randn(tokens, d, dtype=torch.float64)
    with torch.no_grad():
        y = ffn(x)
    sd = {k: v.numpy() for k, v in ffn.state_dict().items()}
    return x.numpy(), y.numpy(), sd


def make_ffn():
    arrays = {}
    for i, (d, nb, tokens) in enumerate([(64, 4, 10), (16, 2, 7), (128, 3, 5)]):
        x, y, sd = ffn_case(d, nb, 11 + i, tokens)
        arrays[f"c{i}_x"] = x
        arrays[f"c{i}_y"] = y
        arrays[f"c{i}_nb"] = nb
        for k, v in sd.items():
            arrays[f"c{i}_p_{k}"] = v
    arrays["n_cases"] = 3
    save("ffn", **arrays)


def make_block():
    arrays = {}
    for i, (L, C, beta_mode) in enumerate([(37, 16, "learned"), (32, 32, "fixed"), (5, 8, "learned")]):
        torch.manual_seed(42 + i)
        blk = DeltaPhaseHolographicBlock(d_model=64, n_heads=4, chunk_size=C, beta_mode=beta_mode).double()
        blk.eval()
        x = torch.randn(2, L, 64, dtype=torch.float64)
        with torch.no_grad():
            out, M = blk(x)
            st = None
            outs = []
            for t in range(L):
                o, st = blk.step(x[:, t:t + 1], st)
                outs.append(o)
            out_s = torch.cat(outs, 1)
        p = f"c{i}_"
        arrays.update({p + "x": x.numpy(), p + "out": out.numpy(), p + "M": M.numpy(),
                       p + "out_step": out_s.numpy(), p + "M_step": st[1].numpy(),
                       p + "conv_state": st[0].numpy(), p + "C": C,
                       p + "beta_mode": np.array(beta_mode)})
        for k, v in blk.state_dict().items():
            arrays[p + "p_" + k] = v.numpy()
    arrays["n_cases"] = 3
    save("block", **arrays)


def make_complex_beta():
    """ComplexBetaDeltaPhaseBlock (layers.py:294-418) in fp64: block forward (from a zero
    and from a random state) and the step loop.  Forward hooks record what the reference
    itself feeds its token loop (the w_k / w_q / w_v / w_phi outputs) and what the loop
    returns (the input of norm_retrieved), so the core is pinned on its own too."""
    arrays = {}
    cases = [(37, False, 1.0), (9, True, 3.0), (1, False, 1.0), (64, True, 1.0)]
    for i, (L, init, phi_scale) in enumerate(cases):
        torch.manual_seed(90 + i)
        d, H = 64, 4
        blk = ComplexBetaDeltaPhaseBlock(d_model=d, n_heads=H).double()
        blk.eval()
        with torch.no_grad():
            blk.w_phi.weight.mul_(phi_scale)
        x = torch.randn(2, L, d, dtype=torch.float64)
        M0 = torch.randn(2, H, d // H, d // H, dtype=torch.complex128) if init else None
        seen = {}

        def keep(name):
            def hook(mod, inp, out):
                seen.setdefault(name, out.detach().clone())
            return hook

        hooks = [getattr(blk, n).register_forward_hook(keep(n)) for n in ("w_k", "w_q", "w_v", "w_phi")]
        hooks.append(blk.norm_retrieved.register_forward_pre_hook(
            lambda mod, inp: seen.setdefault("retrieved", inp[0].detach().clone())))
        with torch.no_grad():
            out, M = blk(x, memory_state=None if M0 is None else M0.clone())
        for hk in hooks:
            hk.remove()
        with torch.no_grad():
            st = None if M0 is None else (None, M0.clone())
            outs = []
            for t in range(L):
                o, st = blk.step(x[:, t:t + 1], st)
                outs.append(o)
            out_s = torch.cat(outs, 1)
        heads = lambda y: y.view(2, L, H, d // H).transpose(1, 2).numpy()  # noqa: E731
        p = f"c{i}_"
        arrays.update({p + "x": x.numpy(), p + "out": out.numpy(), p + "M": M.numpy(),
                       p + "out_step": out_s.numpy(), p + "M_step": st[1].numpy(),
                       p + "conv_state": st[0].numpy(),
                       p + "theta_k": heads(seen["w_k"]), p + "theta_q": heads(seen["w_q"]),
                       p + "v": heads(seen["w_v"]), p + "phi": seen["w_phi"].transpose(1, 2).numpy(),
                       p + "retrieved": seen["retrieved"].view(2, L, H, d // H).transpose(1, 2).numpy()})
        if M0 is not None:
            arrays[p + "M0"] = M0.numpy()
        for k, v in blk.state_dict().items():
            arrays[p + "p_" + k] = v.numpy()
    arrays["n_cases"] = len(cases)
    arrays["n_heads"] = 4
    save("complex_beta", **arrays)


def make_grad():
    """Gradients, as the reference trains: autograd (float64) of _chunkwise_delta_reference
    (triton_chunk_delta.py:211-252) for the real beta, and of the two blocks for a seeded
    loss sum(out * R) + Re sum(conj(dM) M) -- with forward hooks recording the core's
    inputs, their gradients and the gradient reaching the core's output (the input of
    norm_retrieved), plus every parameter's gradient."""
    arrays = {}
    cases = [(1, 2, 64, 16, 16, True, True), (2, 1, 96, 32, 32, False, False), (1, 1, 8, 8, 8, True, True)]
    for i, (B, H, L, D, C, init, with_dM) in enumerate(cases):
        rng = np.random.default_rng(300 + i)
        tk, tq, v, beta = core_inputs(rng, B, H, L, D)
        dout = rng.standard_normal((B, H, L, D))
        M0 = (rng.standard_normal((B, H, D, D)) + 1j * rng.standard_normal((B, H, D, D))) if init else None
        dM = (rng.standard_normal((B, H, D, D)) + 1j * rng.standard_normal((B, H, D, D))) if with_dM else None
        t = [torch.from_numpy(np.asarray(a, np.float64)).requires_grad_(True) for a in (tk, tq, v, beta)]
        m0 = None if M0 is None else torch.from_numpy(M0).requires_grad_(True)
        out, M = _chunkwise_delta_reference(*t, C, m0)
        outs, gos = [out], [torch.from_numpy(dout)]
        if dM is not None:
            outs.append(M)
            gos.append(torch.from_numpy(dM))
        grads = torch.autograd.grad(outs, t + ([m0] if m0 is not None else []), gos)
        p = f"c{i}_"
        arrays.update({p + "theta_k": tk, p + "theta_q": tq, p + "v": v, p + "beta": beta, p + "dout": dout,
                       p + "C": C, p + "d_theta_k": grads[0].numpy(), p + "d_theta_q": grads[1].numpy(),
                       p + "d_v": grads[2].numpy(), p + "d_beta": grads[3].numpy()})
        if M0 is not None:
            arrays[p + "M0"] = M0
            arrays[p + "d_M0"] = grads[4].numpy()
        if dM is not None:
            arrays[p + "dM"] = dM
    arrays["n_cases"] = len(cases)

    # the two blocks: parameter gradients and the core's own view of them
    for name, make in (("hb", lambda: DeltaPhaseHolographicBlock(d_model=32, n_heads=2, chunk_size=8)),
                       ("cb", lambda: ComplexBetaDeltaPhaseBlock(d_model=32, n_heads=2))):
        torch.manual_seed(77)
        blk = make().double()
        blk.train()
        H, dk, L = 2, 16, 20
        x = torch.randn(2, L, 32, dtype=torch.float64)
        R = torch.randn(2, L, 32, dtype=torch.float64)
        M0 = torch.randn(2, H, dk, dk, dtype=torch.complex128).requires_grad_(True)
        dM = torch.randn(2, H, dk, dk, dtype=torch.complex128)
        seen = {}

        def keep(nm):
            def hook(mod, inp, out):
                out.retain_grad()
                seen.setdefault(nm, out)
            return hook

        def keep_in(mod, inp):
            inp[0].retain_grad()
            seen.setdefault("retrieved", inp[0])

        gate = "w_beta" if name == "hb" else "w_phi"
        hooks = [getattr(blk, n).register_forward_hook(keep(n)) for n in ("w_k", "w_q", "w_v", gate)]
        hooks.append(blk.norm_retrieved.register_forward_pre_hook(keep_in))
        out, M = blk(x, memory_state=M0)
        loss = (out * R).sum() + (torch.conj(dM) * M).real.sum()
        loss.backward()
        for hk in hooks:
            hk.remove()
        Lp = seen["w_k"].shape[1]  # the holographic block pads L to a chunk multiple (layers.py:185-190)
        heads = lambda y: y.view(2, Lp, H, dk).transpose(1, 2).detach().numpy()  # noqa: E731
        dret = seen["retrieved"].grad.view(2, L, H, dk).transpose(1, 2).numpy()
        dout = np.zeros((2, H, Lp, dk))
        dout[:, :, :L] = dret
        p = name + "_"
        arrays.update({p + "x": x.numpy(), p + "R": R.numpy(), p + "M0": M0.detach().numpy(), p + "dM": dM.numpy(),
                       p + "out": out.detach().numpy(), p + "M": M.detach().numpy(),
                       p + "d_M0": M0.grad.numpy(),
                       p + "theta_k": heads(seen["w_k"]), p + "theta_q": heads(seen["w_q"]),
                       p + "v": heads(seen["w_v"]),
                       p + "d_theta_k": heads(seen["w_k"].grad), p + "d_theta_q": heads(seen["w_q"].grad),
                       p + "d_v": heads(seen["w_v"].grad),
                       p + "gate_raw": seen[gate].transpose(1, 2).detach().numpy(),
                       p + "d_gate_raw": seen[gate].grad.transpose(1, 2).numpy(),
                       p + "dout": dout, p + "L": L})
        for k, v in blk.state_dict().items():
            arrays[p + "p_" + k] = v.numpy()
        for k, prm in blk.named_parameters():
            arrays[p + "g_" + k] = prm.grad.numpy()
    save("grad", **arrays)


def make_laplace_grad():
    """LaplacePhaseCore gradients as the reference trains it: autograd (float64) of its
    chunk loop (layers.py:481-561).  Core level: `_project` patched to build K, Q, v, beta
    and r from leaf tensors (theta_k, log|k|, theta_q, log|q|, v, log r, beta), so the
    gradients of exactly those inputs are recorded.  Module level: every parameter's
    gradient for a seeded loss sum(out * R) + Re sum(conj(dM) M)."""
    arrays = {}
    cases = [(2, 2, 40, 8, 8, True), (1, 2, 33, 16, 32, False), (2, 1, 64, 16, 16, True)]
    for i, (B, H, L, D, C, init) in enumerate(cases):
        rng = np.random.default_rng(500 + i)
        core = LaplacePhaseCore(d_model=H * D, n_heads=H, d_k=D, chunk_size=C).double()
        leaves = {
            "theta_k": rng.uniform(0, 2 * np.pi, (B, H, L, D)), "logmag_k": -0.5 * rng.random((B, H, L, D)),
            "theta_q": rng.uniform(0, 2 * np.pi, (B, H, L, D)), "logmag_q": -0.5 * rng.random((B, H, L, D)),
            "v": rng.standard_normal((B, H, L, D)), "log_decay": -np.log1p(np.exp(rng.standard_normal((B, H, L, D)))),
            "beta": 2.0 / (1.0 + np.exp(-rng.standard_normal((B, H, L))))}
        T = {k: torch.from_numpy(a).requires_grad_(True) for k, a in leaves.items()}

        def project(x, ts, T=T):
            K = torch.complex(torch.exp(T["logmag_k"]) * torch.cos(T["theta_k"]),
                              torch.exp(T["logmag_k"]) * torch.sin(T["theta_k"]))
            Q = torch.complex(torch.exp(T["logmag_q"]) * torch.cos(T["theta_q"]),
                              torch.exp(T["logmag_q"]) * torch.sin(T["theta_q"]))
            return K, Q, T["v"], T["beta"], torch.exp(T["log_decay"])

        core._project = project
        M0 = torch.from_numpy(rng.standard_normal((B, H, D, D)) + 1j * rng.standard_normal((B, H, D, D))) if init else None
        if M0 is not None:
            M0.requires_grad_(True)
        dout = rng.standard_normal((B, L, H * D))
        dM = rng.standard_normal((B, H, D, D)) + 1j * rng.standard_normal((B, H, D, D))
        x = torch.zeros(B, L, H * D, dtype=torch.float64)
        out, M = core(x, memory_state=M0)
        loss = (out * torch.from_numpy(dout)).sum() + (torch.conj(torch.from_numpy(dM)) * M).real.sum()
        loss.backward()
        p = f"c{i}_"
        for k, a in leaves.items():
            arrays[p + k] = a
            arrays[p + "d_" + k] = T[k].grad.numpy()
        arrays.update({p + "C": C, p + "dM": dM, p + "out": out.detach().view(B, L, H, D).transpose(1, 2).numpy(),
                       p + "M": M.detach().numpy(),
                       p + "dout": dout.reshape(B, L, H, D).transpose(0, 2, 1, 3)})
        if M0 is not None:
            arrays[p + "M0"] = M0.detach().numpy()
            arrays[p + "d_M0"] = M0.grad.numpy()
    arrays["n_cases"] = len(cases)
    # module level
    torch.manual_seed(61)
    core = LaplacePhaseCore(d_model=32, n_heads=2, d_k=16, chunk_size=8).double()
    with torch.no_grad():
        core.w_sigma_k.weight.mul_(3.0)
    x = torch.randn(2, 29, 32, dtype=torch.float64)
    R = torch.randn(2, 29, 32, dtype=torch.float64)
    M0 = torch.randn(2, 2, 16, 16, dtype=torch.complex128).requires_grad_(True)
    dM = torch.randn(2, 2, 16, 16, dtype=torch.complex128)
    out, M = core(x, memory_state=M0)
    ((out * R).sum() + (torch.conj(dM) * M).real.sum()).backward()
    arrays.update({"mod_x": x.numpy(), "mod_R": R.numpy(), "mod_M0": M0.detach().numpy(), "mod_dM": dM.numpy(),
                   "mod_out": out.detach().numpy(), "mod_M": M.detach().numpy(), "mod_d_M0": M0.grad.numpy()})
    for k, v in core.state_dict().items():
        arrays["mod_p_" + k] = v.numpy()
    for k, prm in core.named_parameters():
        arrays["mod_g_" + k] = prm.grad.numpy()
    save("laplace_grad", **arrays)


MAKERS = {"core": make_core, "gram": make_gram, "laplace": make_laplace, "spectral": make_spectral,
          "ffn": make_ffn, "block": make_block, "complex_beta": make_complex_beta, "grad": make_grad,
          "laplace_grad": make_laplace_grad}

if __name__ == "__main__":
    for name in (sys.argv[1:] or list(MAKERS)):
        MAKERS[name]()
