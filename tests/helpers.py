"""Shared helpers of the test suite: seeded inputs, golden loading, GPU transfer."""
import os

import numpy as np
import torch

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load_golden(name):
    return np.load(os.path.join(GOLDEN, name + ".npz"))


def core_inputs(seed, B, H, L, D, Dv=None):
    """theta ~ U[0, 2pi), v ~ N(0, 1), beta = 2 sigmoid(N(0, 1)) (float32)."""
    Dv = D if Dv is None else Dv
    rng = np.random.default_rng(seed)
    tk = rng.uniform(0.0, 2 * np.pi, (B, H, L, D)).astype(np.float32)
    tq = rng.uniform(0.0, 2 * np.pi, (B, H, L, D)).astype(np.float32)
    v = rng.standard_normal((B, H, L, Dv)).astype(np.float32)
    beta = (2.0 / (1.0 + np.exp(-rng.standard_normal((B, H, L))))).astype(np.float32)
    return tk, tq, v, beta


def to_dev(a, dtype=None, device="cuda"):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(device)
    return t if dtype is None else t.to(dtype)


def round_bf16(a):
    """numpy copy of a, rounded through bfloat16 (the values a bf16 kernel sees)."""
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16).float().numpy()


def rel_l2(a, b):
    a = a.detach().cpu().numpy() if isinstance(a, torch.Tensor) else np.asarray(a)
    b = b.detach().cpu().numpy() if isinstance(b, torch.Tensor) else np.asarray(b)
    if np.iscomplexobj(a) or np.iscomplexobj(b):
        a = np.stack([np.real(a), np.imag(a)], -1)
        b = np.stack([np.real(b), np.imag(b)], -1)
    a = a.astype(np.float64)
    b = b.astype(np.float64)
    den = np.linalg.norm(b.ravel())
    return float(np.linalg.norm((a - b).ravel()) / (den if den > 0 else 1.0))


def report(name, **errs):
    """Prints the measured errors of a parity case (``pytest -s`` shows them), so the
    margin against the tolerance is on record, not only pass / fail."""
    print("PARITY %s %s" % (name, " ".join("%s=%.3e" % kv for kv in errs.items())), flush=True)


# Tolerances of the specification: relative L2 against the reference's fp64 path.
TOL_F32 = 2e-3   # float32 inputs, fp32 accumulation
TOL_BF16 = 1e-2  # bfloat16 inputs, fp32 accumulation
