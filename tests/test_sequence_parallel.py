"""Sequence-parallel LaplacePhaseCore (delta_phase_b200.sequence_parallel): boundary-state
hand-off between ranks.  CPU: gloo ranks with a float64 segment solver, checked against
the token-loop oracle on the whole sequence.  GPU (two or more devices): NCCL ranks on
the CUDA kernel, checked against one GPU solving the whole sequence."""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import laplace as olap


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(B, H, L, D, seed=0):
    rng = np.random.default_rng(seed)
    tk = rng.uniform(0, 2 * np.pi, (B, H, L, D))
    tq = rng.uniform(0, 2 * np.pi, (B, H, L, D))
    mk = -np.logaddexp(0, rng.standard_normal((B, H, L, D))) * 0.3
    mq = -np.logaddexp(0, rng.standard_normal((B, H, L, D))) * 0.3
    v = rng.standard_normal((B, H, L, D))
    lr = -np.logaddexp(0, rng.standard_normal((B, H, L, D)))
    beta = 2 / (1 + np.exp(-rng.standard_normal((B, H, L))))
    M0 = (rng.standard_normal((B, H, D, D)) + 1j * rng.standard_normal((B, H, D, D))) * 0.3
    return tk, mk, tq, mq, v, lr, beta, M0


def _segment_oracle(tk, mk, tq, mq, v, lr, beta, chunk_size, initial_state, out=None):
    """float64 CPU stand-in for the CUDA segment solver (same signature)."""
    K = torch.exp(mk + 1j * tk).numpy()
    Q = torch.exp(mq + 1j * tq).numpy()
    M0 = None if initial_state is None else initial_state.numpy()
    o, M = olap.laplace_sequential(K, Q, v.numpy(), beta.numpy(), np.exp(lr.numpy()), M0)
    out.copy_(torch.from_numpy(o))
    return out, torch.from_numpy(M)


def _cpu_rank(rank, world, port, B, H, L, D, cuts, micro, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from delta_phase_b200.sequence_parallel import laplace_chunkwise_sp
        tk, mk, tq, mq, v, lr, beta, M0 = _inputs(B, H, L, D)
        a, b = cuts[rank], cuts[rank + 1]
        seg = [torch.from_numpy(np.ascontiguousarray(x[:, :, a:b])) for x in (tk, mk, tq, mq, v, lr, beta)]
        out = torch.empty(B, H, b - a, D, dtype=torch.float64)
        out, M = laplace_chunkwise_sp(*seg, 64, torch.from_numpy(M0), micro_groups=micro,
                                      segment_fn=_segment_oracle, out=out)
        np.savez(os.path.join(outdir, f"r{rank}.npz"), out=out.numpy(), M=M.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,cuts,micro,B", [
    (2, [0, 70, 128], 1, 2),
    (3, [0, 40, 41, 128], 2, 3),
])
def test_state_handoff_matches_whole_sequence(world, cuts, micro, B):
    H, L, D = 2, 128, 8
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_cpu_rank, args=(world, _free_port(), B, H, L, D, cuts, micro, d), nprocs=world,
                           start_method="spawn", join=True)
        parts = [np.load(os.path.join(d, f"r{r}.npz")) for r in range(world)]
        out = np.concatenate([p["out"] for p in parts], axis=2)
        M_last = parts[-1]["M"]
    tk, mk, tq, mq, v, lr, beta, M0 = _inputs(B, H, L, D)
    ref_out, ref_M = olap.laplace_sequential(np.exp(mk + 1j * tk), np.exp(mq + 1j * tq), v, beta, np.exp(lr), M0)
    np.testing.assert_allclose(out, ref_out, rtol=1e-10, atol=1e-10)
    np.testing.assert_allclose(M_last, ref_M, rtol=1e-10, atol=1e-10)


def _gpu_rank(rank, world, port, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        from delta_phase_b200.sequence_parallel import laplace_chunkwise_sp
        B, H, L, D = 4, 3, 64 * 6, 64
        tk, mk, tq, mq, v, lr, beta, M0 = _inputs(B, H, L, D, seed=1)
        seg_len = L // world
        a, b = rank * seg_len, (rank + 1) * seg_len
        dev = torch.device("cuda", rank)
        bf = lambda x: torch.from_numpy(np.ascontiguousarray(x[:, :, a:b])).to(dev, torch.bfloat16)  # noqa: E731
        out, M = laplace_chunkwise_sp(bf(tk), bf(mk), bf(tq), bf(mq), bf(v), bf(lr), bf(beta), 64,
                                      torch.from_numpy(M0).to(dev, torch.complex64), micro_groups=2)
        torch.cuda.synchronize()
        np.savez(os.path.join(outdir, f"g{rank}.npz"), out=out.cpu().numpy(), M=M.cpu().numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_nccl_sequence_parallel_matches_one_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import delta_phase_b200 as dp
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_gpu_rank, args=(world, _free_port(), d), nprocs=world, start_method="spawn", join=True)
        parts = [np.load(os.path.join(d, f"g{r}.npz")) for r in range(world)]
    out_sp = np.concatenate([p["out"] for p in parts], axis=2)
    B, H, L, D = 4, 3, 64 * 6, 64
    tk, mk, tq, mq, v, lr, beta, M0 = _inputs(B, H, L, D, seed=1)
    bf = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to("cuda:0", torch.bfloat16)  # noqa: E731
    out1, M1 = dp.laplace_chunkwise(bf(tk), bf(mk), bf(tq), bf(mq), bf(v), bf(lr), bf(beta), 64,
                                    torch.from_numpy(M0).to("cuda:0", torch.complex64))
    # segments start on chunk boundaries, so the split solve is the same arithmetic
    np.testing.assert_allclose(out_sp, out1.cpu().numpy(), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(parts[-1]["M"], M1.cpu().numpy(), rtol=1e-5, atol=1e-5)
