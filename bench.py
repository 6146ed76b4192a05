"""Benchmark of the DeltaPhase hot path on B200.

Default workload (the headline metric): the chunkwise complex delta-rule forward at
B=8, H=16, L=8192, d_k=d_v=64, C=64, bf16 inputs, fp32 accumulation and output, on
each GPU (batch x head sharding, weak scaling: global batch = 8 x n_gpus; no
collective on the data path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload core|cbeta|train|decode|laplace|laplace-sp|ffn|lm]

Multi-GPU: launch with torch.distributed.run (one process per GPU); rank 0 prints one
JSON line.  ``--impl reference`` times the reference's own chunkwise path on the host
cores: its public ``delta_phase_chunkwise_fused`` (torch, float32, no_grad) from the
unmodified install in ``baseline/_ref``, or, when that install is absent, the numpy port
of the same path.  On one GPU the headline line also carries a ``secondary`` object with
the other workloads (Laplace, FFN, decode step, complex-beta core, LM prefill and decode),
a few steps each.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "delta-core tokens/s (H=16,d_k=64,L=8K) & % roofline at 1/2/4/8 B200"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

CORE = dict(B=8, H=16, L=8192, D=64, C=64)


def core_algorithmic_bytes(B, H, L, D, Dv, in_bytes=2, beta_bytes=2, out_bytes=4):
    """Compulsory HBM bytes of one chunkwise forward: theta_k, theta_q, v, beta read once,
    out written once, final complex64 state written once (zero initial state)."""
    per_head_token = 2 * D * in_bytes + Dv * in_bytes + beta_bytes + Dv * out_bytes
    return B * H * L * per_head_token + B * H * Dv * D * 8


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    except (OSError, ValueError):
        return dict(PEAKS_FALLBACK), "fallback"


def read_profile_traffic(name):
    """Per-launch DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) recorded
    from an ncu capture in profiles/<name> (line 'traffic_bytes_per_launch: N')."""
    path = os.path.join(ROOT, "profiles", name)
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return int(float(line.split(":", 1)[1].strip()))
    except OSError:
        pass
    return None


class ClockSampler:
    """Samples the SM clock and clock-event (throttle) reasons through NVML every few
    milliseconds while the timed region runs."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, device_index, period_s=0.002):
        self.idx = device_index
        self.period = period_s
        self.samples = []
        self.reasons = set()
        self._stop = threading.Event()
        self._first = threading.Event()
        self._t = None
        self.max_mhz = None

    def start(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            phys = int(vis.split(",")[self.idx]) if vis else self.idx
            self._h = pynvml.nvmlDeviceGetHandleByIndex(phys)
            self._nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._h = None
            return
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        self._first.wait(timeout=1.0)  # sampling is running before the timed region starts

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for name, bit in self.REASONS.items():
                    if mask & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            self._first.set()
            time.sleep(self.period)

    def stop(self):
        if self._t is None:
            return None
        self._stop.set()
        self._t.join(timeout=2)
        if not self.samples:
            return None
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples), "source": "NVML"}


# ------------------------------------------------------------------ distributed plumbing
def nccl_debug_env(world, env):
    """NCCL's communicator set-up lines (nranks, ranks, devices) for a multi-rank run, so a
    reader can check the communicator spans every GPU of the run.

    A caller that sets NCCL_DEBUG itself keeps its own setting and destination.  Otherwise
    NCCL logs its INIT lines to a file of this process (NCCL opens the file for writing,
    which would truncate a log that stderr is redirected to, and its default destination,
    stdout, carries the result line); echo_nccl_log copies them to stderr once the
    communicator exists.  NCCL reads these variables when it initialises, so they are set
    before torch is imported.  Returns the file's path, or None when nothing was set."""
    if world <= 1 or "NCCL_DEBUG" in env:
        return None
    path = os.path.join(tempfile.gettempdir(), f"bench_nccl_{os.getpid()}.log")
    env["NCCL_DEBUG"] = "INFO"
    env.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
    env["NCCL_DEBUG_FILE"] = path
    return path


def echo_nccl_log(path, out):
    """Copy NCCL's log file (nccl_debug_env) to `out` and remove it; NCCL keeps writing its
    later lines (tear-down) to the unlinked file."""
    if path is None:
        return
    try:
        with open(path, "r", errors="replace") as f:
            text = f.read()
        os.unlink(path)
    except OSError:  # no log written: the report line below still names the process group
        return
    if text:
        out.write(text if text.endswith("\n") else text + "\n")
        out.flush()


def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    nccl_log = nccl_debug_env(world, os.environ)
    import torch
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        dist.barrier()  # the communicator exists on every rank: its set-up lines are written
        echo_nccl_log(nccl_log, sys.stderr)
        # the process group as torch sees it (stderr; NCCL's own INIT lines come with it)
        try:
            v = torch.cuda.nccl.version()
            nccl_v = ".".join(str(x) for x in v) if isinstance(v, (tuple, list)) else str(v)
        except Exception:  # the report must not stop the benchmark
            nccl_v = "unknown"
        print(f"bench.py: process group backend={dist.get_backend()} rank={dist.get_rank()} "
              f"world_size={dist.get_world_size()} device=cuda:{local} nccl={nccl_v}", file=sys.stderr, flush=True)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def gather_over_ranks(x, world):
    """Every rank's value of x (a float), in rank order."""
    if world == 1:
        return [x]
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [float(o.item()) for o in out]


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------ CPU baseline (port)
def cpu_core_sample(units=2, L=8192, D=64, C=64, seed=0):
    """Time the numpy float32 port of the reference chunkwise path (oracle.core) on
    `units` (b, h) units of length L.  Returns (seconds, head_tokens)."""
    from oracle import core as ocore
    rng = np.random.default_rng(seed)
    tk = rng.uniform(0, 2 * np.pi, (1, units, L, D)).astype(np.float32)
    tq = rng.uniform(0, 2 * np.pi, (1, units, L, D)).astype(np.float32)
    v = rng.standard_normal((1, units, L, D)).astype(np.float32)
    beta = (2 / (1 + np.exp(-rng.standard_normal((1, units, L))))).astype(np.float32)
    t0 = time.perf_counter()
    ocore.chunkwise_delta(tk, tq, v, beta, C, None, dtype=np.float32)
    return time.perf_counter() - t0, units * L


REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def reference_chunkwise():
    """The reference's own public entry point, ``delta_phase.kernels.delta_phase_chunkwise_fused``
    (delta_phase/kernels/triton_chunk_delta.py:278-291), imported from the unmodified install
    in baseline/_ref; None when that install is absent."""
    if not os.path.isdir(os.path.join(REF_DIR, "delta_phase")):
        return None
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    try:
        from delta_phase.kernels import delta_phase_chunkwise_fused
    except Exception:
        return None
    return delta_phase_chunkwise_fused


def ref_core_sample(fn, units=16, L=8192, D=64, C=64, seed=0):
    """Time the reference's chunkwise forward (its own PyTorch path on CPU, float32, under
    no_grad: the inference dispatch of delta_phase_chunkwise_fused) on `units` (b, h) units
    of length L.  Returns (seconds, head_tokens)."""
    import torch
    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(seed)
    tk = torch.rand(1, units, L, D, generator=g) * (2 * np.pi)
    tq = torch.rand(1, units, L, D, generator=g) * (2 * np.pi)
    v = torch.randn(1, units, L, D, generator=g)
    beta = 2 * torch.sigmoid(torch.randn(1, units, L, generator=g))
    with torch.no_grad():
        t0 = time.perf_counter()
        fn(tk, tq, v, beta, C, None)
        return time.perf_counter() - t0, units * L


def cpu_core_baseline(units, L=8192):
    """One bounded CPU sample of the core workload: the reference's own code when it is
    installed (kind "reference"), else the numpy port (kind "port").
    Returns (seconds, head_tokens, kind, description)."""
    fn = reference_chunkwise()
    if fn is not None:
        s, ht = ref_core_sample(fn, units=units, L=L)
        return s, ht, "reference", ("reference delta_phase_chunkwise_fused (torch fp32 CPU, no_grad; "
                                    "unmodified install in baseline/_ref)")
    s, ht = cpu_core_sample(units=units, L=L)
    return s, ht, "port", "numpy float32 port of the reference chunkwise path (oracle.core)"


def repeat_for(fn, min_seconds=10.0):
    """Run fn() until at least min_seconds have passed; returns (seconds, repetitions)."""
    t0, reps = time.perf_counter(), 0
    while True:
        fn(reps)
        reps += 1
        secs = time.perf_counter() - t0
        if secs >= min_seconds:
            return secs, reps


def cpu_threads():
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads") for i in threadpool_info() if i.get("user_api") == "blas"]
        if n and n[0]:
            return int(n[0])
    except Exception:
        pass
    return os.cpu_count() or 1


# ------------------------------------------------------------------ workloads
def make_core_inputs(dev, seed, B, H, L, D):
    import torch
    g = torch.Generator(device=dev).manual_seed(seed)
    tk = (torch.rand(B, H, L, D, device=dev, generator=g) * (2 * np.pi)).to(torch.bfloat16)
    tq = (torch.rand(B, H, L, D, device=dev, generator=g) * (2 * np.pi)).to(torch.bfloat16)
    v = torch.randn(B, H, L, D, device=dev, generator=g).to(torch.bfloat16)
    beta = (2 * torch.sigmoid(torch.randn(B, H, L, device=dev, generator=g))).to(torch.bfloat16)
    return tk, tq, v, beta


def run_core(args, world, rank, local):
    import torch
    from delta_phase_b200 import _capi
    from delta_phase_b200.kernels import chunkwise_forward

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    B, H, L, D, C = (CORE[k] for k in ("B", "H", "L", "D", "C"))
    tk, tq, v, beta = make_core_inputs(dev, 1000 + rank, B, H, L, D)
    out = torch.empty(B, H, L, D, device=dev, dtype=torch.float32)
    stream = torch.cuda.current_stream(dev)

    def step():
        chunkwise_forward(tk, tq, v, beta, C, None, out=out)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    clocks = ClockSampler(local)
    clocks.start()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    barrier(world)
    ms = ev0.elapsed_time(ev1) / args.steps
    ms_max = max_over_ranks(ms, world)
    tokens = world * B * L
    value = tokens / (ms_max / 1e3)

    # e2e: through the public API from pinned host buffers, result read back to host, every
    # step.  Steps are pipelined the way a streaming caller would run them: the inputs of
    # step i + 1 go up (copy stream) while step i computes and its outputs come down
    # (second copy stream); device buffers are double-buffered and ordered by events.
    host = [t.cpu().pin_memory() for t in (tk, tq, v, beta)]
    out_h = [torch.empty(B, H, L, D, dtype=torch.float32).pin_memory() for _ in range(2)]
    M_h = [torch.empty(B, H, D, D, dtype=torch.complex64).pin_memory() for _ in range(2)]
    dev_in = [[torch.empty_like(t) for t in (tk, tq, v, beta)] for _ in range(2)]
    dev_out = [torch.empty(B, H, L, D, device=dev, dtype=torch.float32) for _ in range(2)]
    s_up, s_down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]
    ev_read = [torch.cuda.Event() for _ in range(2)]
    for e in ev_done + ev_read:
        e.record(stream)

    def e2e_step(i):
        k = i & 1
        with torch.cuda.stream(s_up):
            s_up.wait_event(ev_done[k])  # step i - 2 is done reading this input slot
            for d_, h_ in zip(dev_in[k], host):
                d_.copy_(h_, non_blocking=True)
            ev_in[k].record(s_up)
        stream.wait_event(ev_in[k])
        stream.wait_event(ev_read[k])  # step i - 2's outputs have left this slot
        _, M = chunkwise_forward(*dev_in[k], C, None, out=dev_out[k])
        ev_done[k].record(stream)
        with torch.cuda.stream(s_down):
            s_down.wait_event(ev_done[k])
            out_h[k].copy_(dev_out[k], non_blocking=True)
            M_h[k].copy_(M, non_blocking=True)
            M.record_stream(s_down)
            ev_read[k].record(s_down)

    e2e_steps = max(4, min(args.steps, 10))
    for i in range(2):
        e2e_step(i)
    torch.cuda.synchronize()
    barrier(world)
    ev0.record(stream)
    for i in range(e2e_steps):
        e2e_step(i)
    stream.wait_stream(s_up)
    stream.wait_stream(s_down)
    ev1.record(stream)
    torch.cuda.synchronize()
    e2e_rank_ms = ev0.elapsed_time(ev1) / e2e_steps
    e2e_per_rank = gather_over_ranks(e2e_rank_ms, world)
    e2e_ms = max(e2e_per_rank)
    h2d = sum(t.numel() * t.element_size() for t in host)
    d2h = out_h[0].numel() * 4 + M_h[0].numel() * 8

    peaks, src = load_peaks()
    alg_bytes = core_algorithmic_bytes(B, H, L, D, D)
    achieved = alg_bytes / (ms / 1e3) / 1e9
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded: theta~U[0,2pi), v~N(0,1), beta=2*sigmoid(N(0,1)))",
        "config": {"workload": "chunkwise complex delta-rule forward, config B=8,H=16,L=8192,"
                               "d_k=d_v=64,C=64 per GPU, bf16 in / fp32 accum+out",
                   "global_batch": B * world, "seq_len": L, "heads": H, "d_k": D, "chunk": C,
                   "parallelism": f"batch x head sharding over {world} GPU(s), no collective",
                   "l2": f"inputs+outputs {alg_bytes / 1e6:.0f} MB per step > 126 MB L2; no flush"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"],
                     "traffic": read_profile_traffic("core_pipe_kernel_b8h16l8192_ncu_full.md"),
                     "algorithmic_bytes_per_launch": alg_bytes,
                     "peak_source": f"{src} (MEASURED_PEAKS.json hbm_gbs)" if src == "measured" else src,
                     "kernel": "dp_core_fwd (one launch per step)"},
        "e2e": {"value": tokens / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
                "path": "kernels.chunkwise_forward from pinned host buffers, out + M read back every step; "
                        "steps pipelined over two copy streams (inputs of step i+1 up while step i "
                        "computes and its outputs come down)",
                "per_rank_ms_per_step": e2e_per_rank,
                "per_rank_host_link_gbs": [(h2d + d2h) / (m / 1e3) / 1e9 for m in e2e_per_rank]},
        "gpu_launches": args.steps,
        "clocks": clk,
        "library": _capi.version(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        parts = []
        _, reps = repeat_for(lambda i: parts.append(cpu_core_baseline(args.cpu_units)), min_seconds=10.0)
        secs, ht = sum(p[0] for p in parts), sum(p[1] for p in parts)  # timed regions only
        line["cpu_baseline"] = {
            "value": ht / H / secs, "unit": "tokens/s", "cores": os.cpu_count() if parts[0][2] == "reference"
            else cpu_threads(), "kind": parts[0][2],
            "sample": f"{reps} x {args.cpu_units} (b,h) units x L=8192 of the H=16 workload, {parts[0][3]}, "
                      f"{secs:.1f} s; tokens/s = head-tokens / 16 / s"}
    return line


def _timed(step, steps, warmup, stream):
    """Device time per step (ms) of `step` over `steps` iterations after `warmup`."""
    import torch
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def _timed_clk(step, steps, warmup, stream, local):
    """_timed with the SM clocks and throttle reasons sampled during the timed steps."""
    import torch
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    ms = _timed(step, steps, 0, stream)
    return ms, sampler.stop()


def _line(metric, value, unit, args, world, ms, config, **extra):
    d = {"metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
         "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
         "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded)", "config": config}
    d.update(extra)
    return d


def cpu_cbeta_sample(units=2, L=512, D=64, seed=0):
    """Time the numpy float32 port of the reference's complex-beta token loop
    (oracle.core.complex_beta_recurrent) on `units` (b, h) units of L tokens."""
    from oracle import core as ocore
    rng = np.random.default_rng(seed)
    tk = rng.uniform(0, 2 * np.pi, (1, units, L, D)).astype(np.float32)
    tq = rng.uniform(0, 2 * np.pi, (1, units, L, D)).astype(np.float32)
    v = rng.standard_normal((1, units, L, D)).astype(np.float32)
    phi = rng.standard_normal((1, units, L)).astype(np.float32)
    t0 = time.perf_counter()
    ocore.complex_beta_recurrent(tk, tq, v, phi, None, dtype=np.float32)
    return time.perf_counter() - t0, units * L


def run_cbeta(args, world, rank, local):
    """Complex-beta (Householder) rule of ComplexBetaDeltaPhaseBlock at the core's
    shape: B=8, H=16, L=8192, d_k=64, bf16 inputs, phi ~ N(0, 1) (beta = 1 + e^{i phi})."""
    import torch
    from delta_phase_b200.kernels import chunkwise_forward
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    B, H, L, D = (CORE[k] for k in ("B", "H", "L", "D"))
    tk, tq, v, _ = make_core_inputs(dev, 3000 + rank, B, H, L, D)
    g = torch.Generator(device=dev).manual_seed(4000 + rank)
    phi = torch.randn(B, H, L, device=dev, generator=g).to(torch.bfloat16)
    out = torch.empty(B, H, L, D, device=dev, dtype=torch.float32)
    stream = torch.cuda.current_stream(dev)

    def step():
        chunkwise_forward(tk, tq, v, phi, 64, None, out=out, complex_beta=True)

    barrier(world)
    clocks = ClockSampler(local)
    clocks.start()
    ms = _timed(step, args.steps, args.warmup, stream)
    clk = clocks.stop()
    ms_max = max_over_ranks(ms, world)
    peaks, src = load_peaks()
    alg_bytes = core_algorithmic_bytes(B, H, L, D, D)
    achieved = alg_bytes / (ms / 1e3) / 1e9
    line = _line("complex-beta delta-core tokens/s (H=16,d_k=64,L=8K)", world * B * L / (ms_max / 1e3),
                 "tokens/s", args, world, ms_max,
                 {"workload": "ComplexBetaDeltaPhaseBlock core (beta = 1 + e^{i phi}), chunkwise on fp16 "
                              "operand tiles, B=8,H=16,L=8192,d_k=64 per GPU, bf16 in / fp32 out",
                  "global_batch": B * world, "seq_len": L, "heads": H, "d_k": D,
                  "parallelism": f"batch x head sharding over {world} GPU(s), no collective",
                  "l2": f"inputs+outputs {alg_bytes / 1e6:.0f} MB per step > 126 MB L2; no flush"},
                 roofline={"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                           "frac": achieved / peaks["hbm_gbs"], "traffic": None,
                           "algorithmic_bytes_per_launch": alg_bytes, "peak_source": src,
                           "kernel": "dp_core_cbeta_fwd (one launch per step)"},
                 gpu_launches=args.steps, clocks=clk)
    line["data"] = "synthetic (seeded: theta~U[0,2pi), v~N(0,1), phi~N(0,1))"
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        parts = []
        _, reps = repeat_for(lambda i: parts.append(cpu_cbeta_sample(seed=i)))
        secs, ht = sum(p[0] for p in parts), sum(p[1] for p in parts)
        line["cpu_baseline"] = {
            "value": ht / H / secs, "unit": "tokens/s", "cores": cpu_threads(), "kind": "port",
            "sample": f"{reps} x 2 (b,h) units x 512 tokens, numpy float32 port of the reference's "
                      f"complex-beta token loop (oracle.core.complex_beta_recurrent), {secs:.1f} s; "
                      "tokens/s = head-tokens / 16 / s"}
    return line


def run_train(args, world, rank, local):
    """Training step of the chunkwise core at B=8, H=16, L=8192, d_k=64 (bf16
    phases/values): forward (tensor-core kernel) and backward (dp_core_bwd) through
    DeltaPhaseCudaFunction, gradients of theta_k, theta_q, v and beta."""
    import torch
    from delta_phase_b200.kernels import DeltaPhaseCudaFunction
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    B, H, L, D = (CORE[k] for k in ("B", "H", "L", "D"))
    tk, tq, v, beta = make_core_inputs(dev, 5000 + rank, B, H, L, D)
    ins = [t.requires_grad_(True) for t in (tk, tq, v, beta)]
    g = torch.Generator(device=dev).manual_seed(6000 + rank)
    dout = torch.randn(B, H, L, D, device=dev, generator=g)
    stream = torch.cuda.current_stream(dev)

    def step():
        out, _ = DeltaPhaseCudaFunction.apply(*ins, 64, None, False)
        torch.autograd.grad(out, ins, dout)

    barrier(world)
    clocks = ClockSampler(local)
    clocks.start()
    ms = _timed(step, args.steps, args.warmup, stream)
    clk = clocks.stop()
    ms_max = max_over_ranks(ms, world)
    line = _line("delta-core training step tokens/s (fwd+bwd, H=16,d_k=64,L=8K)", world * B * L / (ms_max / 1e3),
                 "tokens/s", args, world, ms_max,
                 {"workload": "chunkwise core forward + backward (dp_core_fwd + dp_core_bwd), B=8,H=16,L=8192,"
                              "d_k=64 per GPU, bf16 in, fp32 gradients",
                  "global_batch": B * world, "seq_len": L, "heads": H, "d_k": D,
                  "parallelism": f"batch x head sharding over {world} GPU(s), no collective"},
                 gpu_launches=2 * args.steps, clocks=clk)
    line["roofline"] = None
    return line


def run_laplace(args, world, rank, local):
    """LaplacePhaseCore chunk solve at B=4, H=16, L=32768, d_k=64 (gated decay:
    log r = -softplus(N(0,1)), unit phasors, bf16 inputs)."""
    import torch
    import torch.nn.functional as F
    from delta_phase_b200.kernels import laplace_chunkwise
    dev = torch.device("cuda", local)
    B, H, L, D = 4, 16, args.seq_len, 64
    g = torch.Generator(device=dev).manual_seed(2000 + rank)
    bf = torch.bfloat16
    tk = (torch.rand(B, H, L, D, device=dev, generator=g) * 2 * np.pi).to(bf)
    tq = (torch.rand(B, H, L, D, device=dev, generator=g) * 2 * np.pi).to(bf)
    v = torch.randn(B, H, L, D, device=dev, generator=g).to(bf)
    logr = (-F.softplus(torch.randn(B, H, L, D, device=dev, generator=g))).to(bf)
    beta = (2 * torch.sigmoid(torch.randn(B, H, L, device=dev, generator=g))).to(bf)
    out = torch.empty(B, H, L, D, device=dev)
    stream = torch.cuda.current_stream(dev)
    ms, clk = _timed_clk(lambda: laplace_chunkwise(tk, None, tq, None, v, logr, beta, 64, None, out),
                         args.steps, args.warmup, stream, local)
    ms = max_over_ranks(ms, world)
    alg = B * H * L * (4 * D * 2 + 2 + D * 4) + B * H * D * D * 8
    peaks, _ = load_peaks()
    line = _line("laplace-core tokens/s (B=4,H=16,L=32K,d_k=64)", world * B * L / (ms / 1e3), "tokens/s",
                 args, world, ms, {"workload": f"LaplacePhaseCore chunk solve, B=4,H=16,L={L},d_k=64,C=64",
                                   "global_batch": B * world, "seq_len": L},
                 roofline={"bound": "hbm", "achieved": alg / (ms / 1e3) / 1e9, "peak": peaks["hbm_gbs"],
                           "unit": "GB/s", "frac": alg / (ms / 1e3) / 1e9 / peaks["hbm_gbs"],
                           "algorithmic_bytes_per_launch": alg}, clocks=clk, gpu_launches=args.steps)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import laplace as olap
        rng = np.random.default_rng(0)
        Ls, u = 2048, 2
        K = np.exp(1j * rng.uniform(0, 2 * np.pi, (1, u, Ls, D))).astype(np.complex64)
        Q = np.exp(1j * rng.uniform(0, 2 * np.pi, (1, u, Ls, D))).astype(np.complex64)
        vv = rng.standard_normal((1, u, Ls, D)).astype(np.float32)
        bb = (2 / (1 + np.exp(-rng.standard_normal((1, u, Ls))))).astype(np.float32)
        rr = np.exp(-np.logaddexp(0, rng.standard_normal((1, u, Ls, D)))).astype(np.float32)
        secs, reps = repeat_for(lambda i: olap.laplace_chunkwise(K, Q, vv, bb, rr, 64, None, dtype=np.float32))
        line["cpu_baseline"] = {"value": reps * u * Ls / H / secs, "unit": "tokens/s", "cores": cpu_threads(),
                                "kind": "port", "sample": f"{reps} x {u} (b,h) units x L={Ls}, numpy float32 port "
                                f"of LaplacePhaseCore.forward's chunk loop, {secs:.1f} s; "
                                "tokens/s = head-tokens / 16 / s"}
    return line


def run_laplace_sp(args, world, rank, local):
    """Sequence-parallel LaplacePhaseCore: one B=4, H=16, L=32768 sequence split into
    `world` contiguous segments, boundary states passed rank to rank over NCCL (one
    micro-group: the kernel's segment time does not shrink with fewer units, so finer
    pipelining only adds stages).  Strong scaling (fixed total work); a step is the whole
    sequence."""
    import torch
    import torch.nn.functional as F
    from delta_phase_b200.sequence_parallel import laplace_chunkwise_sp
    dev = torch.device("cuda", local)
    B, H, L, D = 4, 16, 32768, 64
    Ls = L // world
    g = torch.Generator(device=dev).manual_seed(3000 + rank)
    bf = torch.bfloat16
    tk = (torch.rand(B, H, Ls, D, device=dev, generator=g) * 2 * np.pi).to(bf)
    tq = (torch.rand(B, H, Ls, D, device=dev, generator=g) * 2 * np.pi).to(bf)
    v = torch.randn(B, H, Ls, D, device=dev, generator=g).to(bf)
    logr = (-F.softplus(torch.randn(B, H, Ls, D, device=dev, generator=g))).to(bf)
    beta = (2 * torch.sigmoid(torch.randn(B, H, Ls, device=dev, generator=g))).to(bf)
    out = torch.empty(B, H, Ls, D, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        laplace_chunkwise_sp(tk, None, tq, None, v, logr, beta, 64, None, micro_groups=1, out=out)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    clocks = sampler.stop()
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
    alg = B * H * L * (4 * D * 2 + 2 + D * 4) + B * H * D * D * 8
    peaks, _ = load_peaks()
    line = _line("laplace-core sequence-parallel tokens/s (B=4,H=16,L=32K,d_k=64)", B * L / (ms / 1e3),
                 "tokens/s", args, world, ms,
                 {"workload": "LaplacePhaseCore chunk solve, one B=4,H=16,L=32768 sequence split over the GPUs",
                  "global_batch": B, "seq_len": L,
                  "parallelism": f"sequence parallel over {world} GPU(s), NCCL send/recv of boundary states"},
                 scaling="strong", clocks=clocks,
                 roofline={"bound": "hbm", "achieved": alg / (ms / 1e3) / 1e9 / world, "peak": peaks["hbm_gbs"],
                           "unit": "GB/s", "frac": alg / (ms / 1e3) / 1e9 / world / peaks["hbm_gbs"],
                           "algorithmic_bytes_per_launch": alg // world})
    return line


def run_ffn(args, world, rank, local):
    """Spectral Lerp FFN on 16 x 4096 tokens, d_model = 1024, nb = 4, bf16 activations."""
    import torch
    from delta_phase_b200 import LearnableSubstrateLerpFFN
    dev = torch.device("cuda", local)
    tokens, d, nb = 16 * 4096, 1024, 4
    torch.manual_seed(3000 + rank)
    ffn = LearnableSubstrateLerpFFN(d, nb).to(dev)
    with torch.no_grad():
        for n, p in ffn.named_parameters():
            p.copy_(torch.randn_like(p) * (1.0 if n == "substrate_logits" else 0.02))
    x = torch.randn(tokens, d, device=dev).to(torch.bfloat16)
    stream = torch.cuda.current_stream(dev)
    with torch.no_grad():
        ms, clk = _timed_clk(lambda: ffn(x), args.steps, args.warmup, stream, local)
    ms = max_over_ranks(ms, world)
    flops = tokens * (2 * 6 * d * d + 2 * d * d)  # folded combine GEMM + DCT-II GEMM
    peaks, _ = load_peaks()
    line = _line("lerp-ffn tokens/s (d=1024, nb=4)", world * tokens / (ms / 1e3), "tokens/s", args, world, ms,
                 {"workload": "LearnableSubstrateLerpFFN forward, 65536 tokens, d=1024, nb=4, bf16",
                  "global_batch": 16 * world, "seq_len": 4096},
                 roofline={"bound": "tensor", "achieved": flops / (ms / 1e3) / 1e12,
                           "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                           "frac": flops / (ms / 1e3) / 1e12 / peaks["bf16_tflops"],
                           "flops_per_launch": flops,
                           "note": "folded algorithm: 2*6d^2 + 2d^2 FLOP/token (the reference's own "
                                   "algorithm needs 6*nb*d^2 + 12 d^2 = 37.7 MFLOP/token)"}, clocks=clk)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import spectral as ospec
        params = {k: v.detach().float().cpu().numpy() for k, v in ffn.state_dict().items()}
        xs = x[:512].float().cpu().numpy()
        secs, reps = repeat_for(lambda i: ospec.lerp_ffn(xs, params, dtype=np.float32))
        line["cpu_baseline"] = {"value": reps * 512 / secs, "unit": "tokens/s", "cores": cpu_threads(),
                                "kind": "port", "sample": f"{reps} x 512 tokens, numpy float32 port of "
                                f"LearnableSubstrateLerpFFN.forward, {secs:.1f} s"}
    return line


def run_decode(args, world, rank, local, B=64, H=16, D=64):
    """Decode step on a (B, H, 64, 64) complex state, 256 steps captured in one CUDA graph."""
    import torch
    from delta_phase_b200.kernels import decode_step
    dev = torch.device("cuda", local)
    g = torch.Generator(device=dev).manual_seed(4000 + rank)
    M = torch.randn(B, H, D, D, device=dev, dtype=torch.complex64, generator=g) * 0.1
    n = 256
    tk = torch.rand(n, B, H, D, device=dev, generator=g) * 2 * np.pi
    tq = torch.rand(n, B, H, D, device=dev, generator=g) * 2 * np.pi
    v = torch.randn(n, B, H, D, device=dev, generator=g)
    beta = 2 * torch.sigmoid(torch.randn(n, B, H, device=dev, generator=g))
    out = torch.empty(B, H, D, device=dev)
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for t in range(3):
            decode_step(M, tk[t], tq[t], v[t], beta[t], out=out, state_out=M)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            for t in range(n):
                decode_step(M, tk[t], tq[t], v[t], beta[t], out=out, state_out=M)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    ms, clk = _timed_clk(graph.replay, args.steps, args.warmup, stream, local)
    ms = max_over_ranks(ms / n, world)
    byt = B * H * (2 * D * D * 8 + 3 * D * 4 + 4 + D * 4)
    peaks, _ = load_peaks()
    return _line("decode step latency (B*H=%d, d_k=64)" % (B * H), ms, "ms/step", args, world, ms,
                 {"workload": f"decode step, state ({B},{H},64,64) complex64, fp32 inputs, "
                              f"{n} steps per CUDA graph", "global_batch": B * world},
                 higher_is_better=False, gpu_launches=n * args.steps, clocks=clk,
                 roofline={"bound": "hbm", "achieved": byt / (ms / 1e3) / 1e9, "peak": peaks["hbm_gbs"],
                           "unit": "GB/s", "frac": byt / (ms / 1e3) / 1e9 / peaks["hbm_gbs"],
                           "algorithmic_bytes_per_launch": byt})


def run_lm(args, world, rank, local):
    """DeltaPhase LM, d_model 1024, 16 heads of 64, 12 layers, vocab 32000 (the d_model 768
    configuration cannot be built by the reference): prefill 16 x 4096 tokens, then decode."""
    import torch
    from delta_phase_b200 import DeltaPhaseConfig, DeltaPhaseModel
    dev = torch.device("cuda", local)
    torch.manual_seed(5000 + rank)
    cfg = DeltaPhaseConfig(dim=1024, n_heads=16, n_layers=12, vocab_size=32000, chunk_size=64)
    model = DeltaPhaseModel(cfg).to(dev).eval()
    B, L, ndec = 16, 4096, args.decode_steps
    ids = torch.randint(0, 32000, (B, L), device=dev)
    stream = torch.cuda.current_stream(dev)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        torch.cuda.nvtx.range_push("lm_prefill")  # lets a profiler select the prefill passes
        pre_ms, pre_clk = _timed_clk(lambda: model(ids), max(1, args.steps // 4), 1, stream, local)
        torch.cuda.nvtx.range_pop()
        _, states = model.forward_with_states(ids)
        st = [(None, M) for M in states]
        nxt = ids[:, -1:]

        def dec():
            nonlocal st
            logits, st = model.step(nxt, st)
        dec_eager_ms = _timed(dec, min(ndec, 32), 2, stream)
    # the whole step as one CUDA graph, state buffers updated in place
    from delta_phase_b200 import DecodeGraph
    graph = DecodeGraph(model, B, states=[(None, M) for M in states], autocast_dtype=torch.bfloat16)
    torch.cuda.nvtx.range_push("lm_decode_graph")  # lets a profiler select the decode replays
    dec_ms, dec_clk = _timed_clk(lambda: graph.step(nxt), ndec, 3, stream, local)
    torch.cuda.nvtx.range_pop()
    del graph
    pre_ms = max_over_ranks(pre_ms, world)
    dec_ms = max_over_ranks(dec_ms, world)
    dec_eager_ms = max_over_ranks(dec_eager_ms, world)
    return _line("LM prefill tokens/s (12x1024, 16 heads, vocab 32000)", world * B * L / (pre_ms / 1e3),
                 "tokens/s", args, world, pre_ms,
                 {"workload": "DeltaPhaseModel prefill B=16 x L=4096 then decode, bf16 autocast",
                  "global_batch": B * world, "seq_len": L, "model": "d1024-h16-l12"},
                 decode={"ms_per_token": dec_ms, "steps": ndec, "batch": B,
                         "path": "DecodeGraph (one CUDA graph per token step)",
                         "eager_ms_per_token": dec_eager_ms, "clocks": dec_clk},
                 clocks=pre_clk)


def run_reference(args, world, rank):
    """CPU arm: the reference's own chunkwise path (its public delta_phase_chunkwise_fused,
    torch on the host cores) when installed in baseline/_ref, else the numpy port."""
    if rank != 0:
        return None
    B, H, L, D, C = (CORE[k] for k in ("B", "H", "L", "D", "C"))
    for _ in range(args.warmup):
        cpu_core_baseline(1, L=1024)
    times, ht, kind, desc = [], 0, "port", ""
    for _ in range(args.steps):
        s, ht, kind, desc = cpu_core_baseline(args.cpu_units)
        times.append(s)
    secs = statistics.median(times)
    value = ht / H / secs
    return {
        "metric": METRIC, "impl": "reference", "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": secs * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded, same distributions as the GPU arm)",
        "config": {"workload": "chunkwise complex delta-rule forward, B=8,H=16,L=8192,d_k=64,C=64 "
                               "(timed on a bounded sample of (b,h) units)",
                   "global_batch": B * world, "seq_len": L},
        "cpu_baseline": {"value": value, "unit": "tokens/s",
                         "cores": os.cpu_count() if kind == "reference" else cpu_threads(), "kind": kind,
                         "sample": f"{args.cpu_units} (b,h) units x L=8192 per step (median of {args.steps}), "
                                   f"{desc}; tokens/s = head-tokens/16/s"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def run_secondary(args, world, rank, local):
    """The other workloads, each a few steps, for the headline line's `secondary` object:
    Laplace (B=4, H=16, L=32768), the Lerp FFN (65536 x 1024), the decode step
    (B*H = 1024), the complex-beta core (the headline shape) and the 12-layer LM (prefill
    16 x 4096, decode B=16)."""
    import copy

    import torch
    sub = copy.copy(args)
    sub.no_cpu_baseline = True
    sub.warmup = 3
    out = {}
    keep = ("metric", "value", "unit", "ms_per_step", "higher_is_better", "config", "roofline", "clocks",
            "decode", "gpu_launches")
    for name, fn, steps in (("laplace", run_laplace, 10), ("ffn", run_ffn, 10), ("decode", run_decode, 4),
                            ("cbeta", run_cbeta, 10), ("lm", run_lm, 8)):
        sub.steps = steps
        sub.seq_len = 32768
        sub.decode_steps = 64
        try:
            line = fn(sub, world, rank, local)
            out[name] = {k: line[k] for k in keep if k in line}
        except Exception as e:  # a failing secondary must not hide the headline number
            out[name] = {"error": f"{type(e).__name__}: {e}"[:300]}
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="core",
                    choices=["core", "cbeta", "train", "laplace", "laplace-sp", "ffn", "decode", "lm"])
    ap.add_argument("--decode-steps", type=int, default=256)
    ap.add_argument("--seq-len", type=int, default=32768,
                    help="laplace workload only: sequence length (the headline is 32768; smaller for profiling)")
    ap.add_argument("--cpu-units", type=int, default=16)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--secondary", default="auto", choices=["auto", "on", "off"],
                    help="core workload: also run the other workloads briefly (auto: on one GPU only)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        line = run_reference(args, world, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    world, rank, local = dist_setup(args.gpus)
    run = {"core": run_core, "cbeta": run_cbeta, "train": run_train, "laplace": run_laplace, "laplace-sp": run_laplace_sp,
           "ffn": run_ffn, "decode": run_decode, "lm": run_lm}[args.workload]
    line = run(args, world, rank, local)
    if args.workload == "core" and (args.secondary == "on" or (args.secondary == "auto" and world == 1)):
        line["secondary"] = run_secondary(args, world, rank, local)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
