"""bench.py's NCCL log plumbing on a real communicator (one GPU, one rank): NCCL writes its
INIT lines to the per-process file that nccl_debug_env names, echo_nccl_log copies them to
stderr, and stdout carries nothing of NCCL's."""
import os
import socket
import subprocess
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SCRIPT = r"""
import datetime, os, sys
sys.path.insert(0, {root!r})
import bench
path = bench.nccl_debug_env(2, os.environ)   # as a rank of a two-rank run would
import torch, torch.distributed as dist
torch.cuda.set_device(0)
dist.init_process_group("nccl", init_method="tcp://127.0.0.1:{port}", rank=0, world_size=1,
                        timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", 0))
dist.barrier()
bench.echo_nccl_log(path, sys.stderr)
dist.destroy_process_group()
print("log removed" if not os.path.exists(path) else "log left")
"""


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.gpu
def test_nccl_init_lines_reach_stderr_not_stdout():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    env = {k: v for k, v in os.environ.items() if not k.startswith("NCCL_DEBUG")}
    r = subprocess.run([sys.executable, "-c", SCRIPT.format(root=ROOT, port=_free_port())], env=env,
                       capture_output=True, text=True, timeout=180)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == "log removed", r.stdout
    assert "NCCL INFO" in r.stderr, r.stderr[-2000:]
