"""bench.py's host-side plumbing for multi-rank runs (no GPU): where NCCL's communicator
set-up lines go, and that they reach stderr without touching stdout (the result line)."""
import io
import os

import bench


def test_single_rank_sets_nothing():
    env = {}
    assert bench.nccl_debug_env(1, env) is None
    assert env == {}


def test_caller_setting_is_kept():
    env = {"NCCL_DEBUG": "WARN"}
    assert bench.nccl_debug_env(4, env) is None
    assert env == {"NCCL_DEBUG": "WARN"}


def test_multi_rank_logs_to_a_file_of_this_process():
    env = {"NCCL_DEBUG_SUBSYS": "INIT,NET"}
    path = bench.nccl_debug_env(2, env)
    assert path is not None and str(os.getpid()) in os.path.basename(path)
    assert env["NCCL_DEBUG"] == "INFO"
    assert env["NCCL_DEBUG_FILE"] == path
    assert env["NCCL_DEBUG_SUBSYS"] == "INIT,NET"  # a caller's subsystem list stays


def test_log_is_echoed_once_and_removed(tmp_path):
    path = tmp_path / "nccl.log"
    lines = "host:1:1 NCCL INFO comm 0x1 rank 0 nRanks 2 nNodes 1 localRanks 2 localRank 0\n" \
            "host:1:1 NCCL INFO ncclCommInitRankConfig comm 0x1 rank 0 nranks 2 - Init COMPLETE"
    path.write_text(lines)
    out = io.StringIO()
    bench.echo_nccl_log(str(path), out)
    assert out.getvalue() == lines + "\n"
    assert not path.exists()


def test_missing_log_writes_nothing(tmp_path):
    out = io.StringIO()
    bench.echo_nccl_log(str(tmp_path / "absent.log"), out)
    bench.echo_nccl_log(None, out)
    assert out.getvalue() == ""
