"""Sequence-parallel LaplacePhaseCore chunk solve (long contexts over several GPUs).

The Laplace recurrence (LaplacePhaseCore.forward, delta_phase/layers.py:481-561) is
exact given the state at the start of a segment, so a sequence split into P contiguous
segments, one per rank, is solved by passing each (batch, head) unit's boundary state
from rank p - 1 to rank p (32 KB per unit at d_k = d_v = 64) with NCCL point-to-point
sends.  The units are pipelined in micro-groups (contiguous batch ranges): rank p solves
micro-group g while rank p + 1 solves g - 1.

What this buys is capacity (each GPU holds L / P tokens), not speed: the kernel's time
for a segment is set by its per-chunk latency, not by how many units it holds, so P
ranks in a pipeline of m micro-groups take (P + m - 1) / P of one GPU's time for the
whole sequence.  m = 1 (the default) is therefore the fastest choice for this kernel:
one GPU's time plus P - 1 state hand-offs.  Micro-groups pay off only for a segment
solver whose time grows with the number of units.
The gated state transition is a per-row 2D x 2D operator (the decay differs per value
channel), so shipping transition operators instead of states (to let all ranks start at
once) would cost d_v times the state per unit; the mode therefore passes states only.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .kernels import laplace_chunkwise


def _batch_ranges(B, micro_groups):
    m = max(1, min(int(micro_groups), B))
    step = -(-B // m)
    return [(b0, min(B, b0 + step)) for b0 in range(0, B, step)]


def laplace_chunkwise_sp(theta_k, logmag_k, theta_q, logmag_q, v, log_decay, beta, chunk_size=32,
                         initial_state=None, group=None, micro_groups=1, segment_fn=None, out=None):
    """Solve this rank's segment of a sequence split over the ranks of ``group``.

    The tensors hold this rank's tokens (rank p owns positions p L_seg .. (p + 1) L_seg of
    every (b, h) unit; segments need not have equal lengths).  ``initial_state`` (complex
    (B, H, Dv, D)) is the state before the whole sequence and is read on rank 0 only.
    Every rank must call this with the same B, H, micro_groups.

    Returns ``(out, M)``: this rank's outputs (B, H, L_seg, Dv) and the state after its
    segment -- on the last rank, the state after the whole sequence.
    ``segment_fn`` (default: the CUDA kernel's ``laplace_chunkwise``) solves one segment
    with the same signature; it is a parameter so the hand-off logic can be exercised on
    any backend.
    """
    seg = laplace_chunkwise if segment_fn is None else segment_fn
    if dist.is_available() and dist.is_initialized():
        rank, world = dist.get_rank(group), dist.get_world_size(group)
    else:  # no process group: one rank holds the whole sequence
        rank, world = 0, 1
    prev_rank = dist.get_global_rank(group, rank - 1) if (group is not None and rank > 0) else rank - 1
    next_rank = (dist.get_global_rank(group, rank + 1) if (group is not None and rank + 1 < world)
                 else rank + 1)
    B, H, L, D = theta_k.shape
    Dv = v.shape[-1]
    dev = theta_k.device
    if out is None:
        out = torch.empty(B, H, L, Dv, device=dev, dtype=torch.float32)
    ranges = _batch_ranges(B, micro_groups)

    # receives posted up front (they match in order); one buffer per micro-group
    recv_bufs, recv_work = [], []
    if rank > 0:
        for b0, b1 in ranges:
            buf = torch.empty(b1 - b0, H, Dv, D, 2, device=dev, dtype=out.dtype)  # (re, im) of the state
            recv_bufs.append(buf)
            recv_work.append(dist.irecv(buf, src=prev_rank, group=group))

    def sl(t, b0, b1):
        return None if t is None else t[b0:b1]

    states, send_work = [], []
    for g, (b0, b1) in enumerate(ranges):
        if rank > 0:
            recv_work[g].wait()
            s_in = torch.view_as_complex(recv_bufs[g])
        else:
            s_in = None if initial_state is None else initial_state[b0:b1]
        _, M_g = seg(sl(theta_k, b0, b1), sl(logmag_k, b0, b1), sl(theta_q, b0, b1), sl(logmag_q, b0, b1),
                     sl(v, b0, b1), sl(log_decay, b0, b1), sl(beta, b0, b1), chunk_size, s_in,
                     out=out[b0:b1])
        states.append(M_g)
        if rank + 1 < world:
            msg = torch.view_as_real(M_g.contiguous())
            send_work.append((dist.isend(msg, dst=next_rank, group=group), msg))  # msg kept alive
    for w, _ in send_work:
        w.wait()
    M = torch.cat(states, 0) if len(states) > 1 else states[0]
    return out, M
