"""Row sharding of the conversion and GEMM path across the GPUs of one node.

The path has no exchange step: every conversion is elementwise over rows and
the GEMM is independent per block of output rows (M) with B replicated. Each
process (one per GPU, torchrun) therefore converts or multiplies its own
contiguous block of rows and nothing crosses NVLink on the data path. The
optional replicated-output mode gathers the row blocks to every rank with one
all-gather (NCCL over NVLink/NVSwitch on GPUs, gloo on CPU), for callers that
need the full result everywhere.

Failure detection between steps: a rank that leaves the job between two
steps announces it in the process group's key-value store (`announce_leave`,
before the barrier that closes its last step), and every other rank checks
the store before it launches its next step (`check_peers`), so the survivors
stop on the host with `PeerLeft` instead of entering a collective that can
never complete.

The reference is single-device and has no counterpart of this module.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist


def shard_rows(total: int, world_size: int, rank: int) -> tuple[int, int]:
    """Contiguous, balanced [start, stop) row block of `rank` (the first
    total % world_size ranks get one extra row)."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError(f"bad rank {rank} of {world_size}")
    base, extra = divmod(total, world_size)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def _world(group):
    if not dist.is_available() or not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


def gather_rows(local: torch.Tensor, total_rows: int, group=None) -> torch.Tensor:
    """All-gather row blocks produced by shard_rows into the full tensor on
    every rank. Blocks are padded to the largest block size so that a single
    all_gather_into_tensor (one NCCL call) moves them."""
    ws, _ = _world(group)
    if ws == 1:
        return local
    rows_max = shard_rows(total_rows, ws, 0)[1]
    tail = tuple(local.shape[1:])
    # byte view so that fp8/fp4 payloads travel unchanged
    dt = local.dtype
    row_bytes = local.element_size()
    for d in tail:
        row_bytes *= d
    lb = local.contiguous().view(torch.uint8).reshape(local.shape[0], row_bytes)
    if total_rows % ws == 0:  # equal blocks: gather straight into the result, no padding or concatenation
        full = torch.empty((total_rows,) + tail, dtype=dt, device=local.device)
        fb = full.view(torch.uint8).reshape(total_rows, row_bytes)
        if dist.get_backend(group) == "nccl":
            dist.all_gather_into_tensor(fb, lb, group=group)
        else:
            dist.all_gather(list(fb.chunk(ws)), lb, group=group)
        return full
    padded = torch.zeros((rows_max, row_bytes), dtype=torch.uint8, device=local.device)
    padded[: lb.shape[0]] = lb
    out = torch.empty((ws * rows_max, row_bytes), dtype=torch.uint8, device=local.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, padded, group=group)
    else:
        dist.all_gather(list(out.chunk(ws)), padded, group=group)
    parts = []
    for r in range(ws):
        s, e = shard_rows(total_rows, ws, r)
        parts.append(out[r * rows_max: r * rows_max + (e - s)])
    full = torch.cat(parts)
    return full.view(dt).reshape((total_rows,) + tail)


def sharded_rows_apply(x: torch.Tensor, fn: Callable[[torch.Tensor], torch.Tensor], group=None,
                       gather: bool = False) -> torch.Tensor:
    """Apply a row-wise function (a conversion) to this rank's block of rows
    of `x`; with gather=True return the full result on every rank."""
    ws, rank = _world(group)
    s, e = shard_rows(x.shape[0], ws, rank)
    local = fn(x[s:e])
    return gather_rows(local, x.shape[0], group) if gather else local


def sharded_scaled_mm(a: torch.Tensor, mat2: torch.Tensor, scale_a: torch.Tensor, scale_b: torch.Tensor,
                      group=None, gather: bool = False, **kwargs) -> torch.Tensor:
    """torch._scaled_mm with A's rows (M) split across ranks and mat2
    replicated; rowwise scale_a is split with A. Returns this rank's rows, or
    the full (M, N) result on every rank with gather=True."""
    ws, rank = _world(group)
    M = a.shape[0]
    s, e = shard_rows(M, ws, rank)
    sa = scale_a[s:e] if scale_a.numel() > 1 else scale_a
    local = torch._scaled_mm(a[s:e], mat2, sa, scale_b, **kwargs)
    return gather_rows(local, M, group) if gather else local


class PeerLeft(RuntimeError):
    """A rank of the job announced that it left between steps."""


def _leave_key(rank: int) -> str:
    return f"fp8b200/left/{rank}"


def announce_leave(store, rank: int) -> None:
    """Record in the job's store that `rank` leaves. Call it in the rank's
    last step before the collective that closes the step (a barrier), so that
    every other rank finds the record when it next calls check_peers; then
    leave with no kernel or collective in flight."""
    store.set(_leave_key(rank), "1")


def check_peers(store, world_size: int, rank: int) -> None:
    """Raise PeerLeft if any other rank announced that it left. A non-blocking
    store lookup per rank; call it before launching a step's kernels and
    collectives."""
    gone = [r for r in range(world_size) if r != rank and store.check([_leave_key(r)])]
    if gone:
        raise PeerLeft(f"rank(s) {gone} left the job; rank {rank} stops before its next step")
