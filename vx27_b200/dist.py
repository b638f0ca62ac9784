"""Multi-GPU plumbing for the attention hot path: one process per GPU, torch.distributed
for process groups and the one collective the path has.

* Sequence sharding (configs 2 and 3a): every sequence's state and KV cache are
  independent, so ranks take disjoint sequence ranges and exchange nothing.
* KV-range sharding of one long sequence (config 3b): rank r owns cache positions
  [r*P/N, (r+1)*P/N); each rank computes a partial record per layer
  (vx27_gqa_partial), one all-gather moves every layer's records to every rank, and
  vx27_gqa_combine merges them (log-sum-exp). The exchange is tiny (24 heads x 258
  floats per layer per rank), so all layers' records travel in a single call.
The helpers work on any backend (NCCL on GPUs, gloo on CPU for the host-side tests).
"""
from __future__ import annotations

import datetime
import os


def shard_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """[begin, end) of rank's share of `total` items, as equal as possible, in order."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(total, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def init_from_env(backend: str, timeout_s: int = 120):
    """Initialises the default process group from torchrun's environment; returns
    (rank, world, local_rank). A short timeout makes a missing rank end the job with an
    error instead of a hang."""
    import torch
    import torch.distributed as dist
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        kw = dict(timeout=datetime.timedelta(seconds=timeout_s))
        if backend == "nccl":
            torch.cuda.set_device(local)
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend, **kw)
    return rank, world, local


def gather_records(local, world: int, group=None):
    """All-gather of this rank's records (a flat tensor) -> tensor [world, numel]."""
    import torch
    import torch.distributed as dist
    flat = local.reshape(-1)
    out = torch.empty(world * flat.numel(), dtype=flat.dtype, device=flat.device)
    if world == 1:
        out.copy_(flat)
    else:
        dist.all_gather_into_tensor(out, flat, group=group)  # flat output: gloo and NCCL
    return out.view(world, flat.numel())
