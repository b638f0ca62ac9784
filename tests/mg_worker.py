"""Rank program of tests/test_multigpu.py (launched by torchrun, one process per GPU):
config 3b's KV-sharded decode over NCCL compared with the unsharded decode on rank 0,
and config 2's sequence-sharded step on every rank."""
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from vx27_b200.dist import init_from_env  # noqa: E402
from vx27_b200.hybrid import HybridConfig, HybridDecoder  # noqa: E402
from vx27_b200.longctx import LongContextGQA  # noqa: E402


def main(out_path):
    rank, world, local = init_from_env("nccl", timeout_s=120)
    P, layers = 9000, 2
    shard = LongContextGQA(1, ctx=P, layers=layers, rank=rank, world=world, split_kv=True)
    shard.step()
    torch.cuda.synchronize()
    res = {}
    if rank == 0:
        whole = LongContextGQA(1, ctx=P, layers=layers)
        whole.step()
        torch.cuda.synchronize()
        a, b = shard.out.float(), whole.out.float()
        res["split_kv_rel_err"] = float((a - b).abs().max() / b.abs().max())
    # every rank holds the same merged output
    out = shard.out.float().reshape(-1)
    gathered = torch.empty(world * out.numel(), device=out.device)
    dist.all_gather_into_tensor(gathered, out)
    g = gathered.view(world, -1)
    res["ranks_agree"] = bool(all(torch.equal(g[0], g[r]) for r in range(world)))
    # sequence-sharded hybrid step: each rank its own sequences
    dec = HybridDecoder(HybridConfig(batch=2, ctx=256, steps=2, seed=2 + 1000 * rank))
    dec.step()
    torch.cuda.synchronize()
    ok = torch.tensor([1.0 if torch.isfinite(dec.att_out.float()).all() else 0.0], device="cuda")
    dist.all_reduce(ok)
    res["hybrid_finite_ranks"] = int(ok.item())
    if rank == 0:
        with open(out_path, "w") as f:
            json.dump(res, f)
    del shard, dec
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])
