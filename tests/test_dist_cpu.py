"""Host-side logic of the multi-GPU paths, on CPU ranks (gloo, world size 2): the shard
partition, and the config 3b exchange -- each rank's partial record over its KV range,
one all-gather (vx27_b200.dist.gather_records), the log-sum-exp combine -- equals the
single-pass attention. The per-rank arithmetic is the CPU oracle's; the GPU kernels of the
same records are checked in test_gqa_gpu.py / test_longctx_gpu.py."""
import os
import socket

import numpy as np
import pytest

from vx27_b200.dist import shard_range


def test_shard_range_partitions_in_order():
    for total in (0, 1, 7, 16, 262144, 262145):
        for world in (1, 2, 3, 8):
            spans = [shard_range(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [e - b for b, e in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, out_dir):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    from oracle import oracle as orc
    from vx27_b200.dist import gather_records, init_from_env
    init_from_env("gloo", timeout_s=60)
    nq, nkv, hd, P = 24, 4, 256, 700
    kc = orc.normal(nkv * P * hd, 5, 1, bf16=True)
    vc = orc.normal(nkv * P * hd, 5, 2, bf16=True)
    q = orc.normal(nq * hd, 5, 3)
    gate = orc.normal(nq * hd, 5, 4, bf16=True)
    b, e = shard_range(P, world, rank)
    # this rank's shard of the cache, as the rank would hold it
    ks = np.ascontiguousarray(kc.reshape(nkv, P, hd)[:, b:e]).reshape(-1)
    vs = np.ascontiguousarray(vc.reshape(nkv, P, hd)[:, b:e]).reshape(-1)
    o_part = np.zeros(nq * hd, np.float32)
    ml = np.zeros(nq * 2, np.float32)
    orc.lib().orc_gqa_partial(orc.P(q), orc.P(ks), orc.P(vs), e - b, 0, e - b, orc.P(o_part),
                              orc.P(ml), nq, nkv, hd)
    rec = torch.from_numpy(np.concatenate([o_part, ml]))
    allrec = gather_records(rec, world).numpy()  # [world, nq*hd + nq*2]
    o_all = np.ascontiguousarray(allrec[:, :nq * hd])
    ml_all = np.ascontiguousarray(allrec[:, nq * hd:])
    out = np.zeros(nq * hd, np.float32)
    orc.lib().orc_gqa_combine(orc.P(o_all), orc.P(ml_all), world, orc.P(gate), orc.P(out), nq, hd,
                              orc.F_ACT_BF16)
    full = np.zeros(nq * hd, np.float32)
    pos = np.array([P - 1], np.int32)
    orc.lib().orc_gqa_attend(orc.P(q), orc.P(gate), orc.P(kc), orc.P(vc), P, orc.P(pos),
                             orc.P(full), 1, nq, nkv, hd, orc.F_ACT_BF16)
    np.save(os.path.join(out_dir, f"r{rank}.npy"), np.stack([out, full]))
    dist.destroy_process_group()


def test_split_kv_exchange_on_two_cpu_ranks(tmp_path):
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    for r in range(world):
        out, full = np.load(tmp_path / f"r{r}.npy")
        assert np.abs(out - full).max() <= 1e-5 * np.abs(full).max()


def _leaving_rank_main(rank, world, port, out_dir):
    import time
    import torch
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    from vx27_b200.dist import gather_records, init_from_env
    init_from_env("gloo", timeout_s=5)
    if rank == 1:
        os._exit(0)  # leaves between steps, with no collective of its own in flight
    t0 = time.time()
    try:
        gather_records(torch.zeros(8), world)
        res = "no-error"
    except Exception as e:  # the collective must end with an error, not hang
        res = type(e).__name__
    with open(os.path.join(out_dir, "r0.txt"), "w") as f:
        f.write(f"{res} {time.time() - t0:.1f}")
    os._exit(0)


def test_a_rank_that_leaves_ends_the_others_collective_with_an_error(tmp_path):
    """Failure detection on the host: a rank exits between steps; the surviving rank's
    next all-gather (the config 3b exchange) fails within the short process-group timeout
    instead of waiting forever."""
    import time
    import torch.multiprocessing as mp
    ctx = mp.start_processes(_leaving_rank_main, args=(2, _free_port(), str(tmp_path)),
                             nprocs=2, join=False, start_method="spawn")
    deadline = time.time() + 120
    while not ctx.join(timeout=1):
        if time.time() > deadline:
            for p in ctx.processes:
                p.kill()
            pytest.fail("the surviving rank did not return")
    res, secs = (tmp_path / "r0.txt").read_text().split()
    assert res != "no-error" and float(secs) < 60, (res, secs)
