"""Multi-GPU paths on >= 2 GPUs of one box (skipped with fewer): KV-sharded long-context
decode with the NCCL all-gather of partial records equals the unsharded decode, every
rank ends with the same output, and sequence-sharded hybrid steps run independently."""
import json
import os
import socket
import subprocess
import sys

import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_two_rank_split_kv_and_sequence_sharding(cuda, tmp_path):
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 GPUs")
    out = tmp_path / "mg.json"
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
           "--master-port", str(_port()), os.path.join(ROOT, "tests", "mg_worker.py"), str(out)]
    r = subprocess.run(cmd, capture_output=True, text=True, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.loads(out.read_text())
    assert res["split_kv_rel_err"] < 1e-2  # bf16 outputs of nearly equal fp32 values
    assert res["ranks_agree"]
    assert res["hybrid_finite_ranks"] == 2


def test_two_devices_in_one_process(cuda):
    """One host process driving two GPUs: every kernel with a large shared-memory request
    (split-KV decode, DeltaNet decode, both prefill kernels, the BP3 matvec) launches on
    each device and gives the same result there."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import numpy as np
    import oracle.oracle as O
    from vx27_b200 import ops

    def run(dev):
        torch.cuda.set_device(dev)
        bf = torch.bfloat16
        outs = []
        # split-KV decode (one split: direct gated output)
        B, nq, nkv, hd, cap = 8, 24, 4, 256, 300
        kc = torch.empty(B, nkv, cap, hd, dtype=bf, device=dev)
        vc = torch.empty_like(kc)
        q = torch.empty(B, nq, hd, device=dev)
        gate = torch.empty(B, nq, hd, dtype=bf, device=dev)
        for n, t in enumerate((kc, vc, q, gate)):
            ops.fill_normal(t, 5, n)
        out = torch.empty(B, nq, hd, device=dev)
        pos = torch.full((B,), cap - 1, dtype=torch.int32, device=dev)
        ws = torch.empty(ops.gqa_workspace_bytes(B, nq, nkv, hd, cap, 1) // 4 + 1, device=dev)
        ops.gqa_decode_batch(q, gate, kc, vc, pos, out, ws, n_splits=1)
        outs.append(out.cpu())
        # DeltaNet decode
        nqk = nv = 16
        C = (2 * nqk + nv) * 128
        S = torch.empty(B, nv, 128, 128, device=dev)
        ring = torch.zeros(B, 4, C, device=dev)
        qkv = torch.empty(B, C, dtype=bf, device=dev)
        a = torch.empty(B, nv, dtype=bf, device=dev)
        b = torch.empty_like(a)
        w = torch.empty(C, 4, device=dev)
        A = torch.full((nv,), 0.5, device=dev)
        dt = torch.zeros(nv, device=dev)
        for n, t in enumerate((S, qkv, a, b, w)):
            ops.fill_normal(t, 6, n, 0.0, 0.05 if n == 0 else 1.0)
        o = torch.empty(B, nv, 128, device=dev)
        ops.deltanet_decode_batch(S, ring, qkv, a, b, A, dt, w, torch.zeros(B, dtype=torch.int32,
                                  device=dev), o, nqk, nv)
        outs += [o.cpu(), S.cpu()]
        # BP3 matvec
        W = O.packed_weights(O.PMAT_BP3, 64, 1024, 9)
        x = torch.from_numpy(np.random.default_rng(2).standard_normal((3, 1024)).astype(np.float32))
        y = torch.empty(3, 64, device=dev)
        ops.pmat_batch(torch.from_numpy(W).to(dev), O.PMAT_BP3, x.to(dev), y, 64, 1024)
        outs.append(y.cpu())
        torch.cuda.synchronize(dev)
        assert ops.device_status() == 0
        return outs

    r0, r1 = run(0), run(1)
    for u, v in zip(r0, r1):
        assert torch.equal(u, v)
