"""vx27_gqa_decode_batch_noalloc, the decode entry point for callers that cannot give the
library device scratch (their device memory is already spoken for, or they reach the
library through a C interface with no workspace argument). Called through the C ABI and
checked on three calls in a row with different inputs against vx27_gqa_decode_batch, which
takes a caller workspace (bit for bit: same split count, same kernels), and against the
CPU oracle, so contents left in the shared static scratch by one call cannot leak into the
next. This file sorts last so a run that stops at the first
failure has run every other test before it."""
import ctypes as C

import numpy as np
import pytest
import torch

from gpu_util import dev, host, rel_err
from vx27_b200 import ops
from vx27_b200._lib import errbuf, load

pytestmark = pytest.mark.gpu
NQ, NKV, HD = 24, 4, 256
TOL = 1e-4  # the GQA decode tests' own bound against the CPU oracle


def _inputs(orc, seed, B, cap, pos):
    g = lambda n, s, b=True: orc.normal(n, seed, s, bf16=b)
    kc = dev(g(B * NKV * cap * HD, 1), True).view(B, NKV, cap, HD)
    vc = dev(g(B * NKV * cap * HD, 2), True).view(B, NKV, cap, HD)
    q = dev(g(B * NQ * HD, 3, False)).view(B, NQ, HD)
    gate = dev(g(B * NQ * HD, 4), True).view(B, NQ, HD)
    return q, gate, kc, vc, dev(np.asarray(pos, np.int32))


def _with_workspace(q, gate, kc, vc, pos, n_splits):
    B, cap = q.shape[0], kc.shape[2]
    ws = torch.empty(ops.gqa_workspace_bytes(B, NQ, NKV, HD, cap, n_splits) // 4 + 1,
                     device="cuda")
    out = torch.empty(B, NQ, HD, device="cuda")
    ops.gqa_decode_batch(q, gate, kc, vc, pos, out, ws, n_splits=n_splits)
    return out


def _noalloc(q, gate, kc, vc, pos, n_splits, out):
    B, cap = q.shape[0], kc.shape[2]
    e = errbuf()
    p = lambda t: C.c_void_p(t.data_ptr())
    rc = load().vx27_gqa_decode_batch_noalloc(
        p(q), p(gate), p(kc), p(vc), cap, p(pos), p(out), B, NQ, NKV, HD, n_splits,
        ops.F_ACT_BF16, C.c_void_p(torch.cuda.current_stream().cuda_stream), e, 512)
    return rc, e.value.decode(), out


def _oracle(orc, q, gate, kc, vc, pos):
    """The reference's decode attention (src/vx27_qfwd.c:347-371) over the same bf16 cache."""
    L, P = orc.lib(), orc.P
    B, cap = q.shape[0], kc.shape[2]
    h = lambda t: host(t).reshape(-1)
    out = np.zeros(B * NQ * HD, np.float32)
    L.orc_gqa_attend_mt(P(h(q)), P(h(gate)), P(h(kc)), P(h(vc)), cap, P(h(pos)), P(out), B, NQ,
                        NKV, HD, orc.F_ACT_BF16, 8)
    return out


def test_noalloc_matches_workspace_entry_point_twice(cuda, orc):
    calls = [(71, 3, 700, [699, 5, 300], 4),    # first call: 4 splits, ragged positions
             (72, 2, 1100, [1099, 0], 0),       # second: other shapes, automatic splits
             (74, 1, 200, [150], 1)]            # one split: the kernel writes out directly
    for n, (seed, B, cap, pos, n_splits) in enumerate(calls):
        x = _inputs(orc, seed, B, cap, pos)
        ref = _with_workspace(*x, n_splits).cpu().numpy().reshape(-1)
        out = torch.empty(x[0].shape[0], NQ, HD, device="cuda")
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        rc, msg, out = _noalloc(*x, n_splits, out)
        torch.cuda.synchronize()
        assert rc == 0, msg
        if n > 0:  # the device symbol is resolved on the first call; later calls allocate nothing
            assert torch.cuda.mem_get_info()[0] == free_before
        got = out.cpu().numpy().reshape(-1)
        # same split count and kernels as the workspace entry point: the same bits
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
        assert rel_err(got, _oracle(orc, *x)) < TOL
        assert ops.device_status() == 0


def test_noalloc_rejects_batches_beyond_the_static_scratch(cuda, orc):
    x = _inputs(orc, 73, 1, 256, [255])
    rc, msg, _ = _noalloc(*x, 100000, torch.empty(1, NQ, HD, device="cuda"))
    assert rc == -1 and "static scratch" in msg
    B = 400  # one record: 400*24*258*4 bytes > 8 MiB
    rc = load().vx27_gqa_decode_batch_noalloc(
        C.c_void_p(x[0].data_ptr()), C.c_void_p(x[1].data_ptr()), C.c_void_p(x[2].data_ptr()),
        C.c_void_p(x[3].data_ptr()), 256, C.c_void_p(x[4].data_ptr()),
        C.c_void_p(x[0].data_ptr()), B, NQ, NKV, HD, 0, ops.F_ACT_BF16, None, errbuf(), 512)
    assert rc == -1
