"""The CUDA-core split-KV decode (gqa_cc.cu, VX27_F_DECODE_CC), the measured alternative
to the tensor-core decode, against the CPU oracle (the reference's decode attention,
src/vx27_qfwd.c:347-371, over the same bf16 cache) and against the tensor-core kernel on
the same inputs.

Covers ragged positions on both sides of the 32-position stage edges, forced split counts
(one split writes the gated output itself; several are merged by the combine), fp32 and
bf16 activations and outputs, group sizes 1-8, the fused prologue (q from raw
activations, the new K/V row appended bit-identical to vx27_gqa_append), config 1, and the
early cache requests of VX27_F_PREFETCH_KV. Tolerance: 1e-4 relative (the bound of the
other decode tests; the north star allows 2e-2)."""
import numpy as np
import pytest
import torch

from gpu_util import dev, host, rel_err
from test_gqa_gpu import gpu_step, oracle_step, setup
from vx27_b200 import ops

pytestmark = pytest.mark.gpu
NQ, NKV, HD = 24, 4, 256
TOL = 1e-4


@pytest.fixture(scope="module")
def rope(cuda):
    return ops.rope_table(300000)


def _decode(x, B, cap, rope, kernel, n_splits=0, bf16=True, out_bf16=False, fused=False,
            prefetch=False, nq=NQ, nkv=NKV):
    """One decode step on the GPU: append + decode (or the fused form); returns
    (cache K, cache V, out) on the host."""
    kc = dev(x["kc"], True).view(B, nkv, cap, HD)
    vc = dev(x["vc"], True).view(B, nkv, cap, HD)
    qi = dev(x["qi"], bf16).view(B, nq, HD)
    ki = dev(x["ki"], bf16).view(B, nkv, HD)
    vi = dev(x["vi"], bf16).view(B, nkv, HD)
    gate = dev(x["gate"], bf16).view(B, nq, HD)
    pos = dev(x["pos"])
    ws = torch.empty(ops.gqa_workspace_bytes(B, nq, nkv, HD, cap, n_splits) // 4 + 1,
                     device="cuda")
    out = torch.empty(B, nq, HD, device="cuda",
                      dtype=torch.bfloat16 if out_bf16 else torch.float32)
    if fused:
        n = ops.gqa_decode_fused(qi, ki, vi, dev(x["qw"]), dev(x["kw"]), rope, gate, kc, vc, pos,
                                 out, ws, n_splits=n_splits, kernel=kernel, prefetch_kv=prefetch)
    else:
        q = torch.empty(B, nq, HD, device="cuda")
        ops.gqa_append(qi, ki, vi, dev(x["qw"]), dev(x["kw"]), rope, pos, kc, vc, q)
        n = ops.gqa_decode_batch(q, gate, kc, vc, pos, out, ws, n_splits=n_splits, kernel=kernel,
                                 prefetch_kv=prefetch)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    kind, splits, launches = ops.gqa_decode_plan(B, nq, nkv, HD, cap, ws.numel() * 4, n_splits,
                                                 kernel)
    assert n == launches and (kernel == "auto" or kind == kernel)
    return host(kc).reshape(-1), host(vc).reshape(-1), host(out.float()).reshape(-1)


RAGGED = [0, 1, 31, 32, 33, 127, 128, 1000]


@pytest.mark.parametrize("n_splits", [0, 1, 3, 7])
def test_cc_ragged_positions(cuda, orc, rope, n_splits):
    B, cap = len(RAGGED), 1024
    x = setup(orc, 51, B, cap, RAGGED)
    _, _, _, ref = oracle_step(orc, x, B, cap)
    _, _, out = _decode(x, B, cap, rope, "cc", n_splits)
    assert rel_err(out, ref) < TOL


@pytest.mark.parametrize("bf16,out_bf16", [(False, False), (True, True)])
def test_cc_activation_and_output_types(cuda, orc, rope, bf16, out_bf16):
    B, cap = 3, 400
    x = setup(orc, 52, B, cap, [5, 399, 200], bf16=bf16)
    _, _, _, ref = oracle_step(orc, x, B, cap, bf16=bf16)
    for n_splits in (1, 4):
        _, _, out = _decode(x, B, cap, rope, "cc", n_splits, bf16=bf16, out_bf16=out_bf16)
        if out_bf16:
            assert np.all(np.abs(out - ref) <= np.abs(ref) * 2.0 ** -8 + TOL * np.abs(ref).max())
        else:
            assert rel_err(out, ref) < TOL


@pytest.mark.parametrize("nq,nkv", [(8, 8), (16, 8), (16, 4), (32, 4)])
def test_cc_group_sizes(cuda, orc, rope, nq, nkv):
    B, cap = 2, 300
    g = lambda n, s, m=0.0, sd=1.0, b=True: orc.normal(n, 53, s, m, sd, bf16=b)
    x = dict(kc=g(B * nkv * cap * HD, 1), vc=g(B * nkv * cap * HD, 2), qi=g(B * nq * HD, 3),
             ki=g(B * nkv * HD, 4), vi=g(B * nkv * HD, 5), gate=g(B * nq * HD, 6),
             qw=g(HD, 7, 1.0, 0.02, False), kw=g(HD, 8, 1.0, 0.02, False),
             pos=np.array([100, 299], np.int32))
    L, P = orc.lib(), orc.P
    kc, vc = x["kc"].copy(), x["vc"].copy()
    qo = np.zeros(B * nq * HD, np.float32)
    L.orc_gqa_append(P(x["qi"]), P(x["ki"]), P(x["vi"]), P(x["qw"]), P(x["kw"]), P(x["pos"]),
                     P(kc), P(vc), cap, P(qo), B, nq, nkv, HD, 64, 1e7, 1e-6, orc.F_ACT_BF16)
    ref = np.zeros(B * nq * HD, np.float32)
    L.orc_gqa_attend(P(qo), P(x["gate"]), P(kc), P(vc), cap, P(x["pos"]), P(ref), B, nq, nkv, HD,
                     orc.F_ACT_BF16)
    for fused in (False, True):
        _, _, out = _decode(x, B, cap, rope, "cc", 3, fused=fused, nq=nq, nkv=nkv)
        assert rel_err(out, ref) < TOL


@pytest.mark.parametrize("n_splits", [0, 1, 5])
def test_cc_fused_appends_like_gqa_append(cuda, orc, rope, n_splits):
    B, cap = len(RAGGED), 1024
    x = setup(orc, 54, B, cap, RAGGED)
    _, _, _, ref = oracle_step(orc, x, B, cap)
    kc_a, vc_a, _ = _decode(x, B, cap, rope, "tc", 1)  # vx27_gqa_append's rows
    kc_f, vc_f, out = _decode(x, B, cap, rope, "cc", n_splits, fused=True)
    assert np.array_equal(kc_f, kc_a) and np.array_equal(vc_f, vc_a)
    assert rel_err(out, ref) < TOL


def test_cc_config1_matches_oracle_and_tensor_cores(cuda, orc, rope):
    """Config 1: batch 1, ctx 8192 (cache 0..8190 ~N(0,1) bf16, token at 8191), seed 1."""
    B, cap = 1, 8192
    x = setup(orc, 1, B, cap, [8191])
    _, _, _, ref = oracle_step(orc, x, B, cap)
    _, _, out_cc = _decode(x, B, cap, rope, "cc", fused=True)
    _, _, out_tc = _decode(x, B, cap, rope, "tc")
    assert rel_err(out_cc, ref) < TOL
    assert rel_err(out_tc, out_cc) < TOL


@pytest.mark.parametrize("fused", [False, True])
def test_cc_prefetch_gives_the_same_bits(cuda, orc, rope, fused):
    """VX27_F_PREFETCH_KV requests cache rows before the previous kernel (the append) ends;
    the row the append writes is requested after it, so the bits do not change."""
    B, cap = 3, 700
    x = setup(orc, 55, B, cap, [699, 64, 333])
    for n_splits in (1, 4):
        _, _, a = _decode(x, B, cap, rope, "cc", n_splits, fused=fused)
        _, _, b = _decode(x, B, cap, rope, "cc", n_splits, fused=fused, prefetch=True)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_cc_and_tc_agree_on_a_wide_batch(cuda, orc, rope):
    """The library's tensor-core choice and the CUDA-core kernel on the same batch give
    the same attention within the tolerance."""
    B, cap = 64, 520
    pos = np.arange(B, dtype=np.int32) * 8 + 3
    x = setup(orc, 56, B, cap, pos)
    _, _, _, ref = oracle_step(orc, x, B, cap)
    assert ops.gqa_decode_plan(B, NQ, NKV, HD, cap, 1 << 30)[0] == "tc"
    _, _, out_tc = _decode(x, B, cap, rope, "auto")
    _, _, out_cc = _decode(x, B, cap, rope, "cc")
    assert rel_err(out_tc, ref) < TOL and rel_err(out_cc, ref) < TOL


@pytest.mark.parametrize("fused", [False, True])
def test_tc_prefetch_gives_the_same_bits(cuda, orc, rope, fused):
    """The tensor-core kernel with VX27_F_PREFETCH_KV: the first ring round is requested
    before the previous kernel ends, the tile with the token's row after it."""
    B, cap = 3, 700
    x = setup(orc, 57, B, cap, [699, 64, 333])
    _, _, _, ref = oracle_step(orc, x, B, cap)
    for n_splits in (1, 4):
        _, _, a = _decode(x, B, cap, rope, "tc", n_splits, fused=fused)
        _, _, b = _decode(x, B, cap, rope, "tc", n_splits, fused=fused, prefetch=True)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
        assert rel_err(b, ref) < TOL
