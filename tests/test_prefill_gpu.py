"""K4 (vx27_gqa_prefill, causal gated GQA prefill on the tensor cores) against the CPU
oracle (orc_gqa_prefill_rows: the per-token decode path of src/vx27_qfwd.c:339-371 applied
to every prompt position). Tolerance: 2e-2 relative (max-abs error over max-abs value);
q and p enter the tensor cores as bf16."""
import numpy as np
import pytest
import torch

from gpu_util import dev, host, rel_err
from vx27_b200 import ops

pytestmark = pytest.mark.gpu
NQ, NKV, HD = 24, 4, 256
REL_TOL = 2e-2


def make(orc, seed, T, nq=NQ, nkv=NKV, bf16=True):
    g = lambda n, s, m=0.0, sd=1.0, b=bf16: orc.normal(n, seed, s, m, sd, bf16=b)
    return dict(q=g(T * nq * HD, 1), k=g(T * nkv * HD, 2), v=g(T * nkv * HD, 3),
                gate=g(T * nq * HD, 4), qw=g(HD, 5, 1.0, 0.02, False),
                kw=g(HD, 6, 1.0, 0.02, False), nq=nq, nkv=nkv, bf16=bf16)


def oracle_rows(orc, x, T, rows):
    nq, nkv = x["nq"], x["nkv"]
    rows = np.asarray(rows, np.int32)
    out = np.zeros(len(rows) * nq * HD, np.float32)
    orc.lib().orc_gqa_prefill_rows(orc.P(x["q"]), orc.P(x["k"]), orc.P(x["v"]), orc.P(x["gate"]),
                                   orc.P(x["qw"]), orc.P(x["kw"]), T, nq, nkv, HD, 64, 1e7, 1e-6,
                                   orc.P(rows), len(rows), orc.P(out),
                                   orc.F_ACT_BF16 if x["bf16"] else 0)
    return out.reshape(len(rows), nq, HD)


def gpu_prefill(x, T, cap, rope, chunks=None, out_bf16=False, cta_pairs=True):
    """Prefill in one call, or in consecutive chunks (p0 > 0 continues the cache)."""
    nq, nkv, b16 = x["nq"], x["nkv"], x["bf16"]
    q = dev(x["q"], b16).view(T, nq, HD)
    k = dev(x["k"], b16).view(T, nkv, HD)
    v = dev(x["v"], b16).view(T, nkv, HD)
    gate = dev(x["gate"], b16).view(T, nq, HD)
    kc = torch.full((nkv, cap, HD), float("nan"), dtype=torch.bfloat16, device="cuda")
    vc = torch.full((nkv, cap, HD), float("nan"), dtype=torch.bfloat16, device="cuda")
    out = torch.empty(T, nq, HD, dtype=torch.bfloat16 if out_bf16 else torch.float32,
                      device="cuda")
    bounds = chunks or [0, T]
    for a, b in zip(bounds, bounds[1:]):
        ops.gqa_prefill(q[a:b], k[a:b], v[a:b], gate[a:b], dev(x["qw"]), dev(x["kw"]), rope,
                        kc, vc, out[a:b], p0=a, cta_pairs=cta_pairs)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    return out.float().cpu().numpy(), kc, vc


@pytest.fixture(scope="module")
def rope(cuda):
    return ops.rope_table(40000)


@pytest.mark.parametrize("cta_pairs", [True, False])
@pytest.mark.parametrize("T", [1, 64, 200, 300])
def test_small_prompts_all_rows(cuda, orc, rope, T, cta_pairs):
    x = make(orc, 10 + T, T)
    out, _, _ = gpu_prefill(x, T, T + 64, rope, cta_pairs=cta_pairs)
    ref = oracle_rows(orc, x, T, range(T))
    assert rel_err(out.reshape(-1), ref.reshape(-1)) < REL_TOL


@pytest.mark.parametrize("cta_pairs", [True, False])
def test_chunked_continuation_equals_oracle(cuda, orc, rope, cta_pairs):
    """Prefill in three calls at p0 = 0, 130, 257 (cache carried between calls) == one pass."""
    T = 400
    x = make(orc, 99, T)
    out, kc, vc = gpu_prefill(x, T, 512, rope, chunks=[0, 130, 257, 400], cta_pairs=cta_pairs)
    ref = oracle_rows(orc, x, T, range(T))
    assert rel_err(out.reshape(-1), ref.reshape(-1)) < REL_TOL
    # the cache holds finite values past the prompt up to the next multiple of 64
    assert torch.isfinite(kc[:, :448].float()).all() and torch.isfinite(vc[:, :448].float()).all()


def test_config4_gqa_sampled_rows(cuda, orc, rope):
    """Config 4 GQA path: T = 32768, seed 4; rows first, last, tile edges and random."""
    T = 32768
    x = make(orc, 4, T)
    out, _, _ = gpu_prefill(x, T, T, rope, out_bf16=True)
    rows = [0, 1, 63, 64, 127, 128, 4095, 17001, T - 129, T - 1]
    ref = oracle_rows(orc, x, T, rows)
    err = rel_err(out[rows].reshape(-1), ref.reshape(-1))
    print(f"config4 GQA sampled rows rel err {err:.3e}")
    assert err < REL_TOL


@pytest.mark.parametrize("out_bf16", [False, True])
def test_fp32_activations_both_kernels(cuda, orc, rope, out_bf16):
    """fp32 q/k/v/gate (the staged fp32-gate epilogue), both attention kernels, all rows."""
    T = 333
    x = make(orc, 21, T, bf16=False)
    ref = oracle_rows(orc, x, T, range(T))
    outs = []
    for pairs in (True, False):
        out, _, _ = gpu_prefill(x, T, T + 64, rope, out_bf16=out_bf16, cta_pairs=pairs)
        assert rel_err(out.reshape(-1), ref.reshape(-1)) < REL_TOL
        outs.append(out)
    assert rel_err(outs[0].reshape(-1), outs[1].reshape(-1)) < 1e-2


@pytest.mark.parametrize("nq,nkv", [(12, 4), (8, 8), (16, 2)])
def test_group_sizes(cuda, orc, rope, nq, nkv):
    """Odd group sizes (3, 1) run one CTA per head; an even one (8) runs in pairs."""
    T = 260
    x = make(orc, 22, T, nq=nq, nkv=nkv)
    out, _, _ = gpu_prefill(x, T, T + 64, rope)
    ref = oracle_rows(orc, x, T, range(T))
    assert rel_err(out.reshape(-1), ref.reshape(-1)) < REL_TOL


def test_pairs_equal_single_sm_kernel(cuda, orc, rope):
    """The pair kernel's M = 256 MMAs compute the same products as the single-SM kernel's
    M = 128 ones over the same bf16 operands; over 2000 positions the two outputs agree
    to fp32 rounding of the accumulation order (reported), well inside the tolerance."""
    T = 2000
    x = make(orc, 23, T)
    a, _, _ = gpu_prefill(x, T, T, rope, cta_pairs=True)
    b, _, _ = gpu_prefill(x, T, T, rope, cta_pairs=False)
    err = rel_err(a.reshape(-1), b.reshape(-1))
    print(f"pair vs single-SM rel diff {err:.3e}, identical: {np.array_equal(a, b)}")
    assert err < 1e-4
    rows = [0, 127, 128, 1000, 1999]
    assert rel_err(a[rows].reshape(-1), oracle_rows(orc, x, T, rows).reshape(-1)) < REL_TOL


@pytest.mark.parametrize("p0", [0, 70])
def test_prefill_cache_rows_equal_append(cuda, orc, rope, p0):
    """The K/V rows the prefill writes (QK RMSNorm + RoPE at p0 + t, bf16) equal, bit for
    bit, the rows the oracle's per-token append writes (src/vx27_qfwd.c:339-346)."""
    T, cap = 150, 256
    x = make(orc, 24, T)
    q = dev(x["q"], True).view(T, NQ, HD)
    k = dev(x["k"], True).view(T, NKV, HD)
    v = dev(x["v"], True).view(T, NKV, HD)
    gate = dev(x["gate"], True).view(T, NQ, HD)
    kc = torch.zeros((NKV, cap, HD), dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    out = torch.empty(T, NQ, HD, device="cuda")
    ops.gqa_prefill(q, k, v, gate, dev(x["qw"]), dev(x["kw"]), rope, kc, vc, out, p0=p0)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    L, P = orc.lib(), orc.P
    kr = np.zeros(NKV * cap * HD, np.uint16)
    vr = np.zeros_like(kr)
    qo = np.zeros(NQ * HD, np.float32)
    for t in range(T):
        pos = np.array([p0 + t], np.int32)
        L.orc_gqa_append(P(x["q"][t * NQ * HD:]), P(x["k"][t * NKV * HD:]),
                         P(x["v"][t * NKV * HD:]), P(x["qw"]), P(x["kw"]), P(pos), P(kr), P(vr),
                         cap, P(qo), 1, NQ, NKV, HD, 64, 1e7, 1e-6, orc.F_ACT_BF16)
    kg = kc.view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1)
    vg = vc.view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1)
    rows = lambda a: a.reshape(NKV, cap, HD)[:, p0:p0 + T]
    assert np.array_equal(rows(kg), rows(kr)) and np.array_equal(rows(vg), rows(vr))
