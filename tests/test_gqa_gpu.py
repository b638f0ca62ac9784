"""K2 (vx27_gqa_append + vx27_gqa_decode_batch, partial/combine) against the CPU oracle.

Tolerances: the appended K/V rows and the normalised, rotated q match the reference
arithmetic (QK RMSNorm with a double sum, RoPE with the reference's table and rounding);
the attention output is within 2e-2 relative (max-abs error over max-abs value) of the
reference path with the same BF16 cache -- in practice it is ~1e-6."""
import numpy as np
import pytest
import torch

from gpu_util import dev, host, rel_err
from vx27_b200 import ops

pytestmark = pytest.mark.gpu
NQ, NKV, HD = 24, 4, 256
REL_TOL = 2e-2


def setup(orc, seed, B, cap, pos, bf16=True):
    g = lambda n, s, m=0.0, sd=1.0, b=bf16: orc.normal(n, seed, s, m, sd, bf16=b)
    return dict(kc=g(B * NKV * cap * HD, 1, b=True), vc=g(B * NKV * cap * HD, 2, b=True),
                qi=g(B * NQ * HD, 3), ki=g(B * NKV * HD, 4), vi=g(B * NKV * HD, 5),
                gate=g(B * NQ * HD, 6), qw=g(HD, 7, 1.0, 0.02, False),
                kw=g(HD, 8, 1.0, 0.02, False), pos=np.asarray(pos, np.int32))


def oracle_step(orc, x, B, cap, bf16=True):
    L, P = orc.lib(), orc.P
    kc, vc = x["kc"].copy(), x["vc"].copy()
    qo = np.zeros(B * NQ * HD, np.float32)
    flags = orc.F_ACT_BF16 if bf16 else 0
    L.orc_gqa_append(P(x["qi"]), P(x["ki"]), P(x["vi"]), P(x["qw"]), P(x["kw"]), P(x["pos"]),
                     P(kc), P(vc), cap, P(qo), B, NQ, NKV, HD, 64, 1e7, 1e-6, flags)
    out = np.zeros(B * NQ * HD, np.float32)
    L.orc_gqa_attend_mt(P(qo), P(x["gate"]), P(kc), P(vc), cap, P(x["pos"]), P(out), B, NQ, NKV,
                        HD, flags, 8)
    return qo, kc, vc, out


def gpu_step(x, B, cap, rope, n_splits=0, bf16=True, out_bf16=False, kernel="auto"):
    kc = dev(x["kc"], True).view(B, NKV, cap, HD)
    vc = dev(x["vc"], True).view(B, NKV, cap, HD)
    qi = dev(x["qi"], bf16).view(B, NQ, HD)
    ki = dev(x["ki"], bf16).view(B, NKV, HD)
    vi = dev(x["vi"], bf16).view(B, NKV, HD)
    gate = dev(x["gate"], bf16).view(B, NQ, HD)
    pos = dev(x["pos"])
    q = torch.empty(B, NQ, HD, device="cuda")
    ops.gqa_append(qi, ki, vi, dev(x["qw"]), dev(x["kw"]), rope, pos, kc, vc, q)
    ws = torch.empty(ops.gqa_workspace_bytes(B, NQ, NKV, HD, cap, n_splits) // 4 + 1,
                     device="cuda")
    out = torch.empty(B, NQ, HD, device="cuda",
                      dtype=torch.bfloat16 if out_bf16 else torch.float32)
    ops.gqa_decode_batch(q, gate, kc, vc, pos, out, ws, n_splits=n_splits, kernel=kernel)
    out = out.float()
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    return host(q).reshape(-1), host(kc).reshape(-1), host(vc).reshape(-1), host(out).reshape(-1)


def gpu_step_fused(x, B, cap, rope, n_splits=0, bf16=True, out_bf16=False, kernel="auto"):
    """vx27_gqa_decode_fused: append and attention in one kernel."""
    kc = dev(x["kc"], True).view(B, NKV, cap, HD)
    vc = dev(x["vc"], True).view(B, NKV, cap, HD)
    qi = dev(x["qi"], bf16).view(B, NQ, HD)
    ki = dev(x["ki"], bf16).view(B, NKV, HD)
    vi = dev(x["vi"], bf16).view(B, NKV, HD)
    gate = dev(x["gate"], bf16).view(B, NQ, HD)
    pos = dev(x["pos"])
    ws = torch.empty(ops.gqa_workspace_bytes(B, NQ, NKV, HD, cap, n_splits) // 4 + 1,
                     device="cuda")
    out = torch.empty(B, NQ, HD, device="cuda",
                      dtype=torch.bfloat16 if out_bf16 else torch.float32)
    ops.gqa_decode_fused(qi, ki, vi, dev(x["qw"]), dev(x["kw"]), rope, gate, kc, vc, pos, out, ws,
                         n_splits=n_splits, kernel=kernel)
    out = out.float()
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    return host(kc).reshape(-1), host(vc).reshape(-1), host(out).reshape(-1)


@pytest.fixture(scope="module")
def rope(cuda):
    return ops.rope_table(300000)


def test_rope_table_matches_reference(cuda, golden, rope):
    r = host(rope)
    for n, p in enumerate(golden["rope_pos"]):
        if golden["rope_yarn"][n] != 1 or p >= r.shape[0]:
            continue
        assert np.array_equal(r[p, :32], golden["rope_cos"][n])
        assert np.array_equal(r[p, 32:], golden["rope_sin"][n])


def test_golden_driver_inputs(cuda, orc, golden, rope):
    """Same inputs as the reference-generated golden fixture (B=2, pos 10 and 37)."""
    B, cap = 2, 48
    x = setup(orc, 8, B, cap, golden["gq_pos"])
    q, kc, vc, out = gpu_step(x, B, cap, rope)
    assert np.abs(q - golden["gq_qo"]).max() <= 1e-6 * np.abs(golden["gq_qo"]).max()
    krow = kc.reshape(B, NKV, cap, HD)[np.arange(B), :, golden["gq_pos"]]
    mism = np.count_nonzero(krow != golden["gq_krow"])
    assert mism <= krow.size // 1000  # a 1-ulp difference in q/k norm may flip a bf16 rounding
    vrow = vc.reshape(B, NKV, cap, HD)[np.arange(B), :, golden["gq_pos"]]
    assert np.array_equal(vrow, golden["gq_vrow"])
    assert rel_err(out, golden["gq_out"]) < 1e-4


@pytest.mark.parametrize("n_splits", [0, 1, 3, 7])
@pytest.mark.parametrize("kernel", ["tc", "cc"])
def test_ragged_batch(cuda, orc, rope, n_splits, kernel):
    """Sequences at positions 0 (a single key), 1, 127, 128 (tile edges) and 1000."""
    B, cap = 5, 1024
    x = setup(orc, 21, B, cap, [0, 1, 127, 128, 1000])
    qo, kc, vc, ref = oracle_step(orc, x, B, cap)
    q, kcg, vcg, out = gpu_step(x, B, cap, rope, n_splits, kernel=kernel)
    assert rel_err(q, qo) < 1e-6
    assert rel_err(out, ref) < 1e-4 < REL_TOL
    print(f"splits={n_splits}: rel err {rel_err(out, ref):.2e}")


@pytest.mark.parametrize("kernel", ["tc", "cc"])
def test_config1_ctx8192(cuda, orc, rope, kernel):
    """Config 1: batch 1, ctx 8192 (cache 0..8190 ~N(0,1) bf16, token at 8191), seed 1."""
    B, cap = 1, 8192
    x = setup(orc, 1, B, cap, [8191])
    qo, kc, vc, ref = oracle_step(orc, x, B, cap)
    q, kcg, vcg, out = gpu_step(x, B, cap, rope, kernel=kernel)
    err = rel_err(out, ref)
    print(f"config1 rel err {err:.3e}")
    assert err < REL_TOL and err < 1e-4


@pytest.mark.parametrize("n_splits", [0, 1])
@pytest.mark.parametrize("kernel", ["tc", "cc"])
def test_fp32_activations(cuda, orc, rope, n_splits, kernel):
    # n_splits = 1: the split kernel applies the fp32 gate and writes the output itself
    B, cap = 2, 300
    x = setup(orc, 31, B, cap, [5, 299], bf16=False)
    qo, kc, vc, ref = oracle_step(orc, x, B, cap, bf16=False)
    q, _, _, out = gpu_step(x, B, cap, rope, n_splits, bf16=False, kernel=kernel)
    assert rel_err(out, ref) < 1e-4


@pytest.mark.parametrize("n_splits", [1, 4])
@pytest.mark.parametrize("kernel", ["tc", "cc"])
def test_bf16_output(cuda, orc, rope, n_splits, kernel):
    # bf16 gate and bf16 output, written by the split kernel (1) or by the combine (4)
    B, cap = 3, 700
    x = setup(orc, 37, B, cap, [0, 300, 699])
    qo, kc, vc, ref = oracle_step(orc, x, B, cap)
    q, _, _, out = gpu_step(x, B, cap, rope, n_splits, out_bf16=True, kernel=kernel)
    err = rel_err(out, ref)
    print(f"splits={n_splits}: bf16 output rel err {err:.2e}")
    assert err < 2e-2


def test_partial_combine_context_parallel(cuda, orc, rope):
    """Four shards of one 4096-position sequence, each a partial over its slice, merged by
    vx27_gqa_combine == single-pass decode (the config 3b data flow on one GPU)."""
    B, cap = 1, 4096
    x = setup(orc, 41, B, cap, [cap - 1])
    _, _, _, full = gpu_step(x, B, cap, rope)
    kc = dev(x["kc"], True).view(B, NKV, cap, HD)
    vc = dev(x["vc"], True).view(B, NKV, cap, HD)
    q = torch.empty(B, NQ, HD, device="cuda")
    ops.gqa_append(dev(x["qi"], True).view(B, NQ, HD), dev(x["ki"], True).view(B, NKV, HD),
                   dev(x["vi"], True).view(B, NKV, HD), dev(x["qw"]), dev(x["kw"]), rope,
                   dev(x["pos"]), kc, vc, q)
    n = 4
    rec = B * NQ * (HD + 2)
    ws = torch.empty(ops.gqa_partial_workspace_bytes(B, NQ, NKV, HD, cap) // 4 + 1, device="cuda")
    for workspace in (None, ws):  # one CTA per KV head, or split across CTAs and merged
        parts = torch.empty(n * rec, device="cuda")
        for r in range(n):
            ops.gqa_partial(q, kc, vc, r * cap // n, (r + 1) * cap // n,
                            parts[r * rec:(r + 1) * rec], workspace)
        out = torch.empty(B, NQ, HD, device="cuda")
        ops.gqa_combine(parts, n, dev(x["gate"], True).view(B, NQ, HD), out)
        torch.cuda.synchronize()
        assert rel_err(host(out).reshape(-1), full) < 1e-5


@pytest.mark.parametrize("gated,out_bf16", [(True, False), (False, False), (True, True)])
def test_combine_short_and_long_forms_agree(cuda, gated, out_bf16):
    """vx27_gqa_combine merges up to 32 records in one pass (one L2 round trip) and more in
    blocks; both forms sum in record order. 40 records whose last 8 are empty (l = 0, which
    the merge skips) go through the long form and must give the short form's bits for the
    first 32; both match the merge formula in fp64. Record 5 is empty too, and one sequence
    has no valid record at all (its output is 0)."""
    B, n, n_long = 2, 32, 40
    rec = B * NQ * (HD + 2)
    g = torch.Generator().manual_seed(17)
    o = torch.randn(n_long, B * NQ * HD, generator=g)
    m = torch.randn(n_long, B * NQ, generator=g) * 4.0
    l = torch.rand(n_long, B * NQ, generator=g) * 50.0 + 0.5
    l[5] = 0.0
    m[5] = -float("inf")
    l[n:] = 0.0
    m[n:] = -float("inf")
    l[:, NQ:] = 0.0  # sequence 1: every record empty
    m[:, NQ:] = -float("inf")
    parts = torch.cat([o, torch.stack([m, l], -1).reshape(n_long, -1)], 1).reshape(-1).cuda()
    gate = torch.randn(B, NQ, HD, generator=g) if gated else None
    odt = torch.bfloat16 if out_bf16 else torch.float32
    outs = []
    for k in (n, n_long):
        out = torch.empty(B, NQ, HD, device="cuda", dtype=odt)
        ops.gqa_combine(parts[:k * rec], k, None if gate is None else gate.cuda(), out)
        outs.append(out.float().cpu())
    assert torch.equal(outs[0], outs[1])
    # fp64 restatement of the merge
    md, ld, od = m[:n].double(), l[:n].double(), o[:n].double().view(n, B * NQ, HD)
    M = torch.where(ld > 0, md, torch.full_like(md, -float("inf"))).amax(0)
    w = torch.where(ld > 0, ld * torch.exp(md - M), torch.zeros_like(ld))
    L = w.sum(0)
    att = torch.where(L[:, None] > 0, (w[:, :, None] * od).sum(0) / L[:, None].clamp_min(1e-300),
                      torch.zeros(B * NQ, HD, dtype=torch.float64)).view(B, NQ, HD)
    if gate is not None:
        att = att * torch.sigmoid(gate.double())
    assert torch.all(outs[0][1] == 0)
    tol = 1e-2 if out_bf16 else 1e-5
    assert rel_err(outs[0].reshape(-1).numpy(), att.reshape(-1).numpy()) < tol


def test_append_q_only_and_foreign_slot(cuda, orc, rope):
    """k_cache=NULL computes q only; a slot outside the shard leaves the cache untouched."""
    B, cap = 1, 64
    x = setup(orc, 51, B, cap, [100])
    kc = dev(x["kc"], True).view(B, NKV, cap, HD)
    vc = dev(x["vc"], True).view(B, NKV, cap, HD)
    before = host(kc).copy()
    q = torch.empty(B, NQ, HD, device="cuda")
    ops.gqa_append(dev(x["qi"], True).view(B, NQ, HD), dev(x["ki"], True).view(B, NKV, HD),
                   dev(x["vi"], True).view(B, NKV, HD), dev(x["qw"]), dev(x["kw"]), rope,
                   dev(x["pos"]), kc, vc, q, slot_base=0)
    torch.cuda.synchronize()
    assert np.array_equal(host(kc), before)
    q2 = torch.empty(B, NQ, HD, device="cuda")
    ops.gqa_append(dev(x["qi"], True).view(B, NQ, HD), dev(x["ki"], True).view(B, NKV, HD),
                   dev(x["vi"], True).view(B, NKV, HD), dev(x["qw"]), dev(x["kw"]), rope,
                   dev(x["pos"]), None, None, q2)
    torch.cuda.synchronize()
    assert torch.equal(q, q2)


def test_kv_cache_object_roundtrip(cuda, orc):
    import ctypes as C
    from vx27_b200._lib import errbuf, load
    lib = load()
    e = errbuf()
    h = C.c_void_p()
    assert lib.vx27_kv_create(C.byref(h), 2, 3, NKV, HD, 64, e, 512) == 0, e.value
    try:
        k = orc.normal(10 * NKV * HD, 61, 1)
        v = orc.normal(10 * NKV * HD, 61, 2)
        assert lib.vx27_kv_store_f32(h, 1, 2, 5, 10, orc.P(k), orc.P(v), e, 512) == 0
        k2, v2 = np.zeros_like(k), np.zeros_like(v)
        assert lib.vx27_kv_load_f32(h, 1, 2, 5, 10, orc.P(k2), orc.P(v2), e, 512) == 0
        assert np.array_equal(k2, orc.from_bf16(orc.to_bf16(k)))
        assert np.array_equal(v2, orc.from_bf16(orc.to_bf16(v)))
        assert lib.vx27_kv_store_f32(h, 1, 2, 60, 10, orc.P(k), orc.P(v), e, 512) == -1
    finally:
        lib.vx27_kv_destroy(h)


def test_no_output_gate_mtp_drafter(cuda, orc, rope):
    """gate = NULL: the attention without the sigmoid gate, as the MTP drafter runs it with
    use_gate = 0 (src/vx27_mtp.c:232-250) over its own cache; two sequences, one split."""
    B, cap = 2, 700
    x = setup(orc, 61, B, cap, [333, 699])
    L, P = orc.lib(), orc.P
    kc, vc = x["kc"].copy(), x["vc"].copy()
    qo = np.zeros(B * NQ * HD, np.float32)
    L.orc_gqa_append(P(x["qi"]), P(x["ki"]), P(x["vi"]), P(x["qw"]), P(x["kw"]), P(x["pos"]),
                     P(kc), P(vc), cap, P(qo), B, NQ, NKV, HD, 64, 1e7, 1e-6, orc.F_ACT_BF16)
    ref = np.zeros(B * NQ * HD, np.float32)
    L.orc_gqa_attend_mt(P(qo), None, P(kc), P(vc), cap, P(x["pos"]), P(ref), B, NQ, NKV, HD,
                        orc.F_ACT_BF16, 8)
    dkc = dev(x["kc"], True).view(B, NKV, cap, HD)
    dvc = dev(x["vc"], True).view(B, NKV, cap, HD)
    q = torch.empty(B, NQ, HD, device="cuda")
    pos = dev(x["pos"])
    ops.gqa_append(dev(x["qi"], True).view(B, NQ, HD), dev(x["ki"], True).view(B, NKV, HD),
                   dev(x["vi"], True).view(B, NKV, HD), dev(x["qw"]), dev(x["kw"]), rope, pos,
                   dkc, dvc, q)
    ws = torch.empty(ops.gqa_workspace_bytes(B, NQ, NKV, HD, cap, 1) // 4 + 1, device="cuda")
    out = torch.empty(B, NQ, HD, device="cuda")
    ops.gqa_decode_batch(q, None, dkc, dvc, pos, out, ws, n_splits=1)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    assert rel_err(host(out).reshape(-1), ref) < REL_TOL


@pytest.mark.parametrize("n_splits", [0, 1, 3, 7])
@pytest.mark.parametrize("kernel", ["tc", "cc"])
def test_fused_decode_ragged_batch(cuda, orc, rope, n_splits, kernel):
    """The fused kernel (vx27_gqa_decode_fused) on the ragged batch: the appended rows equal
    the separate append kernel's bit for bit, the output the oracle's."""
    B, cap = 5, 1024
    x = setup(orc, 21, B, cap, [0, 1, 127, 128, 1000])
    qo, kc, vc, ref = oracle_step(orc, x, B, cap)
    _, kc_sep, vc_sep, out_sep = gpu_step(x, B, cap, rope, n_splits)
    kcg, vcg, out = gpu_step_fused(x, B, cap, rope, n_splits, kernel=kernel)
    assert np.array_equal(vcg, vc_sep) and np.array_equal(vcg, vc)
    krow_f = kcg.reshape(B, NKV, cap, HD)[np.arange(B), :, x["pos"]]
    krow_s = kc_sep.reshape(B, NKV, cap, HD)[np.arange(B), :, x["pos"]]
    # the norm's double sum runs in another order: a 1-ulp difference may flip a bf16 rounding
    assert np.count_nonzero(krow_f != krow_s) <= krow_f.size // 1000
    # every other cache row is untouched
    keep = np.ones((B, NKV, cap), bool)
    keep[np.arange(B), :, x["pos"]] = False
    assert np.array_equal(kcg.reshape(B, NKV, cap, HD)[keep], x["kc"].reshape(B, NKV, cap, HD)[keep])
    err = rel_err(out, ref)
    print(f"fused splits={n_splits}: rel err {err:.2e} (separate kernels {rel_err(out_sep, ref):.2e})")
    assert err < 1e-4 < REL_TOL


@pytest.mark.parametrize("kernel", ["tc", "cc"])
def test_fused_decode_golden_and_config1(cuda, orc, golden, rope, kernel):
    """Golden driver inputs (pos 10 and 37) and config 1 (ctx 8192) through the fused kernel."""
    B, cap = 2, 48
    x = setup(orc, 8, B, cap, golden["gq_pos"])
    kc, vc, out = gpu_step_fused(x, B, cap, rope, kernel=kernel)
    krow = kc.reshape(B, NKV, cap, HD)[np.arange(B), :, golden["gq_pos"]]
    assert np.count_nonzero(krow != golden["gq_krow"]) <= krow.size // 1000
    vrow = vc.reshape(B, NKV, cap, HD)[np.arange(B), :, golden["gq_pos"]]
    assert np.array_equal(vrow, golden["gq_vrow"])
    assert rel_err(out, golden["gq_out"]) < 1e-4
    B, cap = 1, 8192
    x = setup(orc, 1, B, cap, [8191])
    _, _, _, ref = oracle_step(orc, x, B, cap)
    _, _, out = gpu_step_fused(x, B, cap, rope, kernel=kernel)
    assert rel_err(out, ref) < 1e-4


@pytest.mark.parametrize("bf16,out_bf16", [(False, False), (True, True)])
@pytest.mark.parametrize("kernel", ["tc", "cc"])
def test_fused_decode_dtypes(cuda, orc, rope, bf16, out_bf16, kernel):
    B, cap = 3, 700
    x = setup(orc, 37, B, cap, [0, 300, 699], bf16=bf16)
    _, _, _, ref = oracle_step(orc, x, B, cap, bf16=bf16)
    _, _, out = gpu_step_fused(x, B, cap, rope, 1, bf16=bf16, out_bf16=out_bf16, kernel=kernel)
    assert rel_err(out, ref) < (2e-2 if out_bf16 else 1e-4)
