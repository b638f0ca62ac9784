"""The decode drivers at the configurations BASELINE.json names, against the CPU oracle.

* Config 3 at its stated context: 262144 cache positions, the query token at position
  262143 (16 layers in the benchmark; one layer here, since the layers are independent).
  - 3a, sequence-sharded: two sequences, whole caches on one GPU.
  - 3b, KV-split: one sequence whose cache is split into N = 2, 4 and 8 shards; each
    shard's partial record (vx27_gqa_partial) is merged by vx27_gqa_combine, as the
    ranks of a multi-GPU run do after their all-gather.
  Oracle: the reference's decode attention (src/vx27_qfwd.c:186-211, batch form
  :347-371) restated over the same bf16 cache (orc_gqa_append + orc_gqa_attend_mt).
* Config 2 at its full shape: B = 256 sequences with 4096 cached tokens through all 64
  layers; sequences 0, 1, 128 and 255 of DeltaNet layers 0 and 47 and GQA layers 0 and 15
  are checked against the oracle's batched decode (src/vx27_qfwd.c:276-297 and :339-371
  per sequence), so a wrong item index or stride in the persistent kernels' walk over
  256 x 16 or 256 x 4 x splits items would show.
Tolerances: DeltaNet output/state 1e-4 (bf16 outputs: plus their rounding); GQA 2e-2
relative (bf16 outputs: their rounding, ~4e-3, dominates the kernel's ~1e-6)."""
import os

import numpy as np
import pytest
import torch

from gpu_util import host, rel_err
from vx27_b200.hybrid import HybridConfig, HybridDecoder, N_FULL, N_LIN
from vx27_b200.longctx import HD, NKV, NQ, LongContextGQA

pytestmark = pytest.mark.gpu
CTX3 = 262144
THREADS = max(1, min(32, os.cpu_count() or 1))


def _bits(t):
    return np.ascontiguousarray(host(t).view(np.uint16).reshape(-1))


def _f32(t):
    return np.ascontiguousarray(host(t).astype(np.float32).reshape(-1))


def _oracle_gqa(orc, q_in, k_in, v_in, qw, kw, gate, kc, vc, cap, pos):
    """Append + attention of the oracle for B sequences (all host arrays; kc/vc updated)."""
    L, P = orc.lib(), orc.P
    B = pos.shape[0]
    qo = np.zeros(B * NQ * HD, np.float32)
    L.orc_gqa_append(P(q_in), P(k_in), P(v_in), P(qw), P(kw), P(pos), P(kc), P(vc), cap, P(qo),
                     B, NQ, NKV, HD, 64, 1e7, 1e-6, orc.F_ACT_BF16)
    out = np.zeros(B * NQ * HD, np.float32)
    L.orc_gqa_attend_mt(P(qo), P(gate), P(kc), P(vc), cap, P(pos), P(out), B, NQ, NKV, HD,
                        orc.F_ACT_BF16, THREADS)
    return qo, out


def _bf16_close(got, ref, what):
    """got is a bf16 rounding of a value within 1e-4 (relative to max |ref|) of ref."""
    bound = np.abs(ref) * 2.0 ** -8 + 1e-4 * np.abs(ref).max()
    bad = np.count_nonzero(np.abs(got.astype(np.float64) - ref) > bound)
    assert bad == 0, f"{what}: {bad} elements beyond bf16 rounding + 1e-4"
    assert rel_err(got, ref) < 2e-2


@pytest.fixture(scope="module")
def config3(cuda, orc):
    """Config 3a on one GPU (two sequences, whole caches) and the oracle's result."""
    B = 2
    a = LongContextGQA(B, ctx=CTX3, layers=1)
    kc, vc = _bits(a.kc[0]), _bits(a.vc[0])  # before the step appends position 262143
    ins = [_bits(t[0]) for t in (a.q_in, a.k_in, a.v_in, a.gate)]
    qw, kw = _f32(a.q_norm_w[0]), _f32(a.k_norm_w[0])
    a.step()
    torch.cuda.synchronize()
    pos = np.full(B, CTX3 - 1, np.int32)
    qo, ref = _oracle_gqa(orc, ins[0], ins[1], ins[2], qw, kw, ins[3], kc, vc, CTX3, pos)
    res = dict(out=host(a.out[0].float()).reshape(-1), qn=host(a.qn[0]).reshape(-1), qo=qo,
               ref=ref, krow_gpu=_bits(a.kc[0, :, :, CTX3 - 1]),
               vrow_gpu=_bits(a.vc[0, :, :, CTX3 - 1]),
               krow=kc.reshape(B, NKV, CTX3, HD)[:, :, CTX3 - 1].reshape(-1),
               vrow=vc.reshape(B, NKV, CTX3, HD)[:, :, CTX3 - 1].reshape(-1))
    del a
    torch.cuda.empty_cache()
    return res


def test_config3a_whole_cache_ctx262144(config3):
    r = config3
    assert rel_err(r["qn"], r["qo"]) < 1e-6
    assert np.array_equal(r["vrow_gpu"], r["vrow"])
    # a 1-ulp difference in the norm's double sum may flip a bf16 rounding of k
    assert np.count_nonzero(r["krow_gpu"] != r["krow"]) <= r["krow"].size // 1000
    _bf16_close(r["out"], r["ref"], "config 3a")


@pytest.mark.parametrize("world", [2, 4, 8])
def test_config3b_kv_split_ctx262144(config3, world):
    shards = [LongContextGQA(1, ctx=CTX3, layers=1, rank=r, world=world, split_kv=True)
              for r in range(world)]
    for s in shards:
        s.local_partials()
    gathered = torch.stack([s.parts.reshape(-1) for s in shards])
    shards[0].combine(gathered)
    torch.cuda.synchronize()
    out = host(shards[0].out[0].float()).reshape(-1)
    ref = config3["ref"][:NQ * HD]  # sequence 0 of the whole-cache run
    _bf16_close(out, ref, f"config 3b, {world} shards")
    # only the shard owning position 262143 stored the new token's K/V row
    assert np.array_equal(_bits(shards[-1].vc[0, 0, :, shards[-1].cap - 1]),
                          config3["vrow"][:NKV * HD])


def test_config2_full_shape_sampled_sequences(cuda, orc):
    cfg = HybridConfig(batch=256, ctx=4096, steps=1, seed=2)
    dec = HybridDecoder(cfg)
    seqs = np.array([0, 1, 128, 255])
    ns = len(seqs)
    idx = torch.from_numpy(seqs).to(dec.dev)
    dn_layers, gqa_layers = [0, N_LIN - 1], [0, N_FULL - 1]
    pre = {}
    for i in dn_layers:
        pre["dn", i] = dict(S=_f32(dec.S[i][idx]), ring=_f32(dec.ring[i][idx]),
                            qkv=_bits(dec.qkv[i][idx]), a=_bits(dec.a[i][idx]),
                            b=_bits(dec.b[i][idx]), A_log=_f32(dec.A_log[i]),
                            dt=_f32(dec.dt_bias[i]), w=_f32(dec.conv_w[i]))
    for i in gqa_layers:
        pre["gqa", i] = dict(kc=_bits(dec.kc[i][idx]), vc=_bits(dec.vc[i][idx]),
                             q_in=_bits(dec.q_in[i][idx]), k_in=_bits(dec.k_in[i][idx]),
                             v_in=_bits(dec.v_in[i][idx]), gate=_bits(dec.gate[i][idx]),
                             qw=_f32(dec.q_norm_w[i]), kw=_f32(dec.k_norm_w[i]))
    dec.step()
    torch.cuda.synchronize()
    P, L = orc.P, orc.lib()
    pos = np.full(ns, cfg.ctx, np.int32)
    for i in dn_layers:
        x = pre["dn", i]
        o = np.zeros(ns * cfg.nv * 128, np.float32)
        L.orc_deltanet_decode_batch_mt(P(x["S"]), P(x["ring"]), P(x["qkv"]), P(x["a"]),
                                       P(x["b"]), P(x["A_log"]), P(x["dt"]), P(x["w"]), P(pos),
                                       P(o), ns, cfg.nqk, cfg.nv, 128, orc.F_ACT_BF16, THREADS)
        got = host(dec.dn_out[i][idx].float()).reshape(-1)
        assert np.all(np.abs(got - o) <= np.abs(o) * 2.0 ** -8 + 1e-4), f"DeltaNet layer {i}"
        assert np.abs(_f32(dec.S[i][idx]) - x["S"]).max() < 1e-4, f"DeltaNet layer {i} state"
    for i in gqa_layers:
        x = pre["gqa", i]
        _, ref = _oracle_gqa(orc, x["q_in"], x["k_in"], x["v_in"], x["qw"], x["kw"], x["gate"],
                             x["kc"], x["vc"], cfg.cap, pos)
        got = host(dec.att_out[i][idx].float()).reshape(-1)
        _bf16_close(got, ref, f"GQA layer {i}")
        assert np.array_equal(_bits(dec.vc[i][idx][:, :, cfg.ctx]),
                              x["vc"].reshape(ns, NKV, cfg.cap, HD)[:, :, cfg.ctx].reshape(-1))
    del dec
    torch.cuda.empty_cache()
