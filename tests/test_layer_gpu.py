"""Whole-layer decode steps (vx27_b200/layer.py: projections K5 around K1 / K2) against the
reference's single-token layer forward restated from the oracle's pieces
(src/vx27_qfwd.c:95-154 DeltaNet, :156-214 GQA): the packed matvec (bit-identical to
vx27_pmat), conv1d_step, the zero-centred RMSNorm -> l2norm -> 1/sqrt(hd) q/k
pre-normalisation, gate_params, step_exact per V head, the gated RMSNorm output; RMSNorm
(1+w) + RoPE + BF16 KV append and the attention with the sigmoid gate. Model shapes:
H = 5120, DeltaNet 16 QK / 48 V heads of 128, GQA 24 / 4 heads of 256, BP3_128 weights."""
import numpy as np
import pytest
import torch

import oracle.oracle as O
from vx27_b200 import ops
from vx27_b200.layer import DeltaNetLayer, GQALayer, PackedLinear

pytestmark = pytest.mark.gpu
H = 5120


def packed(rows, cols, seed):
    W = O.packed_weights(O.PMAT_BP3, rows, cols, seed)
    return W, PackedLinear(torch.from_numpy(W).cuda(), O.PMAT_BP3, rows, cols)


def test_deltanet_layer_steps(cuda):
    L, P = O.lib(), O.P
    nqk, nv, hd, B, steps = 16, 48, 128, 2, 3
    qd, C = nqk * hd, (2 * nqk + nv) * hd
    rng = np.random.default_rng(11)
    Wqkv, pqkv = packed(C, H, 1)
    Wz, pz = packed(nv * hd, H, 2)
    Wa, pa = packed(nv, H, 3)
    Wb, pb = packed(nv, H, 4)
    Wo, po = packed(H, nv * hd, 5)
    A_log = np.log(rng.uniform(1, 16, nv)).astype(np.float32)
    dt_bias = (rng.standard_normal(nv) * 0.1).astype(np.float32)
    conv_w = (rng.standard_normal((C, 4)) * 0.5).astype(np.float32)
    norm_w = (1 + rng.standard_normal(hd) * 0.02).astype(np.float32)
    layer = DeltaNetLayer(pqkv, pz, pa, pb, po, torch.from_numpy(A_log).cuda(),
                          torch.from_numpy(dt_bias).cuda(), torch.from_numpy(conv_w).cuda(),
                          torch.from_numpy(norm_w).cuda(), nqk, nv, hd)
    S = torch.zeros(B, nv, hd, hd, device="cuda")
    ring = torch.zeros(B, 4, C, device="cuda")
    S_ref = np.zeros((B, nv, hd, hd), np.float32)
    conv_ref = np.zeros((B, C * 3), np.float32)
    qs = np.float32(1.0) / np.sqrt(np.float32(hd))
    for t in range(steps):
        x = rng.standard_normal((B, H)).astype(np.float32)
        pos = torch.full((B,), t, dtype=torch.int32, device="cuda")
        ao = layer.step(torch.from_numpy(x).cuda(), S, ring, pos).cpu().numpy()
        ao_ref = np.zeros((B, H), np.float32)
        for b in range(B):
            xb = x[b].copy()
            qkv = O.pmat_batch(Wqkv, O.PMAT_BP3, xb, C, H, 1)
            z = O.pmat_batch(Wz, O.PMAT_BP3, xb, nv * hd, H, 1)
            a = O.pmat_batch(Wa, O.PMAT_BP3, xb, nv, H, 1)
            bb = O.pmat_batch(Wb, O.PMAT_BP3, xb, nv, H, 1)
            y = np.zeros(C, np.float32)
            st = conv_ref[b].copy()
            L.orc_conv1d_step(P(st), P(qkv), P(conv_w), P(y), C, 1)
            conv_ref[b] = st
            q, k, v = y[:qd].copy(), y[qd:2 * qd].copy(), y[2 * qd:].copy()
            for hh in range(nqk):
                for arr in (q, k):
                    t_ = np.zeros(hd, np.float32)
                    L.orc_rmsnorm(P(arr[hh * hd:(hh + 1) * hd].copy()), P(norm_w), P(t_), hd,
                                  1e-6, 1)
                    out_ = np.zeros(hd, np.float32)
                    L.orc_l2norm(P(t_), P(out_), hd)
                    arr[hh * hd:(hh + 1) * hd] = out_
            q = (q * qs).astype(np.float32)
            ret = np.zeros(nv * hd, np.float32)
            for vh in range(nv):
                beta, g = O.C.c_double(), O.C.c_double()
                L.orc_gate_params(float(a[vh]), float(A_log[vh]), float(bb[vh]),
                                  float(dt_bias[vh]), O.C.byref(beta), O.C.byref(g))
                qk = vh * nqk // nv
                Sv = S_ref[b, vh].copy()
                rv = np.zeros(hd, np.float32)
                L.orc_step_exact(P(Sv), P(q[qk * hd:(qk + 1) * hd].copy()),
                                 P(k[qk * hd:(qk + 1) * hd].copy()),
                                 P(v[vh * hd:(vh + 1) * hd].copy()), beta.value, g.value, P(rv), hd)
                S_ref[b, vh] = Sv
                ret[vh * hd:(vh + 1) * hd] = rv
            o = np.zeros(nv * hd, np.float32)
            L.orc_gated_rmsnorm(P(ret), P(norm_w), P(z), P(o), nv, hd)
            ao_ref[b] = O.pmat_batch(Wo, O.PMAT_BP3, o, H, nv * hd, 1)
        s_err = float(np.abs(S.cpu().numpy() - S_ref).max())
        a_err = float(np.abs(ao - ao_ref).max() / np.abs(ao_ref).max())
        print(f"step {t}: max|S-ref| {s_err:.2e}, layer output rel err {a_err:.2e}")
        assert s_err < 1e-4
        assert a_err < 1e-4
    assert ops.device_status() == 0


def test_gqa_layer_step(cuda):
    L, P = O.lib(), O.P
    nq, nkv, hd, B, cap = 24, 4, 256, 2, 96
    rng = np.random.default_rng(12)
    Wq, pq = packed(nq * 2 * hd, H, 21)
    Wk, pk = packed(nkv * hd, H, 22)
    Wv, pv = packed(nkv * hd, H, 23)
    Wo, po = packed(H, nq * hd, 24)
    qw = (rng.standard_normal(hd) * 0.02).astype(np.float32)
    kw = (rng.standard_normal(hd) * 0.02).astype(np.float32)
    pos = np.array([7, 90], np.int32)
    kc = O.normal(B * nkv * cap * hd, 12, 1, bf16=True)
    vc = O.normal(B * nkv * cap * hd, 12, 2, bf16=True)
    x = rng.standard_normal((B, H)).astype(np.float32)
    layer = GQALayer(pq, pk, pv, po, torch.from_numpy(qw).cuda(), torch.from_numpy(kw).cuda(),
                     ops.rope_table(cap), nq, nkv, hd)
    kcd = torch.from_numpy(kc.view(np.int16)).cuda().view(torch.bfloat16).view(B, nkv, cap, hd)
    vcd = torch.from_numpy(vc.view(np.int16)).cuda().view(torch.bfloat16).view(B, nkv, cap, hd)
    ws = torch.empty(ops.gqa_workspace_bytes(B, nq, nkv, hd, cap) // 4 + 1, device="cuda")
    ao = layer.step(torch.from_numpy(x).cuda(), kcd, vcd, torch.from_numpy(pos).cuda(),
                    ws).cpu().numpy()
    # the reference: projections, q/gate split per head, RMSNorm(1+w) + RoPE + append, attention
    qg = O.pmat_batch(Wq, O.PMAT_BP3, x.reshape(-1), nq * 2 * hd, H, B).reshape(B, nq, 2, hd)
    qi = np.ascontiguousarray(qg[:, :, 0]).reshape(-1)
    gate = np.ascontiguousarray(qg[:, :, 1]).reshape(-1)
    ki = O.pmat_batch(Wk, O.PMAT_BP3, x.reshape(-1), nkv * hd, H, B)
    vi = O.pmat_batch(Wv, O.PMAT_BP3, x.reshape(-1), nkv * hd, H, B)
    kr, vr = kc.copy(), vc.copy()
    qo = np.zeros(B * nq * hd, np.float32)
    L.orc_gqa_append(P(qi), P(ki), P(vi), P(qw), P(kw), P(pos), P(kr), P(vr), cap, P(qo), B, nq,
                     nkv, hd, 64, 1e7, 1e-6, O.F_NORM_1P)
    att = np.zeros(B * nq * hd, np.float32)
    L.orc_gqa_attend(P(qo), P(gate), P(kr), P(vr), cap, P(pos), P(att), B, nq, nkv, hd, 0)
    ao_ref = O.pmat_batch(Wo, O.PMAT_BP3, att, H, nq * hd, B).reshape(B, H)
    err = float(np.abs(ao - ao_ref).max() / np.abs(ao_ref).max())
    print(f"GQA layer output rel err {err:.2e}")
    assert err < 2e-3
    # the appended K/V rows equal the reference's (bf16 bits)
    kd = kcd.view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1)
    for b in range(B):
        for h in range(nkv):
            o0 = ((b * nkv + h) * cap + pos[b]) * hd
            assert np.array_equal(kd[o0:o0 + hd], kr[o0:o0 + hd])
    assert ops.device_status() == 0
