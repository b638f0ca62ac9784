"""K1 (vx27_deltanet_decode_batch) against the CPU oracle on the same seeded inputs.

Tolerance: DeltaNet output and state within 1e-4 max-abs of the reference path
(conv1d_step -> gate_params -> step_exact per head, src/vx27_qfwd.c:276-297)."""
import numpy as np
import pytest
import torch

from gpu_util import dev, host
from vx27_b200 import ops

pytestmark = pytest.mark.gpu
TOL = 1e-4


def make_layer(orc, seed, B, nqk, nv, hd=128, s_std=0.0):
    Cch = (2 * nqk + nv) * hd
    S = (orc.normal(B * nv * hd * hd, seed, 10, 0.0, s_std) if s_std > 0
         else np.zeros(B * nv * hd * hd, np.float32))
    return dict(S=S, ring=np.zeros(B * 4 * Cch, np.float32),
                conv_w=orc.normal(Cch * 4, seed, 4, 0.0, 0.5),
                A_log=np.log(orc.uniform(nv, seed, 5, 1.0, 16.0)).astype(np.float32),
                dt_bias=orc.normal(nv, seed, 6, 0.0, 0.1), C=Cch)


def run_both(orc, lay, T, B, nqk, nv, seed, bf16, pos0=None, gates_f64=False, out_bf16=False):
    hd = 128
    Cch = lay["C"]
    qkv_all = orc.normal(T * B * Cch, seed, 1, bf16=bf16).reshape(T, B * Cch)
    a_all = orc.normal(T * B * nv, seed, 2, bf16=bf16).reshape(T, B * nv)
    b_all = orc.normal(T * B * nv, seed, 3, bf16=bf16).reshape(T, B * nv)
    pos0 = np.zeros(B, np.int32) if pos0 is None else pos0.astype(np.int32)
    # oracle
    S, ring = lay["S"].copy(), lay["ring"].copy()
    o_ref = np.zeros((T, B * nv * hd), np.float32)
    L = orc.lib()
    flags = orc.F_ACT_BF16 if bf16 else 0
    for t in range(T):
        posv = pos0 + t
        q, a, b = (np.ascontiguousarray(x[t]) for x in (qkv_all, a_all, b_all))
        o = np.zeros(B * nv * hd, np.float32)
        L.orc_deltanet_decode_batch_mt(orc.P(S), orc.P(ring), orc.P(q), orc.P(a), orc.P(b),
                                       orc.P(lay["A_log"]), orc.P(lay["dt_bias"]),
                                       orc.P(lay["conv_w"]), orc.P(posv), orc.P(o), B, nqk, nv,
                                       hd, flags, 8)
        o_ref[t] = o
    # GPU
    dS = dev(lay["S"]).view(B, nv, hd, hd)
    dring = dev(lay["ring"])
    dq = dev(qkv_all, bf16)
    if gates_f64:
        # host-computed gates through the reference-identical C-ABI gate function
        from oracle.oracle import from_bf16
        af = from_bf16(a_all) if bf16 else a_all
        bf = from_bf16(b_all) if bf16 else b_all
        gb = np.zeros((T, B * nv)), np.zeros((T, B * nv))
        for t in range(T):
            for i in range(B * nv):
                gb[0][t, i], gb[1][t, i] = ops.vx27_deltanet_gate_params(
                    float(af[t, i]), float(lay["A_log"][i % nv]), float(bf[t, i]),
                    float(lay["dt_bias"][i % nv]))
        da, db = dev(gb[0]), dev(gb[1])
    else:
        da, db = dev(a_all, bf16), dev(b_all, bf16)
    dA, dd, dw = dev(lay["A_log"]), dev(lay["dt_bias"]), dev(lay["conv_w"])
    dpos = dev(pos0)
    do = torch.empty((T, B * nv * hd), dtype=torch.bfloat16 if out_bf16 else torch.float32,
                     device="cuda")
    for t in range(T):
        ops.deltanet_decode_batch(dS, dring, dq[t], da[t], db[t], dA, dd, dw, dpos, do[t], nqk, nv,
                                  gates_f64=gates_f64)
        ops.add_int(dpos, 1)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    o_gpu = host(do)
    if out_bf16:
        o_gpu = (o_gpu.astype(np.uint32) << 16).view(np.float32)
    return o_ref, S, ring, o_gpu, host(dS).reshape(-1), host(dring)


def test_config0_full_2000_tokens(cuda, orc):
    """Config 0: 16 heads, batch 1, zero state, 2000 tokens, fp32 activations, seed 0."""
    B, nqk, nv, T = 1, 16, 16, 2000
    lay = make_layer(orc, 0, B, nqk, nv)
    o_ref, S_ref, ring_ref, o, S, ring = run_both(orc, lay, T, B, nqk, nv, 0, bf16=False)
    err_o, err_s = np.abs(o - o_ref).max(), np.abs(S - S_ref).max()
    print(f"config0: max|o-ref|={err_o:.3e} max|S-ref|={err_s:.3e}")
    assert err_o < TOL and err_s < TOL
    assert np.array_equal(ring, ring_ref)  # the conv history is copied bits


def test_bf16_grouped_heads_ragged_positions(cuda, orc):
    """Real-model head grouping (48 V heads over 16 QK heads), bf16 activations, a batch
    whose sequences sit at different positions, non-zero initial state."""
    B, nqk, nv, T = 3, 16, 48, 12
    lay = make_layer(orc, 5, B, nqk, nv, s_std=0.05)
    o_ref, S_ref, _, o, S, _ = run_both(orc, lay, T, B, nqk, nv, 5, bf16=True,
                                        pos0=np.array([0, 2, 117]))
    assert np.abs(o - o_ref).max() < TOL and np.abs(S - S_ref).max() < TOL


def test_host_gates_and_bf16_output(cuda, orc):
    B, nqk, nv, T = 2, 2, 6, 6
    lay = make_layer(orc, 6, B, nqk, nv, s_std=0.05)
    o_ref, S_ref, _, o, S, _ = run_both(orc, lay, T, B, nqk, nv, 6, bf16=True, gates_f64=True,
                                        out_bf16=True)
    assert np.abs(S - S_ref).max() < TOL
    # bf16 output: within one bf16 rounding of the fp32 reference
    assert np.all(np.abs(o - o_ref) <= np.abs(o_ref) * 2.0 ** -8 + TOL)


def test_conv_ring_import_export_roundtrip(cuda, orc):
    import ctypes as C
    from vx27_b200._lib import errbuf, load
    B, Cch = 3, 640
    state = orc.normal(B * Cch * 3, 12, 1)
    pos = np.array([0, 5, 1030], np.int32)
    ring = torch.zeros(B * 4 * Cch, device="cuda")
    e = errbuf()
    lib = load()
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.vx27_deltanet_conv_import(C.c_void_p(ring.data_ptr()), state.ctypes.data_as(C.c_void_p),
                                         pos.ctypes.data_as(C.c_void_p), B, Cch, st, e, 512) == 0
    back = np.zeros_like(state)
    assert lib.vx27_deltanet_conv_export(C.c_void_p(ring.data_ptr()), back.ctypes.data_as(C.c_void_p),
                                         pos.ctypes.data_as(C.c_void_p), B, Cch, st, e, 512) == 0
    assert np.array_equal(back, state)


@pytest.mark.parametrize("bf16", [False, True])
def test_gated_rmsnorm_output(cuda, orc, bf16):
    """vx27_deltanet_decode_batch_gated == decode step, then the layer's gated RMSNorm
    output (src/vx27_qfwd.c:146-151) on the oracle's retrieve output; 48 V heads over 16 QK
    heads as in the real model, 3 tokens."""
    B, nqk, nv, hd, T = 3, 16, 48, 128, 3
    lay = make_layer(orc, 31, B, nqk, nv, s_std=0.05)
    Cch = lay["C"]
    L = orc.lib()
    qkv_all = orc.normal(T * B * Cch, 31, 1, bf16=bf16).reshape(T, B * Cch)
    a_all = orc.normal(T * B * nv, 31, 2, bf16=bf16).reshape(T, B * nv)
    b_all = orc.normal(T * B * nv, 31, 3, bf16=bf16).reshape(T, B * nv)
    z_all = orc.normal(T * B * nv * hd, 31, 7, bf16=bf16).reshape(T, B * nv * hd)
    norm_w = orc.normal(hd, 31, 8, 1.0, 0.1)
    flags = orc.F_ACT_BF16 if bf16 else 0
    S, ring = lay["S"].copy(), lay["ring"].copy()
    dS = dev(lay["S"]).view(B, nv, hd, hd)
    dring = dev(lay["ring"])
    from oracle.oracle import from_bf16
    for t in range(T):
        pos = np.full(B, t, np.int32)
        q, a, b = (np.ascontiguousarray(x[t]) for x in (qkv_all, a_all, b_all))
        r = np.zeros(B * nv * hd, np.float32)
        L.orc_deltanet_decode_batch_mt(orc.P(S), orc.P(ring), orc.P(q), orc.P(a), orc.P(b),
                                       orc.P(lay["A_log"]), orc.P(lay["dt_bias"]),
                                       orc.P(lay["conv_w"]), orc.P(pos), orc.P(r), B, nqk, nv,
                                       hd, flags, 8)
        zf = np.ascontiguousarray(from_bf16(z_all[t]) if bf16 else z_all[t])
        y_ref = np.zeros(B * nv * hd, np.float32)
        L.orc_gated_rmsnorm(orc.P(r), orc.P(norm_w), orc.P(zf), orc.P(y_ref), B * nv, hd)
        o = torch.empty(B, nv, hd, device="cuda")
        ops.deltanet_decode_batch_gated(dS, dring, dev(q, bf16).view(B, Cch),
                                        dev(a, bf16).view(B, nv), dev(b, bf16).view(B, nv),
                                        dev(lay["A_log"]), dev(lay["dt_bias"]),
                                        dev(lay["conv_w"]).view(Cch, 4),
                                        torch.from_numpy(pos).cuda(),
                                        dev(z_all[t], bf16).view(B, nv, hd), dev(norm_w), o,
                                        nqk, nv)
        torch.cuda.synchronize()
        assert np.abs(host(o).reshape(-1) - y_ref).max() < TOL
    assert np.abs(host(dS).reshape(-1) - S).max() < TOL
    assert ops.device_status() == 0


def test_decode_tokens_with_checkpoints(cuda, orc):
    """vx27_deltanet_decode_tokens: 5 teacher-forced tokens of one sequence with state and
    conv snapshots after each token (vx27_qlayer_batch's Sckpt/Cckpt), against the oracle
    stepping token by token; then a partial commit of 3 tokens (restore from the
    snapshots) continues exactly like a run that only ever saw those 3 tokens."""
    nqk, nv, hd, T, p0 = 2, 6, 128, 5, 9
    lay = make_layer(orc, 41, 1, nqk, nv, s_std=0.05)
    Cch = lay["C"]
    L = orc.lib()
    lay["ring"] = orc.normal(4 * Cch, 41, 9)  # some history at position p0
    qkv = orc.normal(T * Cch, 41, 1, bf16=True).reshape(T, Cch)
    a = orc.normal(T * nv, 41, 2, bf16=True).reshape(T, nv)
    b = orc.normal(T * nv, 41, 3, bf16=True).reshape(T, nv)
    S, ring = lay["S"].copy(), lay["ring"].copy()
    o_ref, S_ref, c_ref = [], [], []
    for t in range(T):
        p = np.array([p0 + t], np.int32)
        o = np.zeros(nv * hd, np.float32)
        L.orc_deltanet_decode_batch_mt(orc.P(S), orc.P(ring), orc.P(np.ascontiguousarray(qkv[t])),
                                       orc.P(np.ascontiguousarray(a[t])),
                                       orc.P(np.ascontiguousarray(b[t])), orc.P(lay["A_log"]),
                                       orc.P(lay["dt_bias"]), orc.P(lay["conv_w"]), orc.P(p),
                                       orc.P(o), 1, nqk, nv, hd, orc.F_ACT_BF16, 4)
        o_ref.append(o)
        S_ref.append(S.copy())
        r4 = ring.reshape(4, Cch)
        pp = p0 + t
        c_ref.append(np.stack([r4[(pp - 2) & 3], r4[(pp - 1) & 3], r4[pp & 3]], axis=1))
    dS = dev(lay["S"]).view(nv, hd, hd)
    dring = dev(lay["ring"]).view(4, Cch)
    o = torch.empty(T, nv, hd, device="cuda")
    S_ck = torch.empty(T, nv, hd, hd, device="cuda")
    c_ck = torch.empty(T, Cch, 3, device="cuda")
    pos = torch.arange(p0, p0 + T, dtype=torch.int32, device="cuda")
    args = (dev(lay["A_log"]), dev(lay["dt_bias"]), dev(lay["conv_w"]).view(Cch, 4))
    ops.deltanet_decode_tokens(dS, dring, dev(qkv, True), dev(a, True), dev(b, True), *args, pos,
                               o, nqk, nv, S_ckpt=S_ck, conv_ckpt=c_ck)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    for t in range(T):
        assert np.abs(host(o[t]).reshape(-1) - o_ref[t]).max() < TOL
        assert np.abs(host(S_ck[t]).reshape(-1) - S_ref[t]).max() < TOL
        assert np.array_equal(host(c_ck[t]), c_ref[t])
    # partial commit: keep 3 tokens, restore state + conv history, decode token 4 again
    k = 3
    S2 = S_ck[k - 1].clone()
    ring2 = torch.zeros(1, 4, Cch, device="cuda")
    from ctypes import create_string_buffer
    st = np.ascontiguousarray(host(c_ck[k - 1]).reshape(1, Cch, 3))
    e = create_string_buffer(512)
    assert ops.load().vx27_deltanet_conv_import(ops._t(ring2), st.ctypes.data_as(ops.C.c_void_p),
                                                np.array([p0 + k], np.int32).ctypes.data_as(
                                                    ops.C.c_void_p), 1, Cch, None, e, 512) == 0
    o2 = torch.empty(1, nv, hd, device="cuda")
    ops.deltanet_decode_tokens(S2, ring2.view(4, Cch), dev(qkv[k:k + 1], True),
                               dev(a[k:k + 1], True), dev(b[k:k + 1], True), *args, pos[k:k + 1],
                               o2, nqk, nv)
    torch.cuda.synchronize()
    assert np.abs(host(o2).reshape(-1) - o_ref[k]).max() < TOL
    assert np.abs(host(S2).reshape(-1) - S_ref[k]).max() < TOL


def _tokens_vs_oracle(orc, seed, nqk, nv, T, p0, bf16, s_std=0.0, gates_f64=False,
                     positions=None, ckpt=False):
    """One vx27_deltanet_decode_tokens call over T tokens (state resident in the kernel)
    against the oracle stepping token by token (positions p0 + t, or the given ones); with
    ckpt, the per-token state and conv snapshots are compared too."""
    hd = 128
    positions = (np.arange(p0, p0 + T) if positions is None else np.asarray(positions)).astype(np.int32)
    lay = make_layer(orc, seed, 1, nqk, nv, s_std=s_std)
    Cch = lay["C"]
    lay["ring"] = orc.normal(4 * Cch, seed, 9)  # some conv history at position p0
    qkv = orc.normal(T * Cch, seed, 1, bf16=bf16).reshape(T, Cch)
    a = orc.normal(T * nv, seed, 2, bf16=bf16).reshape(T, nv)
    b = orc.normal(T * nv, seed, 3, bf16=bf16).reshape(T, nv)
    S, ring = lay["S"].copy(), lay["ring"].copy()
    L = orc.lib()
    o_ref = np.zeros((T, nv * hd), np.float32)
    S_ref, c_ref = [], []
    for t in range(T):
        o = np.zeros(nv * hd, np.float32)
        L.orc_deltanet_decode_batch_mt(orc.P(S), orc.P(ring), orc.P(np.ascontiguousarray(qkv[t])),
                                       orc.P(np.ascontiguousarray(a[t])),
                                       orc.P(np.ascontiguousarray(b[t])), orc.P(lay["A_log"]),
                                       orc.P(lay["dt_bias"]), orc.P(lay["conv_w"]),
                                       orc.P(positions[t:t + 1].copy()), orc.P(o), 1, nqk, nv,
                                       hd, orc.F_ACT_BF16 if bf16 else 0, 8)
        o_ref[t] = o
        if ckpt:
            S_ref.append(S.copy())
            r4, pp = ring.reshape(4, Cch), int(positions[t])
            c_ref.append(np.stack([r4[(pp - 2) & 3], r4[(pp - 1) & 3], r4[pp & 3]], axis=1))
    dS = dev(lay["S"]).view(nv, hd, hd)
    dring = dev(lay["ring"]).view(4, Cch)
    if gates_f64:
        from oracle.oracle import from_bf16
        af = from_bf16(a) if bf16 else a
        bf_ = from_bf16(b) if bf16 else b
        ga, gb = np.zeros((T, nv)), np.zeros((T, nv))
        for t in range(T):
            for i in range(nv):
                ga[t, i], gb[t, i] = ops.vx27_deltanet_gate_params(
                    float(af[t, i]), float(lay["A_log"][i]), float(bf_[t, i]),
                    float(lay["dt_bias"][i]))
        da, db = dev(ga), dev(gb)
    else:
        da, db = dev(a, bf16), dev(b, bf16)
    o = torch.empty(T, nv, hd, device="cuda")
    pos = dev(positions)
    S_ck = torch.empty(T, nv, hd, hd, device="cuda") if ckpt else None
    c_ck = torch.empty(T, Cch, 3, device="cuda") if ckpt else None
    ops.deltanet_decode_tokens(dS, dring, dev(qkv, bf16), da, db, dev(lay["A_log"]),
                               dev(lay["dt_bias"]), dev(lay["conv_w"]).view(Cch, 4), pos, o, nqk,
                               nv, gates_f64=gates_f64, S_ckpt=S_ck, conv_ckpt=c_ck)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    if ckpt:
        for t in range(T):
            assert np.abs(host(S_ck[t]).reshape(-1) - S_ref[t]).max() < TOL
            assert np.array_equal(host(c_ck[t]), c_ref[t])
    return (np.abs(host(o).reshape(T, -1) - o_ref).max(), np.abs(host(dS).reshape(-1) - S).max(),
            np.array_equal(host(dring).reshape(-1), ring))


def test_tokens_config0_state_resident(cuda, orc):
    """Config 0's 2000 tokens in one vx27_deltanet_decode_tokens call (the kernel keeps each
    head's state in registers across tokens) within the tolerance of the oracle, and the
    conv ring left as 2000 single-token calls leave it."""
    err_o, err_s, ring_eq = _tokens_vs_oracle(orc, 0, 16, 16, 2000, 0, bf16=False)
    print(f"config0 tokens: max|o-ref|={err_o:.3e} max|S-ref|={err_s:.3e}")
    assert err_o < TOL and err_s < TOL and ring_eq


@pytest.mark.parametrize("gates_f64", [False, True])
def test_tokens_grouped_heads_bf16(cuda, orc, gates_f64):
    """48 V heads over 16 QK heads, bf16 activations, non-zero state, a ragged start
    position (the conv history crosses the ring's wrap)."""
    err_o, err_s, ring_eq = _tokens_vs_oracle(orc, 7, 16, 48, 37, 1029, bf16=True, s_std=0.05,
                                              gates_f64=gates_f64)
    assert err_o < TOL and err_s < TOL and ring_eq


def test_tokens_any_positions(cuda, orc):
    """Positions that jump and repeat (the conv history follows the ring by position, as
    T single-token calls would) and a run long enough to cross the kernel's 32-token gate
    batches."""
    positions = [7, 8, 9, 13, 2, 3, 3, 40] + list(range(100, 130))
    err_o, err_s, ring_eq = _tokens_vs_oracle(orc, 8, 2, 6, len(positions), 0, bf16=True,
                                              s_std=0.05, positions=positions)
    assert err_o < TOL and err_s < TOL and ring_eq


def test_tokens_checkpoints_across_gate_batches(cuda, orc):
    """State and conv snapshots after each of 70 tokens (three 32-token gate batches)."""
    err_o, err_s, ring_eq = _tokens_vs_oracle(orc, 9, 2, 6, 70, 31, bf16=True, s_std=0.05,
                                              ckpt=True)
    assert err_o < TOL and err_s < TOL and ring_eq
