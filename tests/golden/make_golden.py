"""Generates the golden vectors in tests/golden/ from the reference's own code.

The reference's hot-path sources (src/vx27_deltanet.c, src/vx27_deltanet_avx2.c,
src/vx27_gqa.c, src/vx27_rope.c, src/vx27_kv.c of DavidPandleton/vx27) are compiled
unmodified into oracle/_ref/libvx27ref.so by `make -C oracle ref`; this script calls
those functions through ctypes on seeded inputs and stores inputs and outputs. For the
batched drivers (one DeltaNet layer over a batch, GQA append + attention), the oracle's
driver loops are run with the reference's functions plugged in (orc_use_reference), so
every per-head computation in those fixtures is the reference's own.

Run:  python tests/golden/make_golden.py      (needs the reference sources)
"""
from __future__ import annotations

import ctypes as C
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
from oracle import oracle as orc  # noqa: E402

_p, _i, _f, _d = C.c_void_p, C.c_int, C.c_float, C.c_double


def ref_lib() -> C.CDLL:
    if not orc.build_ref():
        raise SystemExit("reference sources unavailable: cannot build oracle/_ref")
    l = C.CDLL(orc.REF_LIB)
    protos = {
        "vx27_deltanet_update_ref": (None, [_p, _p, _p, _f, _i]),
        "vx27_deltanet_update_tiled": (None, [_p, _p, _p, _f, _i]),
        "vx27_deltanet_update_avx2": (None, [_p, _p, _p, _f, _i]),
        "vx27_deltanet_retrieve_ref": (None, [_p, _p, _p, _i]),
        "vx27_deltanet_retrieve_tiled": (None, [_p, _p, _p, _i]),
        "vx27_deltanet_retrieve_avx2": (None, [_p, _p, _p, _i]),
        "vx27_deltanet_l2norm": (None, [_p, _p, _i]),
        "vx27_deltanet_step_exact": (None, [_p, _p, _p, _p, _d, _d, _p, _i]),
        "vx27_deltanet_gate_params": (None, [_d, _d, _d, _d, C.POINTER(_d), C.POINTER(_d)]),
        "vx27_conv1d_step": (None, [_p, _p, _p, _p, _i, _i]),
        "vx27_gqa_kv_for_q": (_i, [_i]),
        "vx27_rmsnorm": (None, [_p, _p, _p, _i, _f]),
        "vx27_attn_1q": (None, [_p, _p, _p, _i, _p]),
        "vx27_rope_cos_sin": (None, [_i, _p, _p, _i, _f, _f]),
        "vx27_rope_apply": (None, [_p, _i, _i, _i, _p, _p]),
        "vx27_kv_elems": (C.c_uint64, [_i]),
        "vx27_kv_gb": (_d, [_i, _d]),
        "vx27_kv_fits": (_i, [_i, _d, _d]),
        "vx27_deltanet_state_per_layer": (_i, []),
        "vx27_deltanet_state_total": (_i, []),
        "vx27_deltanet_state_mb": (_d, [_i]),
    }
    for n, (r, a) in protos.items():
        fn = getattr(l, n)
        fn.restype, fn.argtypes = r, a
    return l


P = orc.P
GATE_PINS = [(0.1, 0.5, -0.3, 1.0), (3.0, -1.2, 2.0, 1.0), (-25.0, 0.0, 0.0, 1.0),
             (25.0, 2.0, -2.0, 1.0), (0.0, -5.0, 5.0, -3.0), (-30.0, 1.0, 30.0, 30.0)]


def main() -> None:
    R = ref_lib()
    rng = np.random.default_rng(20261201)
    out = {}

    # gates: the six pinned cases of tests/test_deltanet_exact.c:44-47 + seeded cases
    g_in = np.array(GATE_PINS + [tuple(rng.normal(0, s, 4)) for s in (1, 5, 12) for _ in range(100)],
                    dtype=np.float64)
    g_out = np.zeros((len(g_in), 2))
    for n, (a, al, b, dt) in enumerate(g_in):
        be, gg = C.c_double(), C.c_double()
        R.vx27_deltanet_gate_params(a, al, b, dt, C.byref(be), C.byref(gg))
        g_out[n] = (be.value, gg.value)
    out.update(gate_in=g_in, gate_out=g_out)

    # step_exact chains: hd 128 (1 trial), 32 and 8 (2 trials each), 6 steps
    for hd, trials in ((128, 1), (32, 2), (8, 2)):
        S0 = rng.uniform(-0.5, 0.5, (trials, hd * hd)).astype(np.float32)
        q = rng.uniform(-1, 1, (trials, 6, hd)).astype(np.float32)
        k = rng.uniform(-1, 1, (trials, 6, hd)).astype(np.float32)
        v = (rng.uniform(-1, 1, (trials, 6, hd)) * 2).astype(np.float32)
        beta = rng.uniform(0.05, 0.95, (trials, 6))
        glog = -8.0 * rng.uniform(0, 1, (trials, 6))
        S = S0.copy()
        o = np.zeros((trials, 6, hd), np.float32)
        for t in range(trials):
            st = np.ascontiguousarray(S[t])
            for s in range(6):
                ot = np.zeros(hd, np.float32)
                R.vx27_deltanet_step_exact(P(st), P(np.ascontiguousarray(q[t, s])),
                                           P(np.ascontiguousarray(k[t, s])),
                                           P(np.ascontiguousarray(v[t, s])), float(beta[t, s]),
                                           float(glog[t, s]), P(ot), hd)
                o[t, s] = ot
            S[t] = st
        out.update({f"step{hd}_S0": S0, f"step{hd}_q": q, f"step{hd}_k": k, f"step{hd}_v": v,
                    f"step{hd}_beta": beta, f"step{hd}_g": glog, f"step{hd}_S": S,
                    f"step{hd}_o": o})

    # update / retrieve, inputs of tests/test_deltanet.c:39 plus a random state
    for hd in (128, 8):
        i = np.arange(hd)
        k = ((i % 7) * 0.1 - 0.3).astype(np.float32)
        v = ((i % 5) * 0.2).astype(np.float32)
        q = ((i % 3) * 0.15 - 0.1).astype(np.float32)
        S0 = rng.normal(0, 0.3, hd * hd).astype(np.float32)
        res = {}
        for name in ("ref", "tiled", "avx2"):
            S = S0.copy()
            getattr(R, f"vx27_deltanet_update_{name}")(P(S), P(k), P(v), 0.9, hd)
            o = np.zeros(hd, np.float32)
            getattr(R, f"vx27_deltanet_retrieve_{name}")(P(S), P(q), P(o), hd)
            res[f"ur{hd}_{name}_S"] = S
            res[f"ur{hd}_{name}_o"] = o
        out.update(res)
        out.update({f"ur{hd}_S0": S0, f"ur{hd}_k": k, f"ur{hd}_v": v, f"ur{hd}_q": q})

    # conv1d_step over T=8 steps, C=64 (tests/test_deltanet_exact.c:110-138 shape x2)
    Cc, T = 64, 8
    w = (rng.uniform(-1, 1, Cc * 4) * 0.3).astype(np.float32)
    xs = rng.uniform(-1, 1, (T, Cc)).astype(np.float32)
    st = np.zeros(Cc * 3, np.float32)
    ys = np.zeros((T, Cc), np.float32)
    for t in range(T):
        y = np.zeros(Cc, np.float32)
        R.vx27_conv1d_step(P(st), P(np.ascontiguousarray(xs[t])), P(w), P(y), Cc, 1)
        ys[t] = y
    out.update(conv_w=w, conv_x=xs, conv_y=ys, conv_state=st)

    # l2norm and rmsnorm
    for n in (2, 128, 256, 5120):
        x = rng.normal(0, 2, n).astype(np.float32)
        wv = (1 + rng.normal(0, 0.02, n)).astype(np.float32)
        y1 = np.zeros(n, np.float32)
        y2 = np.zeros(n, np.float32)
        R.vx27_deltanet_l2norm(P(x), P(y1), n)
        R.vx27_rmsnorm(P(x), P(wv), P(y2), n, 1e-6)
        out.update({f"norm{n}_x": x, f"norm{n}_w": wv, f"l2norm{n}": y1, f"rmsnorm{n}": y2})
    y = np.zeros(2, np.float32)
    R.vx27_rmsnorm(P(np.array([3, 4], np.float32)), P(np.ones(2, np.float32)), P(y), 2, 0.0)
    out["rmsnorm_34"] = y

    # RoPE tables and rotation
    pos = np.array([0, 1, 7, 8, 32, 4095, 4096, 8191, 32767, 262143, 1000003], np.int32)
    yarn = np.array([1, 1, 1, 1, 4, 1, 1, 1, 1, 1, 1], np.float32)
    cs = np.zeros((len(pos), 32), np.float32)
    sn = np.zeros((len(pos), 32), np.float32)
    for n, (p_, y_) in enumerate(zip(pos, yarn)):
        c, s = np.zeros(32, np.float32), np.zeros(32, np.float32)
        R.vx27_rope_cos_sin(int(p_), P(c), P(s), 64, 10000000.0, float(y_))
        cs[n], sn[n] = c, s
    vr = rng.normal(0, 1, (len(pos), 4 * 256)).astype(np.float32)
    vrot = vr.copy()
    for n in range(len(pos)):
        row = np.ascontiguousarray(vrot[n])
        R.vx27_rope_apply(P(row), 4, 256, 64, P(cs[n]), P(sn[n]))
        vrot[n] = row
    out.update(rope_pos=pos, rope_yarn=yarn, rope_cos=cs, rope_sin=sn, rope_x=vr, rope_y=vrot)

    # attn_1q, fp32 caches
    for n_pos in (1, 2, 5, 13):
        q = rng.normal(0, 1, 24 * 256).astype(np.float32)
        kc = rng.normal(0, 1, n_pos * 4 * 256).astype(np.float32)
        vc = rng.normal(0, 1, n_pos * 4 * 256).astype(np.float32)
        o = np.zeros(24 * 256, np.float32)
        R.vx27_attn_1q(P(q), P(kc), P(vc), n_pos, P(o))
        out.update({f"attn{n_pos}_q": q, f"attn{n_pos}_k": kc, f"attn{n_pos}_v": vc,
                    f"attn{n_pos}_o": o})

    # sizing
    ctxs = np.array([1, 512, 8192, 65536, 131072, 262144], np.int32)
    out.update(kv_ctx=ctxs,
               kv_elems=np.array([R.vx27_kv_elems(int(c)) for c in ctxs], np.uint64),
               kv_gb=np.array([R.vx27_kv_gb(int(c), 2.0) for c in ctxs]),
               kv_fits=np.array([R.vx27_kv_fits(int(c), b_, 2.5) for c in ctxs
                                 for b_ in (0.5, 2.0)], np.int32),
               sizes=np.array([R.vx27_deltanet_state_per_layer(), R.vx27_deltanet_state_total()]),
               state_mb=np.array([R.vx27_deltanet_state_mb(2), R.vx27_deltanet_state_mb(4)]),
               headmap=np.array([R.vx27_gqa_kv_for_q(h) for h in range(24)], np.int32))

    # batched drivers with the reference's per-head functions plugged in
    assert orc.use_reference(True) and orc.lib().orc_impl_is_reference() == 1
    L = orc.lib()
    B, nqk, nv, hd, steps = 1, 1, 3, 128, 5
    Cch = (2 * nqk + nv) * hd
    S = orc.normal(B * nv * hd * hd, 7, 1, 0.0, 0.05)
    ring = np.zeros(B * 4 * Cch, np.float32)
    conv_w = orc.normal(Cch * 4, 7, 2, 0.0, 0.5)
    A_log = np.log(orc.uniform(nv, 7, 3, 1.0, 16.0)).astype(np.float32)
    dt_bias = orc.normal(nv, 7, 4, 0.0, 0.1)
    os_ = np.zeros((steps, B * nv * hd), np.float32)
    for t in range(steps):
        qkv = orc.normal(B * Cch, 7, 100 + t, bf16=True)
        a = orc.normal(B * nv, 7, 200 + t, bf16=True)
        b = orc.normal(B * nv, 7, 300 + t, bf16=True)
        posv = np.full(B, t, np.int32)
        o = np.zeros(B * nv * hd, np.float32)
        L.orc_deltanet_decode_batch(P(S), P(ring), P(qkv), P(a), P(b), P(A_log), P(dt_bias),
                                    P(conv_w), P(posv), P(o), B, nqk, nv, hd, orc.F_ACT_BF16)
        os_[t] = o
    # inputs are regenerated from the same seeds by the tests (orc.normal is deterministic)
    out.update(dn_S=S, dn_ring=ring, dn_o=os_)

    B, nq, nkv, hd, cap = 2, 24, 4, 256, 48
    posv = np.array([10, 37], np.int32)
    kc = orc.normal(B * nkv * cap * hd, 8, 1, bf16=True)
    vc = orc.normal(B * nkv * cap * hd, 8, 2, bf16=True)
    qi = orc.normal(B * nq * hd, 8, 3, bf16=True)
    ki = orc.normal(B * nkv * hd, 8, 4, bf16=True)
    vi = orc.normal(B * nkv * hd, 8, 5, bf16=True)
    gt = orc.normal(B * nq * hd, 8, 6, bf16=True)
    qw = orc.normal(hd, 8, 7, 1.0, 0.02)
    kw = orc.normal(hd, 8, 8, 1.0, 0.02)
    kc0, vc0 = kc.copy(), vc.copy()
    qo = np.zeros(B * nq * hd, np.float32)
    L.orc_gqa_append(P(qi), P(ki), P(vi), P(qw), P(kw), P(posv), P(kc), P(vc), cap, P(qo), B, nq,
                     nkv, hd, 64, 10000000.0, 1e-6, orc.F_ACT_BF16)
    att = np.zeros(B * nq * hd, np.float32)
    L.orc_gqa_attend(P(qo), P(gt), P(kc), P(vc), cap, P(posv), P(att), B, nq, nkv, hd,
                     orc.F_ACT_BF16)
    kr = kc.reshape(B, nkv, cap, hd)[np.arange(B), :, posv]  # appended rows [B][nkv][hd]
    vr_ = vc.reshape(B, nkv, cap, hd)[np.arange(B), :, posv]
    out.update(gq_pos=posv, gq_krow=kr, gq_vrow=vr_, gq_qo=qo, gq_out=att)
    orc.use_reference(False)

    path = os.path.join(HERE, "golden_ref.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({os.path.getsize(path) / 1e6:.2f} MB, {len(out)} arrays)")


if __name__ == "__main__":
    main()
