"""K3 (vx27_deltanet_prefill_chunked, chunked gated delta rule) against the token-by-token
recurrent reference (step_exact per token and head, src/vx27_deltanet.c:71-102).
Tolerance: chunked prefill within 1e-3 of the recurrent reference, for the
outputs and the final state."""
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest
import torch

from gpu_util import dev, host
from vx27_b200 import ops

pytestmark = pytest.mark.gpu
HD = 128
TOL = 1e-3


def make(orc, seed, T, nqk, nv, s_std=0.0, a_range=(1.0, 16.0)):
    """Config-0 gates by default: A_log = log U[1,16]; a smaller range gives slow decay."""
    g = lambda n, s, m=0.0, sd=1.0, b=True: orc.normal(n, seed, s, m, sd, bf16=b)
    S0 = (orc.normal(nv * HD * HD, seed, 9, 0.0, s_std) if s_std else
          np.zeros(nv * HD * HD, np.float32))
    return dict(q=g(T * nqk * HD, 1), k=g(T * nqk * HD, 2), v=g(T * nv * HD, 3),
                a=g(T * nv, 4), b=g(T * nv, 5),
                A_log=np.log(orc.uniform(nv, seed, 6, *a_range)).astype(np.float32),
                dt=g(nv, 7, 0.0, 0.1, False), S0=S0)


def recurrent(orc, x, T, nqk, nv, threads=8):
    from oracle.oracle import from_bf16
    L, P = orc.lib(), orc.P
    af = np.ascontiguousarray(from_bf16(x["a"]))
    bf = np.ascontiguousarray(from_bf16(x["b"]))
    beta_all = np.zeros((T, nv))
    g_all = np.zeros((T, nv))
    L.orc_gate_params_grid(P(af), P(bf), P(x["A_log"]), P(x["dt"]), T, nv, P(beta_all),
                           P(g_all))
    S = x["S0"].reshape(nv, HD, HD).copy()
    o = np.zeros((nv, T, HD), np.float32)

    def head(vh):
        qk = vh * nqk // nv
        beta = np.ascontiguousarray(beta_all[:, vh])
        glog = np.ascontiguousarray(g_all[:, vh])
        Sh = np.ascontiguousarray(S[vh])
        oh = np.zeros((T, HD), np.float32)
        qh = np.ascontiguousarray(x["q"].reshape(T, nqk, HD)[:, qk])
        kh = np.ascontiguousarray(x["k"].reshape(T, nqk, HD)[:, qk])
        vhv = np.ascontiguousarray(x["v"].reshape(T, nv, HD)[:, vh])
        L.orc_deltanet_recurrent(P(Sh), P(qh), P(kh), P(vhv), HD, P(beta), P(glog), P(oh), T, HD,
                                 orc.F_ACT_BF16)
        S[vh] = Sh
        o[vh] = oh

    with ThreadPoolExecutor(threads) as ex:
        list(ex.map(head, range(nv)))
    return o.transpose(1, 0, 2), S


def gpu(x, T, nqk, nv, out_bf16=False):
    q = dev(x["q"], True).view(T, nqk, HD)
    k = dev(x["k"], True).view(T, nqk, HD)
    v = dev(x["v"], True).view(T, nv, HD)
    a = dev(x["a"], True).view(T, nv)
    b = dev(x["b"], True).view(T, nv)
    S = dev(x["S0"]).view(nv, HD, HD)
    o = torch.empty(T, nv, HD, dtype=torch.bfloat16 if out_bf16 else torch.float32, device="cuda")
    ops.deltanet_prefill_chunked(q, k, v, a, b, dev(x["A_log"]), dev(x["dt"]), S, o)
    torch.cuda.synchronize()
    return o.float().cpu().numpy(), host(S)


@pytest.mark.parametrize("T", [1, 63, 64, 65, 200])
def test_short_prompts(cuda, orc, T):
    nqk = nv = 2
    x = make(orc, 30 + T, T, nqk, nv, s_std=0.05)
    o_ref, S_ref = recurrent(orc, x, T, nqk, nv)
    o, S = gpu(x, T, nqk, nv)
    assert np.abs(o - o_ref).max() < TOL and np.abs(S - S_ref).max() < TOL


def test_grouped_heads(cuda, orc):
    T, nqk, nv = 150, 2, 6
    x = make(orc, 77, T, nqk, nv, s_std=0.05)
    o_ref, S_ref = recurrent(orc, x, T, nqk, nv)
    o, S = gpu(x, T, nqk, nv)
    assert np.abs(o - o_ref).max() < TOL and np.abs(S - S_ref).max() < TOL


def test_slow_decay_long_memory(cuda, orc):
    """Decay rates 1e-3..5e-2 of config 0's: the state carries information across hundreds
    of chunks, so errors in the chunk transfer would accumulate."""
    T, nqk, nv = 4000, 2, 4
    x = make(orc, 55, T, nqk, nv, s_std=0.05, a_range=(0.001, 0.05))
    o_ref, S_ref = recurrent(orc, x, T, nqk, nv)
    o, S = gpu(x, T, nqk, nv)
    eo, es = np.abs(o - o_ref).max(), np.abs(S - S_ref).max()
    print(f"slow decay: max|o-ref| {eo:.3e}, max|S-ref| {es:.3e}, max|S| {np.abs(S_ref).max():.3f}")
    assert eo < TOL and es < TOL


def test_bf16_output_and_f32_rejected(cuda, orc):
    T, nqk, nv = 130, 2, 2
    x = make(orc, 8, T, nqk, nv, s_std=0.05)
    o_ref, S_ref = recurrent(orc, x, T, nqk, nv)
    o, S = gpu(x, T, nqk, nv, out_bf16=True)
    assert np.abs(o - o_ref).max() < 1e-2 and np.abs(S - S_ref).max() < TOL
    q = dev(x["q"], True).view(T, nqk, HD).float()
    with pytest.raises(ops.Vx27Error, match="bf16"):
        ops.deltanet_prefill_chunked(q, q, dev(x["v"], True).view(T, nv, HD).float(),
                                     dev(x["a"], True).view(T, nv), dev(x["b"], True).view(T, nv),
                                     dev(x["A_log"]), dev(x["dt"]),
                                     dev(x["S0"]).view(nv, HD, HD),
                                     torch.empty(T, nv, HD, device="cuda"))


def test_config4_deltanet_32768(cuda, orc):
    """Config 4 DeltaNet path: T = 32768, 16 heads, zero initial state, seed 4."""
    T, nqk, nv = 32768, 16, 16
    x = make(orc, 4, T, nqk, nv)
    o_ref, S_ref = recurrent(orc, x, T, nqk, nv, threads=16)
    o, S = gpu(x, T, nqk, nv)
    eo, es = np.abs(o - o_ref).max(), np.abs(S - S_ref).max()
    print(f"config4 DeltaNet: max|o-ref| {eo:.3e}, max|S-ref| {es:.3e}")
    assert eo < TOL and es < TOL
