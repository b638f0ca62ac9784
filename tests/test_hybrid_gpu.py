"""The batched hybrid decode step (vx27_b200.hybrid, the config 2 driver): layer order,
per-layer wiring against the CPU oracle, and the host-buffer step (copies overlapped with
compute) against the device-resident step."""
import numpy as np
import pytest
import torch

from gpu_util import host, rel_err
from vx27_b200.hybrid import HybridConfig, HybridDecoder, layer_kind

pytestmark = pytest.mark.gpu


def test_layer_order_is_three_deltanet_then_one_gqa():
    kinds = [layer_kind(L) for L in range(64)]
    assert [k[0] for k in kinds[:8]] == [False, False, False, True] * 2
    assert sum(k[0] for k in kinds) == 16
    assert kinds[63] == (True, 15) and kinds[62] == (False, 47)


@pytest.mark.parametrize("fused_gqa", [False, True])
def test_step_layers_match_oracle(cuda, orc, fused_gqa):
    cfg = HybridConfig(batch=3, ctx=200, steps=2, seed=7, fused_gqa=fused_gqa)
    dec = HybridDecoder(cfg)
    # snapshot layer 0 (DeltaNet) and GQA layer 0 (model layer 3) before the step
    S0, ring0 = host(dec.S[0]).copy(), host(dec.ring[0]).copy()
    kc0, vc0 = host(dec.kc[0]).copy(), host(dec.vc[0]).copy()
    ins = {n: host(t) for n, t in zip(["qkv", "a", "b", "q_in", "k_in", "v_in", "gate"],
                                      dec.step_inputs())}
    dec.step()
    torch.cuda.synchronize()
    P, L, B = orc.P, orc.lib(), cfg.batch
    # DeltaNet layer 0
    S = np.ascontiguousarray(S0.reshape(-1))
    ring = np.ascontiguousarray(ring0.reshape(-1))
    o = np.zeros(B * cfg.nv * 128, np.float32)
    pos = np.full(B, cfg.ctx, np.int32)
    bits = lambda t: np.ascontiguousarray(t.view(np.uint16).reshape(-1))
    L.orc_deltanet_decode_batch(P(S), P(ring), P(bits(ins["qkv"][0])), P(bits(ins["a"][0])),
                                P(bits(ins["b"][0])), P(host(dec.A_log[0]).copy()),
                                P(host(dec.dt_bias[0]).copy()),
                                P(np.ascontiguousarray(host(dec.conv_w[0]).reshape(-1))), P(pos),
                                P(o), B, cfg.nqk, cfg.nv, 128, orc.F_ACT_BF16)
    got = host(dec.dn_out[0].float()).reshape(-1)
    assert np.all(np.abs(got - o) <= np.abs(o) * 2.0 ** -8 + 1e-4)  # bf16 output rounding
    assert np.abs(host(dec.S[0]).reshape(-1) - S).max() < 1e-4
    # GQA layer 0
    kc, vc = np.ascontiguousarray(kc0.view(np.uint16).reshape(-1)), \
        np.ascontiguousarray(vc0.view(np.uint16).reshape(-1))
    qo = np.zeros(B * cfg.nq * cfg.hd, np.float32)
    L.orc_gqa_append(P(bits(ins["q_in"][0])), P(bits(ins["k_in"][0])), P(bits(ins["v_in"][0])),
                     P(host(dec.q_norm_w[0]).copy()), P(host(dec.k_norm_w[0]).copy()), P(pos),
                     P(kc), P(vc), cfg.cap, P(qo), B, cfg.nq, cfg.nkv, cfg.hd, 64, 1e7, 1e-6,
                     orc.F_ACT_BF16)
    att = np.zeros(B * cfg.nq * cfg.hd, np.float32)
    L.orc_gqa_attend(P(qo), P(bits(ins["gate"][0])), P(kc), P(vc), cfg.cap, P(pos), P(att), B,
                     cfg.nq, cfg.nkv, cfg.hd, orc.F_ACT_BF16)
    got = host(dec.att_out[0].float()).reshape(-1)
    assert rel_err(got, att) < 1e-2  # bf16 output; the fp32 path is checked in test_gqa_gpu


def test_host_buffer_step_equals_device_step(cuda):
    cfg = HybridConfig(batch=4, ctx=300, steps=3, seed=11)
    a, b = HybridDecoder(cfg), HybridDecoder(cfg)
    hin = [t.cpu().pin_memory() for t in b.step_inputs()]
    hout = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in b.step_outputs()]
    for _ in range(2):
        a.step()
        b.step_host(hin, hout)
    torch.cuda.synchronize()
    for x, y in zip(a.step_outputs(), hout):
        assert torch.equal(x.cpu(), y)
    assert torch.equal(a.S, b.S) and torch.equal(a.kc, b.kc)
