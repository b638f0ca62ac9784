"""The reference's own entry points on the GPU (host pointers, synchronous), against the
golden vectors the reference's sources produced. Bit-exact where the reference function
calls no libm routine; otherwise within the stated tolerance."""
import numpy as np
import pytest

from vx27_b200 import ops

pytestmark = pytest.mark.gpu


def test_update_retrieve_bit_exact(cuda, golden):
    for hd in (128, 8):
        k, v, q = golden[f"ur{hd}_k"], golden[f"ur{hd}_v"], golden[f"ur{hd}_q"]
        for name in ("ref", "tiled", "avx2"):
            S = golden[f"ur{hd}_S0"].copy()
            getattr(ops, f"vx27_deltanet_update_{name}")(S, k, v, 0.9, hd)
            assert np.array_equal(S, golden[f"ur{hd}_{name}_S"]), name
            o = np.zeros(hd, np.float32)
            getattr(ops, f"vx27_deltanet_retrieve_{name}")(S, q, o, hd)
            assert np.array_equal(o, golden[f"ur{hd}_{name}_o"]), name


def test_step_exact_bit_exact(cuda, golden):
    for hd in (128, 32, 8):
        S0 = golden[f"step{hd}_S0"]
        for t in range(S0.shape[0]):
            S = np.ascontiguousarray(S0[t]).copy()
            for s in range(6):
                o = np.zeros(hd, np.float32)
                ops.vx27_deltanet_step_exact(
                    S, np.ascontiguousarray(golden[f"step{hd}_q"][t, s]),
                    np.ascontiguousarray(golden[f"step{hd}_k"][t, s]),
                    np.ascontiguousarray(golden[f"step{hd}_v"][t, s]),
                    float(golden[f"step{hd}_beta"][t, s]), float(golden[f"step{hd}_g"][t, s]), o, hd)
                assert np.array_equal(o, golden[f"step{hd}_o"][t, s])
            assert np.array_equal(S, golden[f"step{hd}_S"][t])


def test_norms_bit_exact(cuda, golden):
    for n in (2, 128, 256, 5120):
        x, w = golden[f"norm{n}_x"], golden[f"norm{n}_w"]
        y = np.zeros(n, np.float32)
        ops.vx27_deltanet_l2norm(x, y, n)
        assert np.array_equal(y, golden[f"l2norm{n}"])
        ops.vx27_rmsnorm(x, w, y, n, 1e-6)
        assert np.array_equal(y, golden[f"rmsnorm{n}"])
    y = np.zeros(2, np.float32)
    ops.vx27_rmsnorm(np.array([3, 4], np.float32), np.ones(2, np.float32), y, 2, 0.0)
    assert np.array_equal(y, golden["rmsnorm_34"])


def test_rope_apply_bit_exact(cuda, golden):
    for n in range(len(golden["rope_pos"])):
        x = np.ascontiguousarray(golden["rope_x"][n]).copy()
        ops.vx27_rope_apply(x, 4, 256, 64, np.ascontiguousarray(golden["rope_cos"][n]),
                            np.ascontiguousarray(golden["rope_sin"][n]))
        assert np.array_equal(x, golden["rope_y"][n])


def test_conv1d(cuda, golden):
    """The weighted sum is bit-exact; SiLU uses a correctly rounded expf, which matches the
    C library's expf except where the latter misrounds (1 ulp)."""
    w, xs = golden["conv_w"], golden["conv_x"]
    st = np.zeros(w.size // 4 * 3, np.float32)
    exact = 0
    for t in range(xs.shape[0]):
        y = np.zeros(xs.shape[1], np.float32)
        ops.vx27_conv1d_step(st, np.ascontiguousarray(xs[t]), w, y, xs.shape[1], 1)
        ref = golden["conv_y"][t]
        assert np.abs(y - ref).max() <= 2 * np.spacing(np.abs(ref)).max()
        exact += int(np.array_equal(y, ref))
    assert np.array_equal(st, golden["conv_state"])
    assert exact >= xs.shape[0] - 1


def test_attn_1q(cuda, golden):
    for n in (1, 2, 5, 13):
        o = np.zeros(24 * 256, np.float32)
        ops.vx27_attn_1q(golden[f"attn{n}_q"], golden[f"attn{n}_k"], golden[f"attn{n}_v"], n, o)
        ref = golden[f"attn{n}_o"]
        assert np.abs(o - ref).max() <= 1e-6 * max(1.0, np.abs(ref).max())


def test_attn_1q_beyond_reference_limit(cuda, orc):
    """The reference caps n_pos at 1024 (static buffer); the GPU version does not."""
    n = 3000
    q = orc.normal(24 * 256, 11, 1)
    k = orc.normal(n * 4 * 256, 11, 2)
    v = orc.normal(n * 4 * 256, 11, 3)
    o = np.zeros(24 * 256, np.float32)
    ops.vx27_attn_1q(q, k, v, n, o)
    ref = np.zeros(24 * 256, np.float32)
    orc.lib().orc_attn_1q(orc.P(q), orc.P(k), orc.P(v), n, 24, 4, 256, orc.P(ref))
    assert np.abs(o - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max())
