"""The device gate mapping against the contract function vx27_deltanet_gate_params.

The reference fixes the gates bit for bit (src/vx27_deltanet.c:58-69, tested with == in
tests/test_deltanet_exact.c:44-57). The host entry point vx27_deltanet_gate_params
reproduces them exactly (the CPU tests pin it). The batched decode and prefill kernels
evaluate the same formula on the device, in double with CUDA's exp/log; this test exports
those device gates (vx27_deltanet_gate_params_dev) and measures them against the host
bits on the reference's six pins, 200,000 random cases across the softplus regimes, and
every bf16 logit below 700 in magnitude at config 2's heads:
  * the double beta and g_log are NOT the host's bits on every input: CUDA's and the C
    library's exp/log each round a few percent of results differently (measured on a
    B200: 2.8% of beta and 6.9% of g_log values differ in the random set, by 1-2 ulp;
    in softplus's range where log(1 + e^x) cancels, a 1-ulp difference of 1 + e^x is
    a few thousand ulp of the result, 8e-13 relative). The test bounds the relative
    difference and the rate and prints both;
  * the fp32 beta and decay = exp(g_log) that the kernels' update uses are identical to
    the host values rounded the same way, on every case.
Bit-exact double gates on the device path come from VX27_F_GATES_F64 (host-computed
gates fed to the kernels)."""
import ctypes as C
import math

import numpy as np
import pytest
import torch

from gpu_util import dev, host
from vx27_b200 import ops
from vx27_b200._lib import check, errbuf, load

pytestmark = pytest.mark.gpu
PINS = [(0.1, 0.5, -0.3, 1.0), (3.0, -1.2, 2.0, 1.0), (-25.0, 0.0, 0.0, 1.0),
        (25.0, 2.0, -2.0, 1.0), (0.0, -5.0, 5.0, -3.0), (-30.0, 1.0, 30.0, 30.0)]


def _device_gates(a, b, A_log, dt, nv, bf16):
    n = a.shape[0]
    out = [torch.empty(n, dtype=torch.float64, device="cuda"),
           torch.empty(n, dtype=torch.float64, device="cuda"),
           torch.empty(n, device="cuda"), torch.empty(n, device="cuda")]
    da, db = dev(a, bf16), dev(b, bf16)
    dA, dd = dev(A_log), dev(dt)
    p = lambda t: C.c_void_p(t.data_ptr())
    e = errbuf()
    check(load().vx27_deltanet_gate_params_dev(p(da), p(db), p(dA), p(dd), *map(p, out), n, nv,
                                               ops.F_ACT_BF16 if bf16 else 0, None, e, 512), e)
    torch.cuda.synchronize()
    return [host(t) for t in out]


def _host_gates(a, b, A_log, dt, nv):
    """vx27_deltanet_gate_params per item (the library's host entry point, which the CPU
    tests pin to the reference) and the fp32 values the kernels derive from it."""
    f = load().vx27_deltanet_gate_params
    n = a.shape[0]
    be, g = np.empty(n), np.empty(n)
    x, y = C.c_double(), C.c_double()
    for i in range(n):
        f(float(a[i]), float(A_log[i % nv]), float(b[i]), float(dt[i % nv]), C.byref(x),
          C.byref(y))
        be[i], g[i] = x.value, y.value
    decay = np.array([math.exp(v) for v in g]).astype(np.float32)  # the C library's exp
    return be, g, be.astype(np.float32), decay


def _ulps(x, y):
    xi, yi = x.view(np.int64), y.view(np.int64)
    same_sign = (xi < 0) == (yi < 0)
    assert same_sign.all()
    return np.abs(xi - yi)


def _compare(name, d, h):
    (bd, gd, bfd, dfd), (bh, gh, bfh, dfh) = d, h
    ub, ug = _ulps(bd, bh), _ulps(gd, gh)
    n = bd.shape[0]
    rate = (np.count_nonzero(ub) + np.count_nonzero(ug)) / (2 * n)
    rel = max(float(np.max(np.abs(bd - bh) / np.abs(bh))),
              float(np.max(np.abs(gd - gh) / np.maximum(np.abs(gh), 1e-300))))
    near = np.percentile(np.maximum(ub, ug), 99.9)
    print(f"{name}: {n} cases, double beta/g_log differ in {np.count_nonzero(ub)}/"
          f"{np.count_nonzero(ug)} ({100 * rate:.3f}%), 99.9th percentile {near:.0f} ulp, "
          f"max {max(ub.max(), ug.max())} ulp, max relative {rel:.2e}")
    assert rel < 1e-11
    assert near <= 8
    assert rate < 0.1
    assert np.array_equal(bfd.view(np.uint32), bfh.view(np.uint32)), f"{name}: fp32 beta"
    assert np.array_equal(dfd.view(np.uint32), dfh.view(np.uint32)), f"{name}: fp32 decay"
    return rate


def test_device_gates_on_the_reference_pins(cuda):
    # fp32 activations: the pins rounded to float are what the device sees, and the host
    # function is given the same values
    v = np.array(PINS, np.float64).astype(np.float32)
    a, Al, b, dt = (np.ascontiguousarray(v[:, i]) for i in range(4))
    n = len(PINS)
    d = _device_gates(a, b, Al, dt, n, False)
    h = _host_gates(a, b, Al, dt, n)
    _compare("pins", d, h)


def test_device_gates_random(cuda, orc):
    n = 200_000
    a = orc.normal(n, 41, 1, 0.0, 8.0)           # all three softplus regimes
    b = orc.normal(n, 41, 2, 0.0, 4.0)
    Al = np.log(orc.uniform(n, 41, 3, 1.0, 16.0)).astype(np.float32)
    dt = orc.normal(n, 41, 4, 0.0, 0.1)
    d = _device_gates(a, b, Al, dt, n, False)
    h = _host_gates(a, b, Al, dt, n)
    _compare("random", d, h)


def test_device_gates_every_bf16_logit(cuda, orc):
    """b over every bf16 value below 700 in magnitude, a over the same grid shifted, at
    config 2's 16 heads
    (A_log = log U[1,16], dt_bias ~ N(0, 0.1))."""
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    f = (bits.astype(np.uint32) << 16).view(np.float32)
    # below 700 in magnitude e^x stays a normal double (further out both sides reach the
    # subnormal range, where a 1-ulp exp difference times exp(A_log) is several ulps)
    keep = np.isfinite(f) & (np.abs(f) < 700)
    b = np.ascontiguousarray(bits[keep])
    a = np.ascontiguousarray(np.roll(b, 977))
    nv = 16
    Al = np.log(orc.uniform(nv, 2, 6, 1.0, 16.0)).astype(np.float32)
    dt = orc.normal(nv, 2, 7, 0.0, 0.1)
    d = _device_gates(a, b, Al, dt, nv, True)
    fa, fb = ((x.astype(np.uint32) << 16).view(np.float32) for x in (a, b))
    h = _host_gates(fa, fb, Al, dt, nv)
    _compare("bf16 grid", d, h)
