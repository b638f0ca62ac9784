"""Pins of the packed-weight matvec restatement (oracle/vx27_oracle.c, orc_pmat_batch)
against the reference's own src/vx27_pmat.c, compiled unmodified into
oracle/_ref/libvx27ref_pmat.so: bit-identical outputs for F32, Q8_K and BP3_128 rows,
single-vector (vx27_pmat) and batched (vx27_pmat_batch) entry points."""
import ctypes as C
import os

import numpy as np
import pytest

import oracle.oracle as O


@pytest.fixture(scope="module")
def refpmat():
    if not os.path.exists(O.REF_PMAT_LIB) and not O.build_ref():
        pytest.skip("reference sources unavailable: oracle/_ref not built")
    if not os.path.exists(O.REF_PMAT_LIB):
        pytest.skip("oracle/_ref/libvx27ref_pmat.so not built")
    lib = C.CDLL(O.REF_PMAT_LIB)
    lib.vx27_pmat.argtypes = [C.c_void_p, C.c_void_p, C.c_uint32, C.c_void_p, C.c_void_p,
                              C.c_int, C.c_int]
    lib.vx27_pmat_batch.argtypes = [C.c_void_p, C.c_void_p, C.c_uint32, C.c_void_p,
                                    C.c_void_p, C.c_int, C.c_int, C.c_int]
    return lib


@pytest.mark.parametrize("dtype", [O.PMAT_F32, O.PMAT_Q8K, O.PMAT_BP3])
@pytest.mark.parametrize("B", [1, 3, 8])
def test_restatement_equals_reference(refpmat, dtype, B):
    rows, cols = 37, 1024
    W = O.packed_weights(dtype, rows, cols, 100 + dtype)
    x = np.random.default_rng(7 + B).standard_normal(B * cols).astype(np.float32)
    y_orc = O.pmat_batch(W, dtype, x, rows, cols, B)
    y_ref = np.empty(B * rows, np.float32)
    if B == 1:
        refpmat.vx27_pmat(None, O.P(W), dtype, O.P(x), O.P(y_ref), rows, cols)
    else:
        refpmat.vx27_pmat_batch(None, O.P(W), dtype, O.P(x), O.P(y_ref), rows, cols, B)
    assert np.array_equal(y_orc.view(np.uint32), y_ref.view(np.uint32))
    # and the batched reference equals B single calls (the reference's own claim)
    if B > 1:
        y1 = np.empty(rows, np.float32)
        for b in range(B):
            refpmat.vx27_pmat(None, O.P(W), dtype, O.P(x[b * cols:(b + 1) * cols].copy()),
                              O.P(y1), rows, cols)
            assert np.array_equal(y1.view(np.uint32), y_ref[b * rows:(b + 1) * rows].view(np.uint32))


def test_bp3_scale_conversion(refpmat):
    # every fp16 bit pattern: normal values convert exactly, subnormals with the
    # reference's exponent-1 mapping, inf/nan kept
    h = np.arange(65536, dtype=np.uint16)
    f = np.array([O.lib().orc_bp3_scale(int(v)) for v in h[::97]], np.float32)
    ref = h[::97].view(np.float16).astype(np.float32)
    normal = ((h[::97] >> 10) & 0x1F) != 0
    finite = ((h[::97] >> 10) & 0x1F) != 31
    m = normal & finite
    assert np.array_equal(f[m], ref[m])
    sub = (~normal) & ((h[::97] & 0x3FF) != 0)
    assert np.all(np.abs(f[sub]) >= 2.0 ** -14)  # mapped with exponent 1, not scaled down


@pytest.mark.parametrize("B", [1, 4])
def test_bp3_special_scales_and_inputs(refpmat, B):
    # zero, negative, largest, subnormal, infinite and NaN group scales; inputs with zeros
    # of both signs and subnormals: bit-identical (a NaN only has to be a NaN)
    rows, cols = 40, 1024
    g = O.packed_weights(O.PMAT_BP3, rows, cols, 55).reshape(-1, 52)
    rng = np.random.default_rng(56)
    specials = np.array([0x0000, 0x8000, 0xA51F, 0x7BFF, 0xFBFF, 0x8001, 0x83FF, 0x0001,
                         0x7C00, 0xFC00, 0x7E00], np.uint16)
    pick = rng.random(len(g)) < 0.15
    g[pick, 48:50] = rng.choice(specials, int(pick.sum())).view(np.uint8).reshape(-1, 2)
    W = g.reshape(-1)
    x = rng.standard_normal(B * cols).astype(np.float32)
    x[rng.random(x.size) < 0.05] = -0.0
    x[rng.random(x.size) < 0.05] = np.float32(-1e-40)
    y_orc = O.pmat_batch(W, O.PMAT_BP3, x, rows, cols, B)
    y_ref = np.empty(B * rows, np.float32)
    if B == 1:
        refpmat.vx27_pmat(None, O.P(W), O.PMAT_BP3, O.P(x), O.P(y_ref), rows, cols)
    else:
        refpmat.vx27_pmat_batch(None, O.P(W), O.PMAT_BP3, O.P(x), O.P(y_ref), rows, cols, B)
    on, rn = np.isnan(y_orc), np.isnan(y_ref)
    assert np.array_equal(on, rn)
    assert np.array_equal(y_orc[~on].view(np.uint32), y_ref[~rn].view(np.uint32))
    assert np.isfinite(y_ref).sum() > rows * B // 3


@pytest.mark.parametrize("dtype", [O.PMAT_F32, O.PMAT_Q8K])
def test_special_values_other_formats(refpmat, dtype):
    # Q8_K block scales d of zero, negative, huge, infinite and NaN; F32 weights with the
    # same specials; inputs with signed zeros and subnormals: bit-identical (NaN as NaN)
    rows, cols, B = 24, 1024, 3
    W = O.packed_weights(dtype, rows, cols, 66).copy()
    rng = np.random.default_rng(67)
    specials = np.array([0.0, -0.0, -1e-3, 3e38, -3e38, np.inf, -np.inf, np.nan], np.float32)
    if dtype == O.PMAT_Q8K:
        blk = W.reshape(-1, 292)
        pick = rng.random(len(blk)) < 0.3
        d = rng.choice(specials, int(pick.sum())).astype(np.float32)
        blk[pick, 0:4] = d.view(np.uint8).reshape(-1, 4)
    else:
        w = W.view(np.float32)
        pick = rng.random(w.size) < 0.001
        w[pick] = rng.choice(specials, int(pick.sum()))
    x = rng.standard_normal(B * cols).astype(np.float32)
    x[rng.random(x.size) < 0.05] = -0.0
    x[rng.random(x.size) < 0.05] = np.float32(1e-40)
    y_orc = O.pmat_batch(W, dtype, x, rows, cols, B)
    y_ref = np.empty(B * rows, np.float32)
    refpmat.vx27_pmat_batch(None, O.P(W), dtype, O.P(x), O.P(y_ref), rows, cols, B)
    on, rn = np.isnan(y_orc), np.isnan(y_ref)
    assert np.array_equal(on, rn)
    assert np.array_equal(y_orc[~on].view(np.uint32), y_ref[~rn].view(np.uint32))
    assert np.isfinite(y_ref).sum() > rows * B // 4
