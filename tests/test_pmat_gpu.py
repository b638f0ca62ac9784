"""K5 packed-weight matvec on the device (vx27_pmat_batch_dev) against the oracle
restatement of src/vx27_pmat.c (itself pinned bit-for-bit to the reference in
tests/test_pmat_pins.py): bit-identical outputs for F32, Q8_K and BP3_128 rows, token
counts 1..19 (passes of 1, 2, 4 and 8 tokens), ragged row counts, the projection shapes
of the model, special group scales and inputs, several projections in one launch."""
import numpy as np
import pytest
import torch

import oracle.oracle as O
from vx27_b200 import ops

pytestmark = pytest.mark.gpu


def run(W, dtype, x, rows, cols, B):
    Wd = torch.from_numpy(W).cuda()
    xd = torch.from_numpy(x.reshape(B, cols)).cuda()
    yd = torch.full((B, rows), float("nan"), device="cuda")
    ops.pmat_batch(Wd, dtype, xd, yd, rows, cols)
    torch.cuda.synchronize()
    return yd.cpu().numpy().reshape(-1)


@pytest.mark.parametrize("dtype", [O.PMAT_F32, O.PMAT_Q8K, O.PMAT_BP3])
@pytest.mark.parametrize("B", [1, 2, 3, 5, 8, 11, 19])
def test_bit_identical_to_reference_arithmetic(cuda, dtype, B):
    rows, cols = 83, 1280 if dtype == O.PMAT_Q8K else 1152
    W = O.packed_weights(dtype, rows, cols, 200 + dtype)
    x = np.random.default_rng(B).standard_normal(B * cols).astype(np.float32)
    y = run(W, dtype, x, rows, cols, B)
    ref = O.pmat_batch(W, dtype, x, rows, cols, B)
    assert np.array_equal(y.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("rows,cols,B", [(48, 5120, 1), (1024, 5120, 3), (5120, 6144, 1)])
def test_projection_shapes_bp3(cuda, rows, cols, B):
    # in_proj_a/b (48 x 5120), k/v_proj (1024 x 5120), out_proj / o_proj (5120 x 6144)
    W = O.packed_weights(O.PMAT_BP3, rows, cols, rows + cols)
    x = np.random.default_rng(3).standard_normal(B * cols).astype(np.float32)
    y = run(W, O.PMAT_BP3, x, rows, cols, B)
    ref = O.pmat_batch(W, O.PMAT_BP3, x, rows, cols, B)
    assert np.array_equal(y.view(np.uint32), ref.view(np.uint32))


def same_bits(y, ref):
    """Bit-identical, except that a NaN only has to be a NaN (the payload of a NaN differs
    between host and device arithmetic)."""
    yn, rn = np.isnan(y), np.isnan(ref)
    return np.array_equal(yn, rn) and np.array_equal(y[~yn].view(np.uint32),
                                                       ref[~rn].view(np.uint32))


SPECIAL_SCALES = np.array([0x0000, 0x8000, 0xA51F, 0x7BFF, 0xFBFF, 0x8001, 0x83FF, 0x0001,
                           0x7C00, 0xFC00, 0x7E00], np.uint16)  # +-0, -0.02, +-65504,
# subnormals (the reference's exponent-1 mapping), +-inf, NaN


@pytest.mark.parametrize("B", [1, 3, 8])
def test_bp3_special_scales_and_inputs(cuda, B):
    """Zero, negative, largest, subnormal, infinite and NaN group scales, and inputs with
    zeros of both signs and subnormal values."""
    rows, cols = 120, 1152
    g = O.packed_weights(O.PMAT_BP3, rows, cols, 77).reshape(-1, 52)
    rng = np.random.default_rng(78)
    pick = rng.random(len(g)) < 0.15
    g[pick, 48:50] = rng.choice(SPECIAL_SCALES, int(pick.sum())).view(np.uint8).reshape(-1, 2)
    W = g.reshape(-1)
    x = rng.standard_normal(B * cols).astype(np.float32)
    x[rng.random(x.size) < 0.05] = 0.0
    x[rng.random(x.size) < 0.05] = -0.0
    x[rng.random(x.size) < 0.05] = np.float32(1e-40) * rng.choice([-1, 1])
    y = run(W, O.PMAT_BP3, x, rows, cols, B)
    ref = O.pmat_batch(W, O.PMAT_BP3, x, rows, cols, B)
    assert np.isfinite(ref).sum() > rows * B // 3  # most rows still finite
    assert same_bits(y, ref)


@pytest.mark.parametrize("dtype", [O.PMAT_F32, O.PMAT_Q8K, O.PMAT_BP3])
@pytest.mark.parametrize("B", [1, 5])
def test_grouped_projections(cuda, dtype, B):
    """Up to four projections of one input in one launch (vx27_pmat_multi_dev), ragged row
    counts: each output equals its own reference matvec."""
    cols = 1280 if dtype == O.PMAT_Q8K else 1152
    rows = [83, 48, 200, 16]
    x = np.random.default_rng(B + 40).standard_normal(B * cols).astype(np.float32)
    Ws = [O.packed_weights(dtype, r, cols, 300 + i) for i, r in enumerate(rows)]
    xd = torch.from_numpy(x.reshape(B, cols)).cuda()
    ys = [torch.full((B, r), float("nan"), device="cuda") for r in rows]
    ops.pmat_multi([torch.from_numpy(W).cuda() for W in Ws], dtype, xd, ys, rows, cols)
    torch.cuda.synchronize()
    for W, r, yd in zip(Ws, rows, ys):
        ref = O.pmat_batch(W, dtype, x, r, cols, B)
        assert np.array_equal(yd.cpu().numpy().reshape(-1).view(np.uint32), ref.view(np.uint32))
    with pytest.raises(ops.Vx27Error):  # five projections: more than one launch serves
        ops.pmat_multi([torch.from_numpy(Ws[0]).cuda()] * 5, dtype, xd, [ys[0]] * 5,
                       [rows[0]] * 5, cols)


def test_bad_arguments_rejected(cuda):
    W = torch.zeros(1000, dtype=torch.uint8, device="cuda")
    x = torch.zeros(1, 200, device="cuda")
    y = torch.zeros(1, 4, device="cuda")
    with pytest.raises(ops.Vx27Error):   # 200 columns: not whole BP3 groups
        ops.pmat_batch(W, O.PMAT_BP3, x, y, 4, 200)
    with pytest.raises(ops.Vx27Error):   # unknown format
        ops.pmat_batch(W, 3, x, y, 4, 200)
