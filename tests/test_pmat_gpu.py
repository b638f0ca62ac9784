"""K5 packed-weight matvec on the device (vx27_pmat_batch_dev) against the oracle
restatement of src/vx27_pmat.c (itself pinned bit-for-bit to the reference in
tests/test_pmat_pins.py): bit-identical outputs for F32, Q8_K and BP3_128 rows, token
counts 1..19 (passes of 1, 2, 4 and 8 tokens), ragged row counts, the projection shapes
of the model."""
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


def test_bad_arguments_rejected(cuda):
    W = torch.zeros(1000, dtype=torch.uint8, device="cuda")
    x = torch.zeros(1, 200, device="cuda")
    y = torch.zeros(1, 4, device="cuda")
    with pytest.raises(ops.Vx27Error):   # 200 columns: not whole BP3 groups
        ops.pmat_batch(W, O.PMAT_BP3, x, y, 4, 200)
    with pytest.raises(ops.Vx27Error):   # unknown format
        ops.pmat_batch(W, 3, x, y, 4, 200)
