"""Kernel counts the GQA wrappers report (they feed bench.py's gpu_launches): derived from
the library's own split choice (vx27_gqa_decode_workspace_size and
vx27_gqa_partial_workspace_size), so no GPU is needed."""
from vx27_b200 import ops

NQ, NKV, HD = 24, 4, 256
REC = lambda B: B * NQ * (HD + 2) * 4


def test_config2_decode_is_one_launch():
    # 256 sequences x 4 KV heads fill the SMs: one split, the split kernel writes out
    ws = ops.gqa_workspace_bytes(256, NQ, NKV, HD, 4160)
    assert ws == REC(256)
    assert ops.gqa_decode_launches(256, NQ, NKV, HD, 4160, ws) == 1


def test_long_single_sequence_splits_and_combines():
    ws = ops.gqa_workspace_bytes(1, NQ, NKV, HD, 8192)
    assert ws > REC(1)  # several splits
    assert ops.gqa_decode_launches(1, NQ, NKV, HD, 8192, ws) == 2
    # a workspace of one record caps the library's choice at one split
    assert ops.gqa_decode_launches(1, NQ, NKV, HD, 8192, REC(1)) == 1
    # an explicit split count wins
    assert ops.gqa_decode_launches(1, NQ, NKV, HD, 8192, ws, n_splits=1) == 1
    assert ops.gqa_decode_launches(1, NQ, NKV, HD, 8192, ws, n_splits=3) == 2


def test_partial_launches():
    span = 131072
    ws = ops.gqa_partial_workspace_bytes(1, NQ, NKV, HD, span)
    assert ws > 0
    assert ops.gqa_partial_launches(1, NQ, NKV, HD, span, ws) == 2
    assert ops.gqa_partial_launches(1, NQ, NKV, HD, span, 0) == 1


def test_plan_kernel_choice():
    # config 1 (one sequence, 4 KV heads): the tensor-core kernel, several splits + combine
    ws = ops.gqa_workspace_bytes(1, NQ, NKV, HD, 8192)
    kind, n, launches = ops.gqa_decode_plan(1, NQ, NKV, HD, 8192, ws)
    assert kind == "tc" and n > 1 and launches == 2
    # config 2 (256 sequences): the tensor-core kernel, one split
    kind, n, launches = ops.gqa_decode_plan(256, NQ, NKV, HD, 4160, REC(256))
    assert (kind, n, launches) == ("tc", 1, 1)
    # the CUDA-core kernel only when asked for; its own split count, capped by the workspace
    kind, n, launches = ops.gqa_decode_plan(1, NQ, NKV, HD, 8192, 1 << 30, kernel="cc")
    assert kind == "cc" and n > 1 and launches == 2
    assert ops.gqa_decode_plan(1, NQ, NKV, HD, 8192, REC(1), kernel="cc")[1:] == (1, 1)
    assert ops.gqa_decode_plan(256, NQ, NKV, HD, 4160, REC(256), kernel="cc")[0] == "cc"
