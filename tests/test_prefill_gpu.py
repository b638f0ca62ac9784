"""K4 (vx27_gqa_prefill, causal gated GQA prefill on the tensor cores) against the CPU
oracle (orc_gqa_prefill_rows: the per-token decode path of src/vx27_qfwd.c:339-371 applied
to every prompt position). Tolerance: 2e-2 relative (max-abs error over max-abs value);
q and p enter the tensor cores as bf16."""
import numpy as np
import pytest
import torch

from gpu_util import dev, host, rel_err
from vx27_b200 import ops

pytestmark = pytest.mark.gpu
NQ, NKV, HD = 24, 4, 256
REL_TOL = 2e-2


def make(orc, seed, T):
    g = lambda n, s, m=0.0, sd=1.0, b=True: orc.normal(n, seed, s, m, sd, bf16=b)
    return dict(q=g(T * NQ * HD, 1), k=g(T * NKV * HD, 2), v=g(T * NKV * HD, 3),
                gate=g(T * NQ * HD, 4), qw=g(HD, 5, 1.0, 0.02, False),
                kw=g(HD, 6, 1.0, 0.02, False))


def oracle_rows(orc, x, T, rows):
    rows = np.asarray(rows, np.int32)
    out = np.zeros(len(rows) * NQ * HD, np.float32)
    orc.lib().orc_gqa_prefill_rows(orc.P(x["q"]), orc.P(x["k"]), orc.P(x["v"]), orc.P(x["gate"]),
                                   orc.P(x["qw"]), orc.P(x["kw"]), T, NQ, NKV, HD, 64, 1e7, 1e-6,
                                   orc.P(rows), len(rows), orc.P(out), orc.F_ACT_BF16)
    return out.reshape(len(rows), NQ, HD)


def gpu_prefill(x, T, cap, rope, chunks=None, out_bf16=False):
    """Prefill in one call, or in consecutive chunks (p0 > 0 continues the cache)."""
    q = dev(x["q"], True).view(T, NQ, HD)
    k = dev(x["k"], True).view(T, NKV, HD)
    v = dev(x["v"], True).view(T, NKV, HD)
    gate = dev(x["gate"], True).view(T, NQ, HD)
    kc = torch.full((NKV, cap, HD), float("nan"), dtype=torch.bfloat16, device="cuda")
    vc = torch.full((NKV, cap, HD), float("nan"), dtype=torch.bfloat16, device="cuda")
    out = torch.empty(T, NQ, HD, dtype=torch.bfloat16 if out_bf16 else torch.float32,
                      device="cuda")
    bounds = chunks or [0, T]
    for a, b in zip(bounds, bounds[1:]):
        ops.gqa_prefill(q[a:b], k[a:b], v[a:b], gate[a:b], dev(x["qw"]), dev(x["kw"]), rope,
                        kc, vc, out[a:b], p0=a)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    return out.float().cpu().numpy(), kc, vc


@pytest.fixture(scope="module")
def rope(cuda):
    return ops.rope_table(40000)


@pytest.mark.parametrize("T", [1, 64, 200, 300])
def test_small_prompts_all_rows(cuda, orc, rope, T):
    x = make(orc, 10 + T, T)
    out, _, _ = gpu_prefill(x, T, T + 64, rope)
    ref = oracle_rows(orc, x, T, range(T))
    assert rel_err(out.reshape(-1), ref.reshape(-1)) < REL_TOL


def test_chunked_continuation_equals_oracle(cuda, orc, rope):
    """Prefill in three calls at p0 = 0, 130, 257 (cache carried between calls) == one pass."""
    T = 400
    x = make(orc, 99, T)
    out, kc, vc = gpu_prefill(x, T, 512, rope, chunks=[0, 130, 257, 400])
    ref = oracle_rows(orc, x, T, range(T))
    assert rel_err(out.reshape(-1), ref.reshape(-1)) < REL_TOL
    # the cache holds finite values past the prompt up to the next multiple of 64
    assert torch.isfinite(kc[:, :448].float()).all() and torch.isfinite(vc[:, :448].float()).all()


def test_config4_gqa_sampled_rows(cuda, orc, rope):
    """Config 4 GQA path: T = 32768, seed 4; rows first, last, tile edges and random."""
    T = 32768
    x = make(orc, 4, T)
    out, _, _ = gpu_prefill(x, T, T, rope, out_bf16=True)
    rows = [0, 1, 63, 64, 127, 128, 4095, 17001, T - 129, T - 1]
    ref = oracle_rows(orc, x, T, rows)
    err = rel_err(out[rows].reshape(-1), ref.reshape(-1))
    print(f"config4 GQA sampled rows rel err {err:.3e}")
    assert err < REL_TOL
