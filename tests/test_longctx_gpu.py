"""Config 3 drivers (vx27_b200.longctx) on one GPU: the KV-sharded data flow (each shard's
partial records, the records of all shards merged) equals the sequence-sharded decode of
the whole cache, for shard boundaries that do not fall on tile edges."""
import pytest
import torch

from gpu_util import host, rel_err
from vx27_b200.longctx import LongContextGQA

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world", [2, 3])
def test_kv_sharded_equals_whole_cache(cuda, world):
    P, layers = 1000, 2
    whole = LongContextGQA(1, ctx=P, layers=layers)
    whole.step()
    shards = [LongContextGQA(1, ctx=P, layers=layers, rank=r, world=world, split_kv=True)
              for r in range(world)]
    for s in shards:
        s.local_partials()
    gathered = torch.stack([s.parts.reshape(-1) for s in shards])
    shards[0].combine(gathered)
    torch.cuda.synchronize()
    # both outputs are bf16 roundings of nearly equal fp32 values
    assert rel_err(host(shards[0].out.float()).reshape(-1),
                   host(whole.out.float()).reshape(-1)) < 1e-2
    # the new token's K landed only on the shard that owns position P-1
    last = shards[-1]
    assert torch.equal(last.kc[:, :, :, last.cap - 1], whole.kc[:, :, :, P - 1])


def test_long_range_partial_split_and_merged(cuda):
    """A 3b-sized shard range is split across CTAs and merged (workspace path)."""
    P = 20000
    whole = LongContextGQA(1, ctx=P, layers=1)
    whole.step()
    one = LongContextGQA(1, ctx=P, layers=1, rank=0, world=1, split_kv=True)
    one.local_partials()
    one.combine(one.parts.reshape(1, -1))
    torch.cuda.synchronize()
    assert rel_err(host(one.out.float()).reshape(-1), host(whole.out.float()).reshape(-1)) < 1e-2


def test_stacked_layers_equal_per_layer_calls(cuda):
    """One step with the layers stacked as the batch (grouped norm weights, one append and
    one decode for all layers) against each layer run on its own: the K/V rows it appends
    are the same bits, the outputs agree within the decode's tolerance (the split counts
    differ)."""
    from vx27_b200 import ops
    from vx27_b200.longctx import HD, NKV, NQ
    P, layers = 3000, 3
    a = LongContextGQA(2, ctx=P, layers=layers, seed=9)
    b = LongContextGQA(2, ctx=P, layers=layers, seed=9)
    a.step()
    for l in range(layers):
        ops.gqa_append(b.q_in[l], b.k_in[l], b.v_in[l], b.q_norm_w[l], b.k_norm_w[l], b.rope,
                       b.pos, b.kc[l], b.vc[l], b.qn[l])
        ops.gqa_decode_batch(b.qn[l], b.gate[l], b.kc[l], b.vc[l], b.pos, b.out[l], b.ws)
    torch.cuda.synchronize()
    assert torch.equal(a.kc[:, :, :, P - 1], b.kc[:, :, :, P - 1])
    assert torch.equal(a.vc[:, :, :, P - 1], b.vc[:, :, :, P - 1])
    assert torch.equal(a.qn, b.qn)
    assert rel_err(host(a.out.float()).reshape(-1), host(b.out.float()).reshape(-1)) < 1e-2
    assert ops.device_status() == 0
