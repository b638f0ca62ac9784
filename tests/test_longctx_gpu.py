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
