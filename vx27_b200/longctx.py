"""Long-context gated GQA decode (config 3): 16 full-attention layers, 24 Q / 4 KV heads of
256, BF16 KV cache at 262144 positions, query at position 262143.

* Sequence-sharded (3a): each rank holds whole caches for its sequences and runs the
  split-KV decode locally (vx27_gqa_append + vx27_gqa_decode_batch per layer).
* KV-sharded (3b): one sequence, rank r holds cache positions shard_range(P, N, r) of
  every layer; per step every rank prepares q (vx27_gqa_append; the store lands only on
  the rank that owns the new position), computes one partial record per layer
  (vx27_gqa_partial), all ranks all-gather the 16 records in one collective, and each
  rank merges them (vx27_gqa_combine).
Seeded synthetic K/V are generated so that a shard's contents equal its slice of the
whole cache (same generator stream, element offset), so results do not depend on N.
"""
from __future__ import annotations

import torch

from . import ops
from .dist import gather_records, shard_range

NQ, NKV, HD, ROPE = 24, 4, 256, 64


class LongContextGQA:
    def __init__(self, batch: int, ctx: int = 262144, layers: int = 16, rank: int = 0,
                 world: int = 1, split_kv: bool = False, seed: int = 3, device="cuda",
                 seq_offset: int = 0):
        self.B, self.P, self.layers = batch, ctx, layers
        self.rank, self.world, self.split_kv = rank, world, split_kv
        self.begin, self.end = shard_range(ctx, world, rank) if split_kv else (0, ctx)
        self.cap = self.end - self.begin
        self.dev = torch.device(device)
        bf, kw = torch.bfloat16, dict(device=self.dev)
        self.kc = torch.empty(layers, batch, NKV, self.cap, HD, dtype=bf, **kw)
        self.vc = torch.empty(layers, batch, NKV, self.cap, HD, dtype=bf, **kw)
        self.q_in = torch.empty(layers, batch, NQ, HD, dtype=bf, **kw)
        self.k_in = torch.empty(layers, batch, NKV, HD, dtype=bf, **kw)
        self.v_in = torch.empty(layers, batch, NKV, HD, dtype=bf, **kw)
        self.gate = torch.empty(layers, batch, NQ, HD, dtype=bf, **kw)
        self.q_norm_w = torch.empty(layers, HD, **kw)
        self.k_norm_w = torch.empty(layers, HD, **kw)
        self.out = torch.empty(layers, batch, NQ, HD, dtype=bf, **kw)
        self.qn = torch.empty(layers, batch, NQ, HD, **kw)
        self.pos = torch.full((batch,), ctx - 1, dtype=torch.int32, **kw)
        self.rope = ops.rope_table(ctx, ROPE, 1e7, 1.0, device=self.dev)
        rec = batch * NQ * (HD + 2)
        self.rec = rec
        self.parts = torch.empty(layers, rec, **kw)
        ws = max(ops.gqa_workspace_bytes(batch, NQ, NKV, HD, self.cap),
                 ops.gqa_partial_workspace_bytes(batch, NQ, NKV, HD, self.cap))
        self.ws = torch.empty(max(ws // 4, 1), **kw)
        # seeded contents: the global cache is [layer][seq][kvh][P][HD]; this rank's rows
        # are positions [begin, end) of sequences seq_offset .. seq_offset + batch - 1
        for l in range(layers):
            for b in range(batch):
                for h in range(NKV):
                    g = ((l * 1_000_003 + (seq_offset + b)) * NKV + h) * ctx + self.begin
                    ops.fill_normal(self.kc[l, b, h], seed, 1, offset=g * HD)
                    ops.fill_normal(self.vc[l, b, h], seed, 2, offset=g * HD)
        for n, t in enumerate((self.q_in, self.k_in, self.v_in, self.gate)):
            ops.fill_normal(t, seed, 10 + n, offset=seq_offset * t[0].numel())
        ops.fill_normal(self.q_norm_w, seed, 20, 1.0, 0.02)
        ops.fill_normal(self.k_norm_w, seed, 21, 1.0, 0.02)
        torch.cuda.synchronize(self.dev)
        ops.device_status()

    def kv_bytes(self) -> int:
        return self.kc.numel() * 2 * 2

    def step(self, stream=None) -> int:
        """One decode step of every layer; returns kernels launched."""
        n = 0
        if not self.split_kv:
            for l in range(self.layers):
                ops.gqa_append(self.q_in[l], self.k_in[l], self.v_in[l], self.q_norm_w[l],
                               self.k_norm_w[l], self.rope, self.pos, self.kc[l], self.vc[l],
                               self.qn[l], stream=stream)
                n += 1 + ops.gqa_decode_batch(self.qn[l], self.gate[l], self.kc[l], self.vc[l],
                                              self.pos, self.out[l], self.ws, stream=stream)
            return n
        n += self.local_partials(stream)
        gathered = gather_records(self.parts, self.world)  # [world, layers*rec]
        return n + self.combine(gathered, stream)

    def local_partials(self, stream=None) -> int:
        """KV-sharded step, local half: q for every layer (the new token's K/V land on the
        shard owning position P-1) and this shard's partial record per layer."""
        n = 0
        for l in range(self.layers):
            ops.gqa_append(self.q_in[l], self.k_in[l], self.v_in[l], self.q_norm_w[l],
                           self.k_norm_w[l], self.rope, self.pos, self.kc[l], self.vc[l],
                           self.qn[l], slot_base=self.begin, stream=stream)
            n += 1 + ops.gqa_partial(self.qn[l], self.kc[l], self.vc[l], 0, self.cap,
                                     self.parts[l], self.ws, stream=stream)
        return n

    def combine(self, gathered, stream=None) -> int:
        """Merges the all-gathered records ([world, layers*rec]) into self.out."""
        flat = gathered.reshape(-1)
        world = gathered.shape[0]
        for l in range(self.layers):
            ops.gqa_combine(flat[l * self.rec:], world, self.gate[l], self.out[l],
                            part_stride=self.layers * self.rec, stream=stream)
        return self.layers
