"""Long-context gated GQA decode (config 3): 16 full-attention layers, 24 Q / 4 KV heads of
256, BF16 KV cache at 262144 positions, query at position 262143.

The layers of config 3 are independent attention calls, so one step treats the 16 layers
stacked as the batch: [layer][sequence] is one batch index of layers x B, with caches,
activations and outputs laid out [layer][B][...] and per-layer norm weights
(vx27_gqa_append_grouped). One call of each kernel then serves every layer, and the
persistent split-KV kernel streams all layers' caches in one launch.
* Sequence-sharded (3a): each rank holds whole caches for its sequences: one append and
  one split-KV decode (vx27_gqa_decode_batch) per step.
* KV-sharded (3b): one sequence, rank r holds cache positions shard_range(P, N, r) of
  every layer; per step every rank prepares q (the store lands only on the rank that
  owns the new position), computes one partial record covering every layer
  (vx27_gqa_partial), all ranks all-gather that record in one collective, and each rank
  merges the N records in one vx27_gqa_combine.
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
        LB = layers * batch  # the stacked batch of one step
        self.pos_lb = torch.full((LB,), ctx - 1, dtype=torch.int32, **kw)
        self.rope = ops.rope_table(ctx, ROPE, 1e7, 1.0, device=self.dev)
        rec = LB * NQ * (HD + 2)  # one partial record covers every layer
        self.rec = rec
        self.parts = torch.empty(rec, **kw)
        ws = max(ops.gqa_workspace_bytes(LB, NQ, NKV, HD, self.cap),
                 ops.gqa_partial_workspace_bytes(LB, NQ, NKV, HD, self.cap))
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

    def _stacked(self):
        """Views with layers x sequences as one batch index."""
        LB = self.layers * self.B
        return dict(q_in=self.q_in.view(LB, NQ, HD), k_in=self.k_in.view(LB, NKV, HD),
                    v_in=self.v_in.view(LB, NKV, HD), gate=self.gate.view(LB, NQ, HD),
                    out=self.out.view(LB, NQ, HD), qn=self.qn.view(LB, NQ, HD),
                    kc=self.kc.view(LB, NKV, self.cap, HD), vc=self.vc.view(LB, NKV, self.cap, HD))

    def step(self, stream=None) -> int:
        """One decode step of every layer; returns kernels launched."""
        if self.split_kv:
            n = self.local_partials(stream)
            gathered = gather_records(self.parts, self.world)  # [world, rec]
            return n + self.combine(gathered, stream)
        v = self._stacked()
        ops.gqa_append(v["q_in"], v["k_in"], v["v_in"], self.q_norm_w, self.k_norm_w, self.rope,
                       self.pos_lb, v["kc"], v["vc"], v["qn"], stream=stream)
        return 1 + ops.gqa_decode_batch(v["qn"], v["gate"], v["kc"], v["vc"], self.pos_lb,
                                        v["out"], self.ws, stream=stream)

    def local_partials(self, stream=None) -> int:
        """KV-sharded step, local half: q for every layer (the new token's K/V land on the
        shard owning position P-1) and this shard's partial record of every layer."""
        v = self._stacked()
        ops.gqa_append(v["q_in"], v["k_in"], v["v_in"], self.q_norm_w, self.k_norm_w, self.rope,
                       self.pos_lb, v["kc"], v["vc"], v["qn"], slot_base=self.begin,
                       stream=stream)
        return 1 + ops.gqa_partial(v["qn"], v["kc"], v["vc"], 0, self.cap, self.parts, self.ws,
                                   stream=stream)

    def combine(self, gathered, stream=None) -> int:
        """Merges the all-gathered records ([world, rec]) into self.out: one launch."""
        v = self._stacked()
        ops.gqa_combine(gathered.reshape(-1), gathered.shape[0], v["gate"], v["out"],
                        part_stride=self.rec, stream=stream)
        return 1
