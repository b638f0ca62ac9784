"""Batched hybrid decode: one token step of B sequences through the 64 attention layers
of the vx27 model (16 x [3 Gated DeltaNet + 1 gated GQA], src/vx27_forward64.c:19 puts
full attention at (L+1) % 4 == 0), with every sequence's state and KV cache resident on
one GPU.

The projections around attention are outside this path, so each layer consumes its own
activations for the step (qkv/a/b for DeltaNet, q/k/v/gate for GQA) and produces its
attention output. Kernels are issued in layer order on one stream; their inputs are
independent, so a layer never waits on the previous one beyond stream order.

Device memory per GPU (B sequences, cache capacity `cap` positions):
  DeltaNet state  48 x B x 16 x 128 x 128 fp32   (B=256: 12.9 GB)
  conv history    48 x B x 4 x 6144 fp32         (1.2 GB)
  KV cache        16 x 2 x B x 4 x cap x 256 bf16 (cap=4160: 69.8 GB)
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops

N_LAYERS, N_LIN, N_FULL = 64, 48, 16


@dataclass
class HybridConfig:
    batch: int = 256
    ctx: int = 4096           # tokens already in every sequence's cache
    steps: int = 64           # decode steps the cache must hold room for
    nqk: int = 16
    nv: int = 16
    lin_hd: int = 128
    nq: int = 24
    nkv: int = 4
    hd: int = 256
    rope_dim: int = 64
    theta: float = 1e7
    eps: float = 1e-6
    seed: int = 2
    # GQA layers: QK norm + RoPE + K/V append fused into the split-KV decode
    # (vx27_gqa_decode_fused, True: 65 launches per step, ~0.8% faster at config 2), or as
    # their own kernel before it (False)
    fused_gqa: bool = True

    @property
    def cap(self) -> int:
        return self.ctx + self.steps

    @property
    def conv_channels(self) -> int:
        return (2 * self.nqk + self.nv) * self.lin_hd


def layer_kind(L: int) -> tuple[bool, int]:
    """(is_full_attention, index within its kind) for model layer L."""
    full = (L + 1) % 4 == 0
    return full, (L // 4 if full else L - (L + 1) // 4)


class HybridDecoder:
    def __init__(self, cfg: HybridConfig, device: str | torch.device = "cuda"):
        self.cfg = c = cfg
        self.dev = torch.device(device)
        B, C = c.batch, c.conv_channels
        bf = torch.bfloat16
        kw = dict(device=self.dev)
        # resident state
        self.S = torch.empty(N_LIN, B, c.nv, c.lin_hd, c.lin_hd, dtype=torch.float32, **kw)
        self.ring = torch.empty(N_LIN, B, 4, C, dtype=torch.float32, **kw)
        self.kc = torch.empty(N_FULL, B, c.nkv, c.cap, c.hd, dtype=bf, **kw)
        self.vc = torch.empty(N_FULL, B, c.nkv, c.cap, c.hd, dtype=bf, **kw)
        self.pos = torch.full((B,), c.ctx, dtype=torch.int32, **kw)
        # weights
        self.conv_w = torch.empty(N_LIN, C, 4, dtype=torch.float32, **kw)
        self.A_log = torch.empty(N_LIN, c.nv, dtype=torch.float32, **kw)
        self.dt_bias = torch.empty(N_LIN, c.nv, dtype=torch.float32, **kw)
        self.q_norm_w = torch.empty(N_FULL, c.hd, dtype=torch.float32, **kw)
        self.k_norm_w = torch.empty(N_FULL, c.hd, dtype=torch.float32, **kw)
        self.rope = ops.rope_table(c.cap, c.rope_dim, c.theta, 1.0, device=self.dev)
        # per-step activations and outputs
        self.qkv = torch.empty(N_LIN, B, C, dtype=bf, **kw)
        self.a = torch.empty(N_LIN, B, c.nv, dtype=bf, **kw)
        self.b = torch.empty(N_LIN, B, c.nv, dtype=bf, **kw)
        self.q_in = torch.empty(N_FULL, B, c.nq, c.hd, dtype=bf, **kw)
        self.k_in = torch.empty(N_FULL, B, c.nkv, c.hd, dtype=bf, **kw)
        self.v_in = torch.empty(N_FULL, B, c.nkv, c.hd, dtype=bf, **kw)
        self.gate = torch.empty(N_FULL, B, c.nq, c.hd, dtype=bf, **kw)
        self.dn_out = torch.empty(N_LIN, B, c.nv, c.lin_hd, dtype=bf, **kw)
        self.att_out = torch.empty(N_FULL, B, c.nq, c.hd, dtype=bf, **kw)
        # scratch
        self.qn = torch.empty(B, c.nq, c.hd, dtype=torch.float32, **kw)
        ws = ops.gqa_workspace_bytes(B, c.nq, c.nkv, c.hd, c.cap)
        self.ws = torch.empty(max(ws // 4, 1), dtype=torch.float32, **kw)
        self.fill_synthetic()

    # ------------------------------------------------------------------ inputs
    def fill_synthetic(self) -> None:
        """Seeded synthetic state and inputs with config 2's distributions."""
        s = self.cfg.seed
        f = ops.fill_normal
        f(self.S, s, 1, 0.0, 0.05)
        f(self.ring, s, 2, 0.0, 1.0)
        f(self.kc, s, 3, 0.0, 1.0)
        f(self.vc, s, 4, 0.0, 1.0)
        f(self.conv_w, s, 5, 0.0, 0.5)
        ops.fill_uniform(self.A_log, s, 6, 1.0, 16.0)
        torch.log_(self.A_log)
        f(self.dt_bias, s, 7, 0.0, 0.1)
        f(self.q_norm_w, s, 8, 1.0, 0.02)
        f(self.k_norm_w, s, 9, 1.0, 0.02)
        for n, t in enumerate(self.step_inputs()):
            f(t, s, 100 + n, 0.0, 1.0)
        torch.cuda.synchronize(self.dev)
        ops.device_status()  # allocates the device status word outside any capture

    def step_inputs(self) -> list[torch.Tensor]:
        return [self.qkv, self.a, self.b, self.q_in, self.k_in, self.v_in, self.gate]

    def step_outputs(self) -> list[torch.Tensor]:
        return [self.dn_out, self.att_out]

    # ------------------------------------------------------------------- step
    def step(self, stream=None, on_layer=None) -> int:
        """One decode step of all sequences through the 64 layers; returns kernels launched.
        on_layer(kind, index, phase) is called before ('pre') and after ('post') the main
        kernel of each layer (bench.py records CUDA events there)."""
        c = self.cfg
        n = 0
        for L in range(N_LAYERS):
            full, i = layer_kind(L)
            if not full:
                if on_layer:
                    on_layer("dn", i, "pre")
                # the kernel before this one belongs to another layer (or is the position
                # advance), so this layer's state can stream in while it drains
                ops.deltanet_decode_batch(self.S[i], self.ring[i], self.qkv[i], self.a[i],
                                          self.b[i], self.A_log[i], self.dt_bias[i],
                                          self.conv_w[i], self.pos, self.dn_out[i], c.nqk, c.nv,
                                          stream=stream, prefetch_state=True)
                if on_layer:
                    on_layer("dn", i, "post")
                n += 1
            else:
                n += self._gqa_layer(i, stream, on_layer)
        ops.add_int(self.pos, 1, stream=stream)
        return n + 1

    def reset_positions(self) -> None:
        self.pos.fill_(self.cfg.ctx)

    # ------------------------------------------------------ host-buffer step
    def layer_inputs(self, L: int) -> list[torch.Tensor]:
        full, i = layer_kind(L)
        if full:
            return [self.q_in[i], self.k_in[i], self.v_in[i], self.gate[i]]
        return [self.qkv[i], self.a[i], self.b[i]]

    def layer_output(self, L: int) -> torch.Tensor:
        full, i = layer_kind(L)
        return self.att_out[i] if full else self.dn_out[i]

    def step_host(self, host_in: list[torch.Tensor], host_out: list[torch.Tensor]) -> int:
        """One decode step with the activations in pinned host memory (host_in matches
        step_inputs(), host_out matches step_outputs()). Layer L's inputs are copied in on a
        copy stream while earlier layers compute, and its output is copied back on a second
        stream as soon as its kernel is done; per-layer events keep the next step's copies
        from overwriting buffers a pending kernel or copy still uses. Returns kernels
        launched."""
        if not hasattr(self, "_h2d"):
            self._h2d = torch.cuda.Stream(self.dev)
            self._d2h = torch.cuda.Stream(self.dev)
            self._done = [None] * N_LAYERS   # kernel of layer L finished (previous step)
            self._out_read = [None] * N_LAYERS  # output of layer L copied out (previous step)
        comp = torch.cuda.current_stream(self.dev)
        names = ["qkv", "a", "b", "q_in", "k_in", "v_in", "gate"]
        hmap = dict(zip(names, host_in))
        n = 0
        c = self.cfg
        for L in range(N_LAYERS):
            full, i = layer_kind(L)
            srcs = ([hmap["q_in"][i], hmap["k_in"][i], hmap["v_in"][i], hmap["gate"][i]] if full
                    else [hmap["qkv"][i], hmap["a"][i], hmap["b"][i]])
            with torch.cuda.stream(self._h2d):
                if self._done[L] is not None:
                    self._h2d.wait_event(self._done[L])
                for d, h in zip(self.layer_inputs(L), srcs):
                    d.copy_(h, non_blocking=True)
                ready = torch.cuda.Event()
                ready.record(self._h2d)
            comp.wait_event(ready)
            if self._out_read[L] is not None:
                comp.wait_event(self._out_read[L])
            if not full:
                ops.deltanet_decode_batch(self.S[i], self.ring[i], self.qkv[i], self.a[i],
                                          self.b[i], self.A_log[i], self.dt_bias[i],
                                          self.conv_w[i], self.pos, self.dn_out[i], c.nqk, c.nv,
                                          stream=comp, prefetch_state=True)
                n += 1
            else:
                n += self._gqa_layer(i, comp)
            done = torch.cuda.Event()
            done.record(comp)
            self._done[L] = done
            with torch.cuda.stream(self._d2h):
                self._d2h.wait_event(done)
                dst = host_out[1][i] if full else host_out[0][i]
                dst.copy_(self.layer_output(L), non_blocking=True)
                rd = torch.cuda.Event()
                rd.record(self._d2h)
                self._out_read[L] = rd
        ops.add_int(self.pos, 1, stream=comp)
        comp.wait_stream(self._d2h)  # the step ends when its outputs are on the host
        return n + 1

    # -------------------------------------------------------------- accounting
    def _gqa_layer(self, i: int, stream, on_layer=None) -> int:
        """One GQA layer's decode; returns the kernels launched. on_layer brackets the
        split-KV decode kernel (with the prologue fused in, that is the whole layer)."""
        c = self.cfg
        n = 0
        if not c.fused_gqa:
            ops.gqa_append(self.q_in[i], self.k_in[i], self.v_in[i], self.q_norm_w[i],
                           self.k_norm_w[i], self.rope, self.pos, self.kc[i], self.vc[i],
                           self.qn, eps=c.eps, stream=stream)
            n += 1
        if on_layer:
            on_layer("gqa", i, "pre")
        if c.fused_gqa:
            n += ops.gqa_decode_fused(self.q_in[i], self.k_in[i], self.v_in[i], self.q_norm_w[i],
                                      self.k_norm_w[i], self.rope, self.gate[i], self.kc[i],
                                      self.vc[i], self.pos, self.att_out[i], self.ws, eps=c.eps,
                                      stream=stream)
        else:
            n += ops.gqa_decode_batch(self.qn, self.gate[i], self.kc[i], self.vc[i], self.pos,
                                      self.att_out[i], self.ws, stream=stream)
        if on_layer:
            on_layer("gqa", i, "post")
        return n

    def bytes_per_step(self, ctx_attended: float) -> dict[str, float]:
        """Algorithmic HBM bytes of one step when each sequence attends ctx_attended
        positions: state read+write, conv history, KV read, activations in/out."""
        c = self.cfg
        B = c.batch
        dn_state = N_LIN * B * c.nv * c.lin_hd * c.lin_hd * 4 * 2
        dn_conv = N_LIN * B * (3 * c.conv_channels * 4 + c.conv_channels * 4)  # 3 taps read, 1 written
        dn_act = N_LIN * B * (c.conv_channels * 2 + 2 * c.nv * 2 + c.nv * c.lin_hd * 2)
        kv = N_FULL * B * c.nkv * ctx_attended * c.hd * 2 * 2
        gqa_act = N_FULL * B * (c.nq * c.hd * 2 * 3 + 2 * c.nkv * c.hd * 2 * 2)
        return dict(dn_state=dn_state, dn_conv=dn_conv, dn_act=dn_act, kv=kv, gqa_act=gqa_act,
                    total=dn_state + dn_conv + dn_act + kv + gqa_act)
