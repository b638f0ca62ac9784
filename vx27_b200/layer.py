"""One decode step of a whole attention layer of the model on the device.

The packed-weight projections (K5, ``vx27_pmat_batch_dev``) around the attention kernels
(K1, K2), with the production layer's normalisations, for B independent sequences of one
token each. Per sequence the step is the reference's single-token layer forward:

DeltaNet layer (src/vx27_qfwd.c:95-154):
  qkv = W_qkv x, z = W_z x, a = W_a x, b = W_b x                        (K5)
  conv1d + SiLU, q/k RMSNorm(1 + w) -> l2norm -> q / sqrt(hd), gates, delta rule,
  RMSNorm(ret) * w * silu(z)                   (K1, gated entry, VX27_F_QK_PRENORM)
  out = W_out o                                                          (K5)
GQA layer (src/vx27_qfwd.c:156-214):
  [q | gate] = W_q x, 256 + 256 per head; k = W_k x; v = W_v x          (K5)
  q/k RMSNorm(1 + w), RoPE, BF16 KV append               (vx27_gqa_append, NORM_1P)
  softmax(q k^T / 16) v * sigmoid(gate)                                 (K2)
  out = W_o att                                                          (K5)

The input x is the layer's normalised hidden state, fp32 [B, H]. The input projections
of a layer read the same x, so they run as one K5 launch (``vx27_pmat_multi_dev``); each
output is bit-identical to its own ``vx27_pmat``. Every tensor lives on the device; the
only non-library operation is the split of the interleaved q_proj output into q and
gate, which the reference does with memcpy (src/vx27_qfwd.c:163-166).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops


@dataclass
class PackedLinear:
    """A projection's weights as uploaded: rows packed rows (the reference's in-memory
    layout for dtype, see include/vx27_pmat.h) in a uint8 device tensor."""
    W: torch.Tensor
    dtype: int
    rows: int
    cols: int

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None,
                 stream=None) -> torch.Tensor:
        if out is None:
            out = torch.empty(x.shape[0], self.rows, device=x.device)
        ops.pmat_batch(self.W, self.dtype, x, out, self.rows, self.cols, stream=stream)
        return out


def project(x: torch.Tensor, *lins: PackedLinear, stream=None) -> list[torch.Tensor]:
    """The projections lins (same dtype and cols) of x [B, cols] in one launch."""
    outs = [torch.empty(x.shape[0], m.rows, device=x.device) for m in lins]
    ops.pmat_multi([m.W for m in lins], lins[0].dtype, x, outs, [m.rows for m in lins],
                   lins[0].cols, stream=stream)
    return outs


@dataclass
class DeltaNetLayer:
    qkv: PackedLinear
    z: PackedLinear
    a: PackedLinear
    b: PackedLinear
    out: PackedLinear
    A_log: torch.Tensor      # [nv] fp32
    dt_bias: torch.Tensor    # [nv] fp32
    conv_w: torch.Tensor     # [C][4] fp32, C = (2 nqk + nv) hd
    norm_w: torch.Tensor     # [hd] fp32, linear_attn.norm.weight
    nqk: int = 16
    nv: int = 48
    hd: int = 128

    def step(self, x: torch.Tensor, S: torch.Tensor, ring: torch.Tensor, pos: torch.Tensor,
             stream=None, prefetch_state: bool = False) -> torch.Tensor:
        """x [B, H] fp32; S [B, nv, hd, hd] and ring [B, 4, C] updated in place; pos [B]
        int32 (the token's position). Returns the layer output [B, H] fp32."""
        B = x.shape[0]
        qkv, z, a, b = project(x, self.qkv, self.z, self.a, self.b, stream=stream)
        o = torch.empty(B, self.nv, self.hd, device=x.device)
        ops.deltanet_decode_batch_gated(S, ring, qkv, a, b, self.A_log, self.dt_bias,
                                        self.conv_w, pos, z, self.norm_w, o, self.nqk, self.nv,
                                        stream=stream, qk_prenorm=True,
                                        prefetch_state=prefetch_state)
        return self.out(o.view(B, self.nv * self.hd), stream=stream)


@dataclass
class GQALayer:
    q: PackedLinear          # rows nq * 2 * hd: per head 256 query rows, then 256 gate rows
    k: PackedLinear
    v: PackedLinear
    o: PackedLinear
    q_norm_w: torch.Tensor   # [hd] fp32 (zero-centred)
    k_norm_w: torch.Tensor
    rope: torch.Tensor       # ops.rope_table(cap) [cap][64]
    nq: int = 24
    nkv: int = 4
    hd: int = 256
    eps: float = 1e-6

    def step(self, x: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
             pos: torch.Tensor, workspace: torch.Tensor, stream=None) -> torch.Tensor:
        """x [B, H] fp32; caches bf16 [B, nkv, cap, hd] (this token's K/V appended at
        pos[b]); workspace: ops.gqa_workspace_bytes(...). Returns [B, H] fp32."""
        B = x.shape[0]
        qg, k_in, v_in = project(x, self.q, self.k, self.v, stream=stream)
        qg = qg.view(B, self.nq, 2, self.hd)
        q_in, gate = qg[:, :, 0].contiguous(), qg[:, :, 1].contiguous()
        k_in, v_in = k_in.view(B, self.nkv, self.hd), v_in.view(B, self.nkv, self.hd)
        qn = torch.empty(B, self.nq, self.hd, device=x.device)
        ops.gqa_append(q_in, k_in, v_in, self.q_norm_w, self.k_norm_w, self.rope, pos,
                       k_cache, v_cache, qn, eps=self.eps, norm_one_plus=True, stream=stream)
        att = torch.empty(B, self.nq, self.hd, device=x.device)
        ops.gqa_decode_batch(qn, gate, k_cache, v_cache, pos, att, workspace, stream=stream)
        return self.o(att.view(B, self.nq * self.hd), stream=stream)
