"""Python mirror of the vx27 hot-path interface over libvx27cuda.

Two groups, matching the two tiers of the C ABI:

* reference mirror -- the functions of src/vx27_deltanet.h, src/vx27_gqa.h,
  src/vx27_rope.h and src/vx27_kv.h of DavidPandleton/vx27 under the same names,
  taking numpy float32 arrays (host memory) and computing on the GPU;
* batched tier -- device-resident entry points taking torch CUDA tensors.

Errors of the batched tier raise Vx27Error with the library's message. Nothing here
computes on the CPU: every tensor operation goes through libvx27cuda.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import Vx27Error, check, errbuf, load

F_ACT_BF16 = 0x1
F_OUT_BF16 = 0x2
F_NORM_1P = 0x4
F_GATES_F64 = 0x8
F_PREFETCH_STATE = 0x10
F_QK_PRENORM = 0x20
F_PREFETCH_KV = 0x40
F_DECODE_CC = 0x80
F_DECODE_TC = 0x100
_KERNEL_FLAGS = {"auto": 0, "cc": F_DECODE_CC, "tc": F_DECODE_TC}
F_PREFILL_CTA1 = 0x200


def _np(a: np.ndarray, dtype=np.float32) -> C.c_void_p:
    if a.dtype != dtype or not a.flags["C_CONTIGUOUS"]:
        raise Vx27Error(f"expected a C-contiguous {np.dtype(dtype).name} array")
    return a.ctypes.data_as(C.c_void_p)  # keeps the array alive with the pointer


# ----------------------------------------------------------- reference mirror
def vx27_deltanet_state_per_layer() -> int:
    return load().vx27_deltanet_state_per_layer()


def vx27_deltanet_state_total() -> int:
    return load().vx27_deltanet_state_total()


def vx27_deltanet_state_mb(bytes_per_elem: int) -> float:
    return load().vx27_deltanet_state_mb(bytes_per_elem)


def vx27_deltanet_update_ref(S, k, v, decay: float, hd: int) -> None:
    load().vx27_deltanet_update_ref(_np(S), _np(k), _np(v), decay, hd)


def vx27_deltanet_update_tiled(S, k, v, decay: float, hd: int) -> None:
    load().vx27_deltanet_update_tiled(_np(S), _np(k), _np(v), decay, hd)


def vx27_deltanet_update_avx2(S, k, v, decay: float, hd: int) -> None:
    load().vx27_deltanet_update_avx2(_np(S), _np(k), _np(v), decay, hd)


def vx27_deltanet_retrieve_ref(S, q, o, hd: int) -> None:
    load().vx27_deltanet_retrieve_ref(_np(S), _np(q), _np(o), hd)


def vx27_deltanet_retrieve_tiled(S, q, o, hd: int) -> None:
    load().vx27_deltanet_retrieve_tiled(_np(S), _np(q), _np(o), hd)


def vx27_deltanet_retrieve_avx2(S, q, o, hd: int) -> None:
    load().vx27_deltanet_retrieve_avx2(_np(S), _np(q), _np(o), hd)


def vx27_deltanet_l2norm(x, y, n: int) -> None:
    load().vx27_deltanet_l2norm(_np(x), _np(y), n)


def vx27_deltanet_step_exact(S, q, k, v, beta: float, g_log: float, o, hd: int) -> None:
    load().vx27_deltanet_step_exact(_np(S), _np(q), _np(k), _np(v), beta, g_log, _np(o), hd)


def vx27_deltanet_gate_params(a: float, A_log: float, b: float, dt_bias: float):
    beta, g = C.c_double(), C.c_double()
    load().vx27_deltanet_gate_params(a, A_log, b, dt_bias, C.byref(beta), C.byref(g))
    return beta.value, g.value


def vx27_conv1d_step(state, x, w, y, C_: int, apply_silu: int) -> None:
    load().vx27_conv1d_step(_np(state), _np(x), _np(w), _np(y), C_, apply_silu)


def vx27_gqa_kv_for_q(q_head: int) -> int:
    return load().vx27_gqa_kv_for_q(q_head)


def vx27_rmsnorm(x, w, y, n: int, eps: float) -> None:
    load().vx27_rmsnorm(_np(x), _np(w), _np(y), n, eps)


def vx27_attn_1q(q, kcache, vcache, n_pos: int, out) -> None:
    load().vx27_attn_1q(_np(q), _np(kcache), _np(vcache), n_pos, _np(out))


def vx27_rope_cos_sin(pos: int, cosv, sinv, rope_dim: int, theta: float, yarn: float) -> None:
    load().vx27_rope_cos_sin(pos, _np(cosv), _np(sinv), rope_dim, theta, yarn)


def vx27_rope_apply(v, n_heads: int, head_dim: int, rope_dim: int, cosv, sinv) -> None:
    load().vx27_rope_apply(_np(v), n_heads, head_dim, rope_dim, _np(cosv), _np(sinv))


def vx27_mrope_cos_sin_text(pos: int, cosv, sinv) -> None:
    load().vx27_mrope_cos_sin_text(pos, _np(cosv), _np(sinv))


def vx27_kv_elems(ctx: int) -> int:
    return load().vx27_kv_elems(ctx)


def vx27_kv_gb(ctx: int, bytes_per_elem: float) -> float:
    return load().vx27_kv_gb(ctx, bytes_per_elem)


def vx27_kv_fits(ctx: int, bytes_per_elem: float, budget_gb: float) -> int:
    return load().vx27_kv_fits(ctx, bytes_per_elem, budget_gb)


# ------------------------------------------------------------- batched tier
# The wrappers run once per launch in an eager decode loop, so their checks use the
# cheapest torch queries (an int device index, the raw current stream).
_cur_dev = None


def _device() -> int:
    global _cur_dev
    if _cur_dev is None:
        import torch
        _cur_dev = torch.cuda.current_device
    return _cur_dev()


def _t(t) -> int | None:
    """Device address of a contiguous tensor on the current device (None for None)."""
    if t is None:
        return None
    if not (t.is_cuda and t.is_contiguous()):
        raise Vx27Error("expected a contiguous CUDA tensor")
    if t.get_device() != _device():
        raise Vx27Error(f"tensor on {t.device}, but the current device is cuda:{_device()}")
    return t.data_ptr()


def _need(t, name: str, numel: int, dtypes, optional: bool = False) -> None:
    """Checks a tensor argument before its pointer reaches a kernel, which trusts sizes:
    a dtype from dtypes and at least numel elements (None allowed when optional)."""
    if t is None:
        if optional:
            return
        raise Vx27Error(f"{name}: required")
    if t.dtype not in dtypes:
        raise Vx27Error(f"{name}: dtype {t.dtype} not one of {', '.join(map(str, dtypes))}")
    if t.numel() < numel:
        raise Vx27Error(f"{name}: {t.numel()} elements, the call needs {numel}")


def _dt():
    import torch
    return torch.float32, torch.bfloat16, torch.int32, torch.float64, torch.uint8


def _check_deltanet(S, conv_ring, qkv, a, b, A_log, dt_bias, conv_w, pos, o, B, nqk, nv, hd,
                    gates_f64, T=None):
    f32, bf16, i32, f64, _ = _dt()
    C_ = (2 * nqk + nv) * hd
    n = T if T is not None else B                       # tokens (rows of the activations)
    _need(S, "S", (1 if T is not None else B) * nv * hd * hd, (f32,))
    _need(conv_ring, "conv_ring", (1 if T is not None else B) * 4 * C_, (f32,))
    _need(qkv, "qkv", n * C_, (f32, bf16))
    for t, nm in ((a, "a"), (b, "b")):
        _need(t, nm, n * nv, (f64,) if gates_f64 else (qkv.dtype,))
    _need(A_log, "A_log", nv, (f32,), optional=gates_f64)
    _need(dt_bias, "dt_bias", nv, (f32,), optional=gates_f64)
    _need(conv_w, "conv_w", C_ * 4, (f32,))
    _need(pos, "pos", n, (i32,))
    _need(o, "o", n * nv * hd, (f32, bf16))


def _stream(stream) -> int:
    """cudaStream_t of stream, or of the current stream of the current device."""
    if stream is None:
        import torch
        return torch._C._cuda_getCurrentRawStream(_device())
    return stream.cuda_stream


def _is_bf16(t) -> bool:
    import torch
    return t.dtype == torch.bfloat16


def deltanet_decode_batch(S, conv_ring, qkv, a, b, A_log, dt_bias, conv_w, pos, o, nqk: int,
                          nv: int, gates_f64: bool = False, stream=None,
                          prefetch_state: bool = False) -> None:
    """One DeltaNet decode step for a batch (vx27_deltanet_decode_batch). prefetch_state:
    the kernel may start reading S while the previous kernel on the stream still runs
    (VX27_F_PREFETCH_STATE) - only when that kernel does not write S."""
    B = S.shape[0]
    hd = S.shape[-1]
    _check_deltanet(S, conv_ring, qkv, a, b, A_log, dt_bias, conv_w, pos, o, B, nqk, nv, hd,
                    gates_f64)
    flags = (F_ACT_BF16 if _is_bf16(qkv) else 0) | (F_OUT_BF16 if _is_bf16(o) else 0) | \
        (F_GATES_F64 if gates_f64 else 0) | (F_PREFETCH_STATE if prefetch_state else 0)
    e = errbuf()
    rc = load().vx27_deltanet_decode_batch(_t(S), _t(conv_ring), _t(qkv), _t(a), _t(b),
                                           _t(A_log), _t(dt_bias), _t(conv_w), _t(pos), _t(o),
                                           B, nqk, nv, hd, flags, _stream(stream), e, 512)
    check(rc, e)


def deltanet_decode_tokens(S, conv_ring, qkv, a, b, A_log, dt_bias, conv_w, pos, o, nqk: int,
                           nv: int, S_ckpt=None, conv_ckpt=None, stream=None,
                           gates_f64: bool = False) -> None:
    """T tokens of one sequence (vx27_deltanet_decode_tokens, one kernel with the state
    resident across the tokens); S [nv][128][128], conv_ring [4][C], qkv [T][C],
    a, b [T][nv] (double beta / g_log with gates_f64), pos [T], o [T][nv][128]; optional
    S_ckpt [T][nv][128][128] and conv_ckpt [T][C][3] snapshots."""
    T = qkv.shape[0]
    _check_deltanet(S, conv_ring, qkv, a, b, A_log, dt_bias, conv_w, pos, o, 1, nqk, nv, 128,
                    gates_f64, T=T)
    f32 = _dt()[0]
    _need(S_ckpt, "S_ckpt", T * nv * 128 * 128, (f32,), optional=True)
    _need(conv_ckpt, "conv_ckpt", T * (2 * nqk + nv) * 128 * 3, (f32,), optional=True)
    flags = (F_ACT_BF16 if _is_bf16(qkv) else 0) | (F_OUT_BF16 if _is_bf16(o) else 0) | \
        (F_GATES_F64 if gates_f64 else 0)
    e = errbuf()
    rc = load().vx27_deltanet_decode_tokens(_t(S), _t(conv_ring), _t(qkv), _t(a), _t(b),
                                            _t(A_log), _t(dt_bias), _t(conv_w), _t(pos), _t(o),
                                            _t(S_ckpt), _t(conv_ckpt), T, nqk, nv, 128, flags,
                                            _stream(stream), e, 512)
    check(rc, e)


def deltanet_decode_batch_gated(S, conv_ring, qkv, a, b, A_log, dt_bias, conv_w, pos, z,
                                norm_w, o, nqk: int, nv: int, gates_f64: bool = False,
                                stream=None, qk_prenorm: bool = False,
                                prefetch_state: bool = False) -> None:
    """Decode step plus the gated RMSNorm output (vx27_deltanet_decode_batch_gated).
    qk_prenorm: the production layer's q/k RMSNorm (1+norm_w), l2norm and 1/sqrt(hd)
    before the delta rule's own normalisation (VX27_F_QK_PRENORM)."""
    B = S.shape[0]
    hd = S.shape[-1]
    flags = (F_ACT_BF16 if _is_bf16(qkv) else 0) | (F_OUT_BF16 if _is_bf16(o) else 0) | \
        (F_GATES_F64 if gates_f64 else 0) | (F_QK_PRENORM if qk_prenorm else 0) | \
        (F_PREFETCH_STATE if prefetch_state else 0)
    _check_deltanet(S, conv_ring, qkv, a, b, A_log, dt_bias, conv_w, pos, o, B, nqk, nv, hd,
                    gates_f64)
    _need(z, "z", B * nv * hd, (qkv.dtype,))
    _need(norm_w, "norm_w", hd, (_dt()[0],))
    e = errbuf()
    rc = load().vx27_deltanet_decode_batch_gated(_t(S), _t(conv_ring), _t(qkv), _t(a), _t(b),
                                                 _t(A_log), _t(dt_bias), _t(conv_w), _t(pos),
                                                 _t(z), _t(norm_w), _t(o), B, nqk, nv, hd,
                                                 flags, _stream(stream), e, 512)
    check(rc, e)


def deltanet_prefill_chunked(q, k, v, a, b, A_log, dt_bias, S, o, workspace=None,
                             gates_f64: bool = False, stream=None) -> None:
    """Chunked gated delta rule over T tokens (vx27_deltanet_prefill_chunked).
    q, k [T][nqk][128], v [T][nv][128], a, b [T][nv], S [nv][128][128] in/out."""
    import torch
    T, nqk, hd = q.shape
    nv = v.shape[1]
    f32, bf16, _, f64, _ = _dt()
    _need(q, "q", T * nqk * hd, (f32, bf16))
    _need(k, "k", T * nqk * hd, (q.dtype,))
    _need(v, "v", T * nv * hd, (q.dtype,))
    for t, nm in ((a, "a"), (b, "b")):  # the library requires bf16 (or f64 gates) itself
        _need(t, nm, T * nv, (f64,) if gates_f64 else (f32, bf16))
    _need(A_log, "A_log", nv, (f32,), optional=gates_f64)
    _need(dt_bias, "dt_bias", nv, (f32,), optional=gates_f64)
    _need(S, "S", nv * hd * hd, (f32,))
    _need(o, "o", T * nv * hd, (f32, bf16))
    need = load().vx27_deltanet_prefill_workspace_size(T, nqk, nv, hd)
    if workspace is None:
        workspace = torch.empty(need // 4 + 1, dtype=torch.float32, device=q.device)
    flags = (F_ACT_BF16 if _is_bf16(q) else 0) | (F_OUT_BF16 if _is_bf16(o) else 0) | \
        (F_GATES_F64 if gates_f64 else 0)
    e = errbuf()
    rc = load().vx27_deltanet_prefill_chunked(_t(q), _t(k), _t(v), _t(a), _t(b), _t(A_log),
                                              _t(dt_bias), _t(S), _t(o), _t(workspace),
                                              workspace.numel() * workspace.element_size(), T,
                                              nqk, nv, hd, flags, _stream(stream), e, 512)
    check(rc, e)


def rope_table(n_pos: int, rope_dim: int = 64, theta: float = 1e7, yarn: float = 1.0,
               device=None):
    """Device RoPE table [n_pos][rope_dim] (cos | sin), values from vx27_rope_cos_sin."""
    import torch
    t = torch.empty((n_pos, rope_dim), dtype=torch.float32, device=device or "cuda")
    e = errbuf()
    check(load().vx27_rope_table_build(_t(t), n_pos, rope_dim, theta, yarn, e, 512), e)
    return t


def gqa_append(q_in, k_in, v_in, q_norm_w, k_norm_w, rope, pos, k_cache, v_cache, q_out,
               eps: float = 1e-6, slot_base: int = 0, norm_one_plus: bool = False,
               stream=None) -> None:
    """QK norm + RoPE + K/V store of one token per sequence (vx27_gqa_append). The norm
    weights are [hd], or [G, hd] for G groups of B / G consecutive sequences each with
    their own weights (vx27_gqa_append_grouped: the layers of a model stacked as the
    batch)."""
    B, nq, hd = q_in.shape
    nkv = k_in.shape[1]
    cap = k_cache.shape[2] if k_cache is not None else 0
    f32, bf16, i32, _, _ = _dt()
    _need(q_in, "q_in", B * nq * hd, (f32, bf16))
    _need(k_in, "k_in", B * nkv * hd, (q_in.dtype,))
    _need(v_in, "v_in", B * nkv * hd, (q_in.dtype,))
    groups = q_norm_w.numel() // hd if q_norm_w.numel() % hd == 0 else 0
    if groups < 1 or B % groups:
        raise Vx27Error(f"q_norm_w: {q_norm_w.numel()} values is not [G][{hd}] with G dividing {B}")
    _need(q_norm_w, "q_norm_w", groups * hd, (f32,))
    _need(k_norm_w, "k_norm_w", groups * hd, (f32,))
    _need(rope, "rope", 1, (f32,))
    _need(pos, "pos", B, (i32,))
    _need(k_cache, "k_cache", B * nkv * cap * hd, (bf16,), optional=True)
    _need(v_cache, "v_cache", B * nkv * cap * hd, (bf16,), optional=True)
    _need(q_out, "q_out", B * nq * hd, (f32,))
    flags = (F_ACT_BF16 if _is_bf16(q_in) else 0) | (F_NORM_1P if norm_one_plus else 0)
    e = errbuf()
    rc = load().vx27_gqa_append_grouped(_t(q_in), _t(k_in), _t(v_in), _t(q_norm_w),
                                        _t(k_norm_w), B // groups, _t(rope), rope.shape[0],
                                        _t(pos), slot_base, _t(k_cache), _t(v_cache), cap,
                                        _t(q_out), B, nq, nkv, hd, rope.shape[1], eps, flags,
                                        _stream(stream), e, 512)
    check(rc, e)


def gqa_workspace_bytes(B: int, nq: int, nkv: int, hd: int, max_ctx: int,
                        n_splits: int = 0) -> int:
    return load().vx27_gqa_decode_workspace_size(B, nq, nkv, hd, max_ctx, n_splits)


def gqa_decode_plan(B: int, nq: int, nkv: int, hd: int, cap: int, ws_bytes: int,
                    n_splits: int = 0, kernel: str = "auto") -> tuple[str, int, int]:
    """The library's choice for a decode call (vx27_gqa_decode_plan): ("tc" | "cc", split
    count, kernels launched: 1 when one split writes the gated output, 2 with a combine)."""
    k, n = C.c_int(), C.c_int()
    launches = load().vx27_gqa_decode_plan(B, nq, nkv, hd, cap, ws_bytes, n_splits,
                                           _KERNEL_FLAGS[kernel], C.byref(k), C.byref(n))
    if launches < 0:
        raise Vx27Error(f"vx27_gqa_decode_plan: bad arguments B={B} nq={nq} nkv={nkv}")
    return ("cc" if k.value else "tc"), n.value, launches


def gqa_decode_launches(B: int, nq: int, nkv: int, hd: int, cap: int, ws_bytes: int,
                        n_splits: int = 0, kernel: str = "auto") -> int:
    """Kernels one decode call launches: the library's split count (its own choice when
    n_splits <= 0, capped by the workspace), then 1 for one split (the split kernel writes
    the gated output) or 2 (split kernel + combine)."""
    return gqa_decode_plan(B, nq, nkv, hd, cap, ws_bytes, n_splits, kernel)[2]


def gqa_partial_launches(B: int, nq: int, nkv: int, hd: int, span: int, ws_bytes: int) -> int:
    """Kernels one vx27_gqa_partial call over span slots launches: 2 when the workspace
    lets it split the range (split kernel + merge), else 1."""
    rec = B * nq * (hd + 2) * 4
    n = min(gqa_partial_workspace_bytes(B, nq, nkv, hd, span) // rec, ws_bytes // rec)
    return 2 if n > 1 else 1


def gqa_decode_batch(q, gate, k_cache, v_cache, pos, out, workspace, n_splits: int = 0,
                     stream=None, kernel: str = "auto", prefetch_kv: bool = False) -> int:
    """Split-KV decode of one token per sequence (vx27_gqa_decode_batch); returns the
    kernels it launched: 1 with one split (the split kernel writes the gated output), 2
    with several (split kernel + combine). kernel: "auto" (the library's choice by batch
    shape), "tc" (tensor cores) or "cc" (CUDA cores); prefetch_kv: VX27_F_PREFETCH_KV."""
    B, nq, hd = q.shape
    nkv, cap = k_cache.shape[1], k_cache.shape[2]
    f32, bf16, i32, _, _ = _dt()
    _need(q, "q", B * nq * hd, (f32,))
    _need(gate, "gate", B * nq * hd, (f32, bf16), optional=True)
    _need(k_cache, "k_cache", B * nkv * cap * hd, (bf16,))
    _need(v_cache, "v_cache", B * nkv * cap * hd, (bf16,))
    _need(pos, "pos", B, (i32,))
    _need(out, "out", B * nq * hd, (f32, bf16))
    flags = (F_ACT_BF16 if gate is not None and _is_bf16(gate) else 0) | \
        (F_OUT_BF16 if _is_bf16(out) else 0) | _KERNEL_FLAGS[kernel] | \
        (F_PREFETCH_KV if prefetch_kv else 0)
    e = errbuf()
    ws_bytes = workspace.numel() * workspace.element_size()
    rc = load().vx27_gqa_decode_batch(_t(q), _t(gate), _t(k_cache), _t(v_cache), cap, _t(pos),
                                      _t(out), _t(workspace), ws_bytes, B, nq, nkv, hd, n_splits,
                                      flags, _stream(stream), e, 512)
    check(rc, e)
    return gqa_decode_launches(B, nq, nkv, hd, cap, ws_bytes, n_splits, kernel)


def gqa_decode_fused(q_in, k_in, v_in, q_norm_w, k_norm_w, rope, gate, k_cache, v_cache, pos,
                     out, workspace, eps: float = 1e-6, norm_one_plus: bool = False,
                     n_splits: int = 0, stream=None, kernel: str = "auto",
                     prefetch_kv: bool = False) -> int:
    """gqa_append + gqa_decode_batch as one kernel (vx27_gqa_decode_fused): the new token's
    K/V rows land in the caches at pos[b] and out gets the gated attention; returns the
    kernels launched (1 with one split, 2 with a combine). kernel and prefetch_kv as for
    gqa_decode_batch."""
    B, nq, hd = q_in.shape
    nkv, cap = k_cache.shape[1], k_cache.shape[2]
    f32, bf16, i32, _, _ = _dt()
    _need(q_in, "q_in", B * nq * hd, (f32, bf16))
    _need(k_in, "k_in", B * nkv * hd, (q_in.dtype,))
    _need(v_in, "v_in", B * nkv * hd, (q_in.dtype,))
    _need(gate, "gate", B * nq * hd, (q_in.dtype,), optional=True)
    _need(q_norm_w, "q_norm_w", hd, (f32,))
    _need(k_norm_w, "k_norm_w", hd, (f32,))
    _need(rope, "rope", 1, (f32,))
    _need(pos, "pos", B, (i32,))
    _need(k_cache, "k_cache", B * nkv * cap * hd, (bf16,))
    _need(v_cache, "v_cache", B * nkv * cap * hd, (bf16,))
    _need(out, "out", B * nq * hd, (f32, bf16))
    flags = (F_ACT_BF16 if _is_bf16(q_in) else 0) | (F_OUT_BF16 if _is_bf16(out) else 0) | \
        (F_NORM_1P if norm_one_plus else 0) | _KERNEL_FLAGS[kernel] | \
        (F_PREFETCH_KV if prefetch_kv else 0)
    ws_bytes = workspace.numel() * workspace.element_size()
    e = errbuf()
    rc = load().vx27_gqa_decode_fused(_t(q_in), _t(k_in), _t(v_in), _t(q_norm_w), _t(k_norm_w),
                                      _t(rope), rope.shape[0], _t(gate), _t(k_cache),
                                      _t(v_cache), cap, _t(pos), _t(out), _t(workspace),
                                      ws_bytes, B, nq, nkv, hd, rope.shape[1], eps, n_splits,
                                      flags, _stream(stream), e, 512)
    check(rc, e)
    return gqa_decode_launches(B, nq, nkv, hd, cap, ws_bytes, n_splits, kernel)


def gqa_partial_workspace_bytes(B: int, nq: int, nkv: int, hd: int, max_range: int) -> int:
    return load().vx27_gqa_partial_workspace_size(B, nq, nkv, hd, max_range)


def gqa_partial(q, k_cache, v_cache, p_begin: int, p_end: int, part, workspace=None,
                stream=None) -> int:
    """Partial record over cache slots [p_begin, p_end) (split across CTAs when a
    workspace is given); returns the kernels launched (1, or 2 with a merge of splits)."""
    B, nq, hd = q.shape
    nkv, cap = k_cache.shape[1], k_cache.shape[2]
    f32, bf16 = _dt()[:2]
    _need(q, "q", B * nq * hd, (f32,))
    _need(k_cache, "k_cache", B * nkv * cap * hd, (bf16,))
    _need(v_cache, "v_cache", B * nkv * cap * hd, (bf16,))
    _need(part, "part", B * nq * (hd + 2), (f32,))
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    e = errbuf()
    rc = load().vx27_gqa_partial(_t(q), _t(k_cache), _t(v_cache), cap, p_begin, p_end, _t(part),
                                 B, nq, nkv, hd, _t(workspace), ws_bytes, _stream(stream), e, 512)
    check(rc, e)
    return gqa_partial_launches(B, nq, nkv, hd, p_end - p_begin, ws_bytes)


def gqa_combine(parts, n_parts: int, gate, out, part_stride: int = 0, stream=None) -> None:
    """Merges n_parts partial records placed part_stride floats apart (0: contiguous);
    gate None: no output gate."""
    B, nq, hd = out.shape
    f32, bf16 = _dt()[:2]
    rec = B * nq * (hd + 2)
    _need(parts, "parts", (n_parts - 1) * (part_stride or rec) + rec, (f32,))
    _need(gate, "gate", B * nq * hd, (f32, bf16), optional=True)
    _need(out, "out", B * nq * hd, (f32, bf16))
    flags = (F_ACT_BF16 if gate is not None and _is_bf16(gate) else 0) | \
        (F_OUT_BF16 if _is_bf16(out) else 0)
    e = errbuf()
    if parts.is_cuda and not parts.is_contiguous():
        raise Vx27Error("parts must be contiguous")
    rc = load().vx27_gqa_combine(C.c_void_p(parts.data_ptr()), n_parts, part_stride, _t(gate),
                                 _t(out), B, nq, hd, flags, _stream(stream), e, 512)
    check(rc, e)


PMAT_F32, PMAT_Q8_K, PMAT_BP3_128 = 0, 2, 4


def pmat_row_bytes(dtype: int, cols: int) -> int:
    return int(load().vx27_pmat_row_bytes(dtype, cols))


def pmat_batch(W, dtype: int, xb, yb, rows: int, cols: int, stream=None) -> None:
    """Packed-weight matvec (vx27_pmat_batch_dev): yb[b, r] = W[r] . xb[b]; W a uint8
    tensor holding rows packed rows of pmat_row_bytes(dtype, cols) bytes, xb [B, cols] and
    yb [B, rows] fp32."""
    import torch
    B = xb.shape[0]
    if xb.dtype != torch.float32 or yb.dtype != torch.float32:
        raise Vx27Error("pmat_batch: xb and yb must be fp32")
    if W.numel() * W.element_size() < rows * pmat_row_bytes(dtype, cols):
        raise Vx27Error("pmat_batch: W holds fewer than rows packed rows")
    _need(xb, "xb", B * cols, (torch.float32,))
    _need(yb, "yb", B * rows, (torch.float32,))
    e = errbuf()
    rc = load().vx27_pmat_batch_dev(_t(W), dtype, _t(xb), _t(yb), rows, cols, B, _stream(stream),
                                    e, 512)
    check(rc, e)


PMAT_MAX_GROUPS = 4


def pmat_multi(Ws, dtype: int, xb, ys, rows, cols: int, stream=None) -> None:
    """Several projections of the same xb [B, cols] in one launch (vx27_pmat_multi_dev):
    ys[i][b, r] = Ws[i][r] . xb[b] for each i, with the same dtype and cols; each output as
    pmat_batch writes it."""
    import torch
    n, B = len(Ws), xb.shape[0]
    if not 1 <= n <= PMAT_MAX_GROUPS or len(ys) != n or len(rows) != n:
        raise Vx27Error(f"pmat_multi: 1..{PMAT_MAX_GROUPS} projections with one output and "
                        f"one row count each")
    _need(xb, "xb", B * cols, (torch.float32,))
    for i in range(n):
        if Ws[i].numel() * Ws[i].element_size() < rows[i] * pmat_row_bytes(dtype, cols):
            raise Vx27Error(f"pmat_multi: W[{i}] holds fewer than {rows[i]} packed rows")
        _need(ys[i], f"y[{i}]", B * rows[i], (torch.float32,))
    Wp = (C.c_void_p * n)(*[_t(w) for w in Ws])
    yp = (C.c_void_p * n)(*[_t(y) for y in ys])
    rp = (C.c_int * n)(*rows)
    e = errbuf()
    rc = load().vx27_pmat_multi_dev(n, Wp, dtype, _t(xb), yp, rp, cols, B, _stream(stream), e,
                                    512)
    check(rc, e)


def gqa_prefill(q_in, k_in, v_in, gate, q_norm_w, k_norm_w, rope, k_cache, v_cache, out,
                workspace=None, p0: int = 0, eps: float = 1e-6, norm_one_plus: bool = False,
                stream=None, cta_pairs: bool = True):
    """Causal gated GQA prefill of T tokens (vx27_gqa_prefill); k_cache/v_cache [nkv][cap][hd].
    cta_pairs=False runs the attention one CTA per (query tile, head) on one SM
    (VX27_F_PREFILL_CTA1) instead of 2-CTA pairs over two SMs (used with an even number of
    query heads per KV head)."""
    import torch
    T, nq, hd = q_in.shape
    nkv = k_in.shape[1]
    cap = k_cache.shape[1]
    f32, bf16 = _dt()[:2]
    _need(q_in, "q_in", T * nq * hd, (f32, bf16))
    for t, nm, n in ((k_in, "k_in", T * nkv * hd), (v_in, "v_in", T * nkv * hd),
                     (gate, "gate", T * nq * hd)):
        _need(t, nm, n, (q_in.dtype,))
    _need(q_norm_w, "q_norm_w", hd, (f32,))
    _need(k_norm_w, "k_norm_w", hd, (f32,))
    _need(rope, "rope", 1, (f32,))
    _need(k_cache, "k_cache", nkv * cap * hd, (bf16,))
    _need(v_cache, "v_cache", nkv * cap * hd, (bf16,))
    _need(out, "out", T * nq * hd, (f32, bf16))
    need = load().vx27_gqa_prefill_workspace_size(T, nq, hd)
    if workspace is None:
        workspace = torch.empty(need // 2 + 1, dtype=torch.int16, device=q_in.device)
    flags = (F_ACT_BF16 if _is_bf16(q_in) else 0) | (F_OUT_BF16 if _is_bf16(out) else 0) | \
        (F_NORM_1P if norm_one_plus else 0) | (0 if cta_pairs else F_PREFILL_CTA1)
    e = errbuf()
    rc = load().vx27_gqa_prefill(_t(q_in), _t(k_in), _t(v_in), _t(gate), _t(q_norm_w),
                                 _t(k_norm_w), _t(rope), rope.shape[0], p0, _t(k_cache),
                                 _t(v_cache), cap, _t(out), _t(workspace),
                                 workspace.numel() * workspace.element_size(), T, nq, nkv, hd,
                                 rope.shape[1], eps, flags, _stream(stream), e, 512)
    check(rc, e)


def fill_normal(t, seed: int, stream_id: int, mean: float = 0.0, std: float = 1.0,
                offset: int = 0, stream=None) -> None:
    """t[e] = element offset+e of the seeded normal stream (seed, stream_id)."""
    e = errbuf()
    rc = load().vx27cuda_fill_normal(_t(t), t.numel(), 1 if _is_bf16(t) else 0, seed, stream_id,
                                     offset, mean, std, _stream(stream), e, 512)
    check(rc, e)


def fill_uniform(t, seed: int, stream_id: int, lo: float, hi: float, stream=None) -> None:
    e = errbuf()
    check(load().vx27cuda_fill_uniform(_t(t), t.numel(), seed, stream_id, lo, hi,
                                       _stream(stream), e, 512), e)


def add_int(t, delta: int, stream=None) -> None:
    e = errbuf()
    check(load().vx27cuda_add_int(_t(t), t.numel(), delta, _stream(stream), e, 512), e)


def device_status(clear: bool = True, stream=None) -> int:
    st = C.c_uint32()
    e = errbuf()
    check(load().vx27cuda_device_status(_stream(stream), C.byref(st), 1 if clear else 0, e, 512), e)
    return st.value
