/*
 * Gated GQA attention on B200 (libvx27cuda). Drop-in for src/vx27_gqa.h of
 * DavidPandleton/vx27 (first block, same signatures, host pointers), plus the batched
 * device-resident decode over a BF16 KV cache (second block).
 */
#ifndef VX27_GQA_H
#define VX27_GQA_H
#include <stddef.h>
#include "vx27cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------- reference entry points (src/vx27_gqa.h) ----------------------- */
/* q_head * 4 / 24. Host integer arithmetic. Replaces src/vx27_gqa.h:8. */
int vx27_gqa_kv_for_q(int q_head);
/* y = x / sqrt(mean(x^2) + eps) * w, sum in double; on the GPU.
 * Replaces src/vx27_gqa.h:9. */
void vx27_rmsnorm(const float *x, const float *w, float *y, int n, float eps);
/* Single-query attention, 24 Q / 4 KV heads of 256, fp32 caches [pos][4][256], on the
 * GPU. Same arithmetic as the reference; the reference's 1024-position limit (a static
 * score buffer) does not apply, and the function is reentrant.
 * Replaces src/vx27_gqa.h:12-13. */
void vx27_attn_1q(const float *q, const float *kcache, const float *vcache, int n_pos,
                  float *out);

/* ---------------- batched device-resident tier (no reference counterpart) ------- */
/*
 * Per-token prologue of a full-attention layer, for B sequences (src/vx27_qfwd.c:
 * 339-346): RMSNorm of q and k per head (eps, weights q_norm_w/k_norm_w [hd]; standard
 * x*s*w, or x*s*(1+w) with VX27_F_NORM_1P), partial NeoX RoPE of the first rope_dim
 * dims at position pos[b] (row pos[b] of a table from vx27_rope_table_build), then a
 * bf16 store of the rotated k and of v into slot pos[b] - slot_base of the caches.
 *   q_in [B][nq][hd], k_in/v_in [B][nkv][hd]   activations (act dtype)
 *   k_cache/v_cache bf16 [B][nkv][cap][hd]; NULL skips the store, as does a slot
 *                   outside [0, cap) (context-parallel shards that do not own pos)
 *   q_out [B][nq][hd] fp32: normalised, rotated q for vx27_gqa_decode_batch
 */
int vx27_gqa_append(const void *q_in, const void *k_in, const void *v_in,
                    const float *q_norm_w, const float *k_norm_w, const float *rope_table,
                    int rope_table_len, const int *pos, int slot_base, void *k_cache,
                    void *v_cache, int cap, float *q_out, int B, int nq, int nkv, int hd,
                    int rope_dim, float eps, int flags, void *stream, char *err,
                    size_t errlen);

/*
 * vx27_gqa_append for sequences in groups that have their own norm weights: sequence b
 * uses row b / seqs_per_weight of q_norm_w and k_norm_w ([B / seqs_per_weight][hd]).
 * With the layers of a model stacked as the batch ([layer][seq] as one index, caches and
 * activations laid out [layer][B][...]), one call serves every layer. No counterpart in
 * the reference (it runs the layers one at a time, src/vx27_qfwd.c:339-346).
 */
int vx27_gqa_append_grouped(const void *q_in, const void *k_in, const void *v_in,
                            const float *q_norm_w, const float *k_norm_w, int seqs_per_weight,
                            const float *rope_table, int rope_table_len, const int *pos,
                            int slot_base, void *k_cache, void *v_cache, int cap, float *q_out,
                            int B, int nq, int nkv, int hd, int rope_dim, float eps, int flags,
                            void *stream, char *err, size_t errlen);

/*
 * Decode attention of q (from vx27_gqa_append) over slots [0, pos[b]] of the caches,
 * softmax(q k^T / sqrt(hd)) v per Q head (Q head h reads KV head h*nkv/nq), then
 * out = att * sigmoid(gate) (src/vx27_qfwd.c:347-371). Split-KV flash decoding: each
 * (sequence, KV head, split) block serves the nq/nkv Q heads of its group; several splits
 * are merged with a log-sum-exp combine, one split writes out directly. n_splits = 0 picks
 * a split count for the device. q must be 8-byte aligned; gate, out and the workspace
 * 16-byte aligned.
 *   gate [B][nq][hd] (act dtype), or NULL for no output gate (the MTP drafter's
 *        use_gate = 0, src/vx27_mtp.c:249); out [B][nq][hd] (fp32 or bf16 per VX27_F_OUT_BF16)
 *   workspace: vx27_gqa_decode_workspace_size(B, nq, nkv, hd, cap, n_splits) bytes of
 *   device memory; a smaller workspace lowers the automatic split count to what fits.
 *   hd must be 256.
 */
size_t vx27_gqa_decode_workspace_size(int B, int nq, int nkv, int hd, int max_ctx,
                                      int n_splits);
int vx27_gqa_decode_batch(const float *q, const void *gate, const void *k_cache,
                          const void *v_cache, int cap, const int *pos, void *out,
                          void *workspace, size_t workspace_bytes, int B, int nq, int nkv,
                          int hd, int n_splits, int flags, void *stream, char *err,
                          size_t errlen);

/*
 * The kernel and split count a vx27_gqa_decode_batch / vx27_gqa_decode_fused call with
 * these arguments runs: *kernel = 0 for the tensor-core split-KV kernel, 1 for the
 * CUDA-core one (VX27_F_DECODE_CC); *splits the
 * split count. Returns the number of kernels the call launches (1: the split kernel
 * writes the gated output; 2: split kernel + combine), or -1 for bad arguments. No
 * counterpart in the reference.
 */
int vx27_gqa_decode_plan(int B, int nq, int nkv, int hd, int cap, size_t workspace_bytes,
                         int n_splits, int flags, int *kernel, int *splits);

/*
 * vx27_gqa_append + vx27_gqa_decode_batch in one kernel: the split kernel forms each
 * (sequence, KV head) group's q from the raw activations (QK RMSNorm, partial RoPE at
 * pos[b], the arithmetic of vx27_gqa_append) and writes the token's normalised, rotated K
 * and raw V rows into the caches at slot pos[b] before its tensor-core loads read that
 * slot; then the same attention and gate as vx27_gqa_decode_batch. Replaces one launch
 * per layer (src/vx27_qfwd.c:339-371 per token).
 *   q_in, gate [B][nq][hd], k_in, v_in [B][nkv][hd] (act dtype, 16-byte aligned);
 *   q_norm_w, k_norm_w [hd] (VX27_F_NORM_1P: zero-centred); rope_table [rope_table_len]
 *   [rope_dim] (vx27_rope_table_build), rope_dim a multiple of 16; caches as for
 *   vx27_gqa_decode_batch; workspace: vx27_gqa_decode_workspace_size(...) bytes.
 * The normalised q is not written out (vx27_gqa_append does that).
 */
int vx27_gqa_decode_fused(const void *q_in, const void *k_in, const void *v_in,
                          const float *q_norm_w, const float *k_norm_w, const float *rope_table,
                          int rope_table_len, const void *gate, void *k_cache, void *v_cache,
                          int cap, const int *pos, void *out, void *workspace,
                          size_t workspace_bytes, int B, int nq, int nkv, int hd, int rope_dim,
                          float eps, int n_splits, int flags, void *stream, char *err,
                          size_t errlen);

/*
 * No counterpart in the reference. vx27_gqa_decode_batch without the workspace: same
 * arguments, same split count (n_splits = 0 picks vx27_gqa_decode_batch's automatic count,
 * capped by the array below), same kernels and results, but the split partial records go
 * to a fixed array of VX27_GQA_NOALLOC_SCRATCH_BYTES in the library's own device memory,
 * and the call itself allocates nothing (no cudaMalloc, no cudaFree, no allocating library
 * call). A bounded wait that times out is recorded in the device status word
 * (vx27cuda_device_status), which is a module global as well.
 * It is for callers that cannot provide device scratch: an engine that has already
 * handed all free device memory to its KV cache and weights, or a host that reaches this
 * library through a fixed C interface (such as the reference's) that has no workspace
 * argument and no way to own a device buffer.
 * Limits and rules:
 *  - the array is 8 MiB and is held on every GPU where the library's module is loaded,
 *    until the process exits; one split's records take B*nq*(hd+2)*4 bytes, so a call
 *    needs n_splits*B*nq*(hd+2)*4 <= 8 MiB (a batch whose single record does not fit, or
 *    an explicit n_splits beyond the array, is rejected with an error);
 *  - the first call on a device, made with that device current, looks up the array's
 *    device address (cudaGetSymbolAddress); with CUDA's lazy module loading (the default)
 *    that lookup may also be what loads the module and reserves the 8 MiB, so it can fail
 *    for lack of device memory: make the first call during set-up, before the KV cache
 *    takes the remaining memory, and before any stream capture;
 *  - all calls on a device share the array and it keeps the last call's contents: two
 *    calls whose kernels overlap on the GPU (different streams, no ordering) race and
 *    both results are undefined; calls ordered on one stream are safe.
 */
#define VX27_GQA_NOALLOC_SCRATCH_BYTES (8u << 20)
int vx27_gqa_decode_batch_noalloc(const float *q, const void *gate, const void *k_cache,
                                  const void *v_cache, int cap, const int *pos, void *out,
                                  int B, int nq, int nkv, int hd, int n_splits, int flags,
                                  void *stream, char *err, size_t errlen);

/*
 * Causal gated GQA prefill of T prompt tokens at positions p0 .. p0+T-1 of one sequence
 * (config 4), on the tensor cores. Per token: QK RMSNorm and partial RoPE as
 * vx27_gqa_append (the rotated k and v are written into the bf16 cache slots p0 + t,
 * ready for decode; slots up to the next multiple of 64 past p0 + T are zeroed); then
 * out[t] = softmax over cache positions [0, p0 + t] of (q_t k^T / sqrt(hd)) v, times
 * sigmoid(gate[t]).
 *   q_in, gate [T][nq][hd], k_in, v_in [T][nkv][hd] (act dtype); out [T][nq][hd]
 *   k_cache, v_cache bf16 [nkv][cap][hd] (batch 1 layout of vx27_kv), p0 + T <= cap
 *   workspace: vx27_gqa_prefill_workspace_size(T, nq, hd) bytes (normalised q, bf16)
 * q and p enter the tensor cores as bf16 (accumulation fp32). hd must be 256.
 */
size_t vx27_gqa_prefill_workspace_size(int T, int nq, int hd);
int vx27_gqa_prefill(const void *q_in, const void *k_in, const void *v_in, const void *gate,
                     const float *q_norm_w, const float *k_norm_w, const float *rope_table,
                     int rope_table_len, int p0, void *k_cache, void *v_cache, int cap,
                     void *out, void *workspace, size_t workspace_bytes, int T, int nq, int nkv,
                     int hd, int rope_dim, float eps, int flags, void *stream, char *err,
                     size_t errlen);

/*
 * Context-parallel pieces. A partial record covers cache slots [p_begin, p_end) (the
 * same range for all B sequences): for each (b, Q head) m = max scaled score,
 * l = sum exp(s - m), o = sum exp(s - m) v / l. Record layout (fp32):
 *   o [B][nq][hd] followed by ml [B][nq][2]; record size B*nq*(hd+2) floats.
 * An empty range yields m = -inf, l = 0, o = 0. vx27_gqa_combine merges n_parts records
 * placed part_stride floats apart (0: back to back; else even, with parts 8-byte
 * aligned) -- m* = max m_i, l* = sum l_i e^{m_i-m*}, o = sum o_i l_i e^{m_i-m*} / l* --
 * and applies the sigmoid gate (none when gate is NULL).
 * A long range is split across CTAs and merged into the one record; the sub-records need
 * vx27_gqa_partial_workspace_size(B, nq, nkv, hd, p_end - p_begin) bytes of workspace (a
 * smaller or NULL workspace lowers the split count, down to one CTA per KV head).
 */
size_t vx27_gqa_partial_workspace_size(int B, int nq, int nkv, int hd, int max_range);
int vx27_gqa_partial(const float *q, const void *k_cache, const void *v_cache, int cap,
                     int p_begin, int p_end, float *part, int B, int nq, int nkv, int hd,
                     void *workspace, size_t workspace_bytes, void *stream, char *err,
                     size_t errlen);
int vx27_gqa_combine(const float *parts, int n_parts, size_t part_stride, const void *gate,
                     void *out, int B, int nq, int hd, int flags, void *stream, char *err,
                     size_t errlen);

#ifdef __cplusplus
}
#endif
#endif
