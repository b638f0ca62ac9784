/*
 * Gated DeltaNet on B200 (libvx27cuda). Drop-in for src/vx27_deltanet.h of
 * DavidPandleton/vx27: the first block repeats that header's entry points with the
 * same signatures and host-pointer semantics; the second block adds the batched,
 * device-resident decode and chunked prefill.
 */
#ifndef VX27_DELTANET_H
#define VX27_DELTANET_H
#include <stddef.h>
#include "vx27cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------- reference entry points (src/vx27_deltanet.h) ----------------- */
/* Sizing, host arithmetic. Replace src/vx27_deltanet.h:10-12. */
int vx27_deltanet_state_per_layer(void);     /* 16*128*128 = 262144 */
int vx27_deltanet_state_total(void);         /* x 48 linear layers */
double vx27_deltanet_state_mb(int bytes_per_elem);

/* S = decay*S + outer(k, v); o = S^T q. One head, hd x hd row-major, run on the GPU.
 * Replace src/vx27_deltanet.h:17-19 (_ref), :22-24 (_tiled), :28-30 (_avx2); each
 * variant reproduces its reference's rounding (separate multiply/add for _ref and
 * _tiled, fused multiply-add for _avx2) and summation order. */
void vx27_deltanet_update_ref(float *S, const float *k, const float *v, float decay, int hd);
void vx27_deltanet_retrieve_ref(const float *S, const float *q, float *o, int hd);
void vx27_deltanet_update_tiled(float *S, const float *k, const float *v, float decay, int hd);
void vx27_deltanet_retrieve_tiled(const float *S, const float *q, float *o, int hd);
void vx27_deltanet_update_avx2(float *S, const float *k, const float *v, float decay, int hd);
void vx27_deltanet_retrieve_avx2(const float *S, const float *q, float *o, int hd);

/* y = x / sqrt(sum x^2 + 1e-6) (sum in double). Replaces src/vx27_deltanet.h:34. */
void vx27_deltanet_l2norm(const float *x, float *y, int n);

/* One exact gated delta-rule step for one V head (hd <= 256), on the GPU with double
 * accumulation like the reference. Replaces src/vx27_deltanet.h:43-44. */
void vx27_deltanet_step_exact(float *S, const float *q, const float *k, const float *v,
                              double beta, double g_log, float *o, int hd);

/* beta = sigmoid(b); g_log = -exp(A_log)*softplus(a + dt_bias). Host double arithmetic,
 * bit-identical to the reference. Replaces src/vx27_deltanet.h:49-50. */
void vx27_deltanet_gate_params(double a, double A_log, double b, double dt_bias,
                               double *beta, double *g_log);

/* Depthwise causal conv1d, width 4, state = last 3 inputs per channel, optional SiLU.
 * Replaces src/vx27_deltanet.h:57-59. */
void vx27_conv1d_step(float *state, const float *x, const float *w, float *y, int C,
                      int apply_silu);

/* ---------------- batched device-resident tier (no reference counterpart) ------- */
/*
 * One decode step of one DeltaNet layer for B sequences, one fused kernel:
 * conv1d(+SiLU) -> l2norm(q,k), q/sqrt(hd) -> gates -> decay, delta update, retrieve.
 * Per sequence the arithmetic is that of src/vx27_qfwd.c:276-297 (conv1d_step,
 * gate_params, step_exact per V head; V head vh reads QK head vh*nqk/nv), computed in
 * fp32 with the state held in registers.
 *   S         [B][nv][hd][hd] fp32, updated in place
 *   conv_ring [B][4][C] fp32, C = (2*nqk + nv)*hd; slot p%4 holds the input of token p,
 *             zero-initialised at position 0 (vx27_deltanet_conv_import converts from the
 *             reference's [C][3] state)
 *   qkv       [B][C] pre-conv activations, channel order q | k | v
 *   a, b      [B][nv] gate logits (act dtype), or with VX27_F_GATES_F64 double beta
 *             (in a) and g_log (in b) computed by vx27_deltanet_gate_params
 *   A_log, dt_bias [nv] fp32; conv_w [C][4] fp32, tap 0 = oldest
 *   pos       [B] int, tokens each sequence has consumed (this token's index)
 *   o         [B][nv][hd] retrieve output (fp32, or bf16 with VX27_F_OUT_BF16)
 * hd must be 128. Flags: VX27_F_ACT_BF16, VX27_F_OUT_BF16, VX27_F_GATES_F64.
 */
int vx27_deltanet_decode_batch(float *S, float *conv_ring, const void *qkv, const void *a,
                               const void *b, const float *A_log, const float *dt_bias,
                               const float *conv_w, const int *pos, void *o, int B, int nqk,
                               int nv, int hd, int flags, void *stream, char *err,
                               size_t errlen);

/*
 * vx27_deltanet_decode_batch followed by the layer's gated RMSNorm output
 * (src/vx27_qfwd.c:146-151, rmsn_std :42-46, silu1 :48), fused in the kernel's epilogue:
 *   o[b][vh][i] = (r[i] * s * norm_w[i]) * silu(z[b][vh][i]),
 *   s = 1 / sqrtf((float)(sum_i r[i]^2 / hd) + 1e-6f)   (sum in double)
 * with r the delta-rule retrieve output of (b, vh).
 *   z       [B][nv][hd] (act dtype), the in_proj_z projection
 *   norm_w  [hd] fp32 (linear_attn.norm.weight, shared by all V heads)
 * Other arguments and flags as vx27_deltanet_decode_batch. No counterpart in the
 * reference's headers (the reference does this inline in vx27_qlayer).
 */
int vx27_deltanet_decode_batch_gated(float *S, float *conv_ring, const void *qkv,
                                     const void *a, const void *b, const float *A_log,
                                     const float *dt_bias, const float *conv_w, const int *pos,
                                     const void *z, const float *norm_w, void *o, int B,
                                     int nqk, int nv, int hd, int flags, void *stream,
                                     char *err, size_t errlen);

/*
 * The gates of vx27_deltanet_decode_batch / _prefill_chunked as the device computes them
 * (no counterpart in the reference; it exists to measure them against
 * vx27_deltanet_gate_params, src/vx27_deltanet.c:58-69). For item i with head vh = i % nv:
 * beta[i], g_log[i] in double from a[i], b[i] (act dtype), A_log[vh], dt_bias[vh] with
 * the device exp/log, and beta_f32[i] = (float)beta[i], decay_f32[i] = (float)exp(g_log[i]),
 * the two values the fp32 update uses. Any output may be NULL. The double values can
 * differ from the host function's in the last bit (neither side's exp/log is correctly
 * rounded on every input); VX27_F_GATES_F64 feeds the host's bits to the kernels instead.
 * Flags: VX27_F_ACT_BF16.
 */
int vx27_deltanet_gate_params_dev(const void *a, const void *b, const float *A_log,
                                  const float *dt_bias, double *beta, double *g_log,
                                  float *beta_f32, float *decay_f32, int n, int nv, int flags,
                                  void *stream, char *err, size_t errlen);

/*
 * T consecutive tokens of ONE sequence through one DeltaNet layer (teacher-forced
 * verification of speculative drafts), with optional snapshots after every token for a
 * partial commit: the semantics of vx27_qlayer_batch's Sckpt/Cckpt
 * (src/vx27_qfwd.h:39-50, src/vx27_qfwd.c:306-307).
 *   S [nv][hd][hd], conv_ring [4][C] (device, this sequence); qkv [T][C], a, b [T][nv]
 *   (act dtype); pos [T] device int, the tokens' positions (normally pos0 + t);
 *   o [T][nv][hd];
 *   S_ckpt    [T][nv][hd][hd] fp32 or NULL: the state after token t
 *   conv_ckpt [T][C][3] fp32 or NULL: the conv history after token t in the reference
 *             layout (oldest first; vx27_deltanet_conv_import restores it)
 * Flags as vx27_deltanet_decode_batch (VX27_F_QK_PRENORM excluded). One kernel runs all T
 * tokens with the state held on chip (8 CTAs per head, 16 state columns each), then a
 * small kernel brings the conv ring up to date; each position sequence gives the result
 * of T single-token calls. Runs on `stream` without synchronising.
 */
int vx27_deltanet_decode_tokens(float *S, float *conv_ring, const void *qkv, const void *a,
                                const void *b, const float *A_log, const float *dt_bias,
                                const float *conv_w, const int *pos, void *o, float *S_ckpt,
                                float *conv_ckpt, int T, int nqk, int nv, int hd, int flags,
                                void *stream, char *err, size_t errlen);

/*
 * Chunked gated delta rule over T prompt tokens (config 4): the token-by-token recurrence
 * of vx27_deltanet_step_exact (l2-normalised q and k, q / sqrt(hd), gates of
 * vx27_deltanet_gate_params) evaluated 64 tokens at a time in the WY/UT form, within
 * 1e-3 of the recurrent reference over 32768 tokens.
 *   q, k [T][nqk][hd], v [T][nv][hd], a, b [T][nv] (act dtype; VX27_F_GATES_F64: a/b are
 *   host-computed beta/g_log as double); A_log, dt_bias [nv] fp32
 *   S [nv][hd][hd] fp32: initial state in, final state out
 *   o [T][nv][hd] (fp32, or bf16 with VX27_F_OUT_BF16)
 *   workspace: vx27_deltanet_prefill_workspace_size(T, nqk, nv, hd) bytes
 * hd must be 128; V head vh reads QK head vh*nqk/nv.
 */
size_t vx27_deltanet_prefill_workspace_size(int T, int nqk, int nv, int hd);
int vx27_deltanet_prefill_chunked(const void *q, const void *k, const void *v, const void *a,
                                  const void *b, const float *A_log, const float *dt_bias,
                                  float *S, void *o, void *workspace, size_t workspace_bytes,
                                  int T, int nqk, int nv, int hd, int flags, void *stream,
                                  char *err, size_t errlen);

/* Conv history conversion between the reference layout state[B][C][3] (host, oldest
 * first) and the device ring [B][4][C] at positions pos[B] (host array). */
int vx27_deltanet_conv_import(float *conv_ring, const float *state, const int *pos, int B,
                              int C, void *stream, char *err, size_t errlen);
int vx27_deltanet_conv_export(const float *conv_ring, float *state, const int *pos, int B,
                              int C, void *stream, char *err, size_t errlen);

#ifdef __cplusplus
}
#endif
#endif
