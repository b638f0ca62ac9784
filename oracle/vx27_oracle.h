/*
 * vx27 oracle -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C CPU restatement of the vx27 attention hot path (Gated DeltaNet decode,
 * gated GQA decode over a BF16 KV cache, partial RoPE, the LSE combine of split-KV
 * partials and the recurrent reference for chunked prefill). It is the parity
 * checker for the CUDA library in vx27_b200/ and the CPU baseline of bench.py.
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference leg
 * may load it. The product library never links or calls anything here.
 *
 * Every function names the reference file:line (DavidPandleton/vx27) it restates.
 * Parity of this restatement is pinned two ways (tests/test_oracle_pins.py):
 *   1. against the reference's own known-answer tests (tests/test_deltanet_exact.c,
 *      test_gqa.c, test_rope.c, test_kv.c, test_deltanet.c), and
 *   2. against golden vectors produced by the reference's own sources compiled
 *      unmodified into oracle/_ref/ (script: tests/golden/make_golden.py).
 *
 * Build flags mirror the reference Makefile (-std=c11, i.e. no FP contraction).
 */
#ifndef VX27_ORACLE_H
#define VX27_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- element formats ---------------------------------------------------- */
uint16_t orc_f32_to_bf16(float x);          /* round to nearest even, NaN kept quiet */
float    orc_bf16_to_f32(uint16_t h);

/* ---- Gated DeltaNet (src/vx27_deltanet.c) -------------------------------- */
void orc_update_ref(float *S, const float *k, const float *v, float decay, int hd);
void orc_retrieve_ref(const float *S, const float *q, float *o, int hd);
void orc_l2norm(const float *x, float *y, int n);
double orc_softplus(double x);
void orc_gate_params(double a, double A_log, double b, double dt_bias,
                     double *beta, double *g_log);
void orc_step_exact(float *S, const float *q, const float *k, const float *v,
                    double beta, double g_log, float *o, int hd);
void orc_conv1d_step(float *state, const float *x, const float *w, float *y,
                     int C, int apply_silu);

/* ---- GQA + RoPE (src/vx27_gqa.c, src/vx27_rope.c, src/vx27_kv.c) -------- */
int  orc_kv_for_q(int q_head, int n_q, int n_kv);
void orc_rmsnorm(const float *x, const float *w, float *y, int n, float eps, int one_plus);
void orc_rope_cos_sin(int pos, float *cosv, float *sinv, int rope_dim, float theta,
                      float yarn_factor);
void orc_rope_apply(float *v, int n_heads, int head_dim, int rope_dim,
                    const float *cosv, const float *sinv);
void orc_attn_1q(const float *q, const float *kcache, const float *vcache, int n_pos,
                 int n_q, int n_kv, int hd, float *out);
uint64_t orc_kv_elems(int ctx);
double   orc_kv_gb(int ctx, double bytes_per_elem);

/* ---- batched drivers with the CUDA performance tier's exact semantics ---- */
/* flags, identical values to include/vx27cuda.h */
#define ORC_F_ACT_BF16 0x1
#define ORC_F_OUT_BF16 0x2
#define ORC_F_NORM_1P  0x4

/* One decode step of one DeltaNet layer for B sequences.
 *   S      [B][nv][hd][hd] fp32 (in/out)
 *   ring   [B][4][C] fp32 conv history, slot p%4 holds the input of token p (in/out)
 *   qkv    [B][C] pre-conv activations, C = (2*nqk+nv)*hd, channels q|k|v
 *   a, b   [B][nv] gate logits;  A_log, dt_bias [nv];  conv_w [C][4]
 *   pos    [B] tokens already consumed;  o [B][nv][hd]
 * Per sequence this is src/vx27_qfwd.c:276-297 without the projections and QK-norm:
 * conv1d_step -> gate_params -> step_exact per V head (V head vh reads QK head vh*nqk/nv).
 * step_fn/conv_fn/gate_fn may be NULL (restatement) or the reference's own symbols. */
typedef void (*orc_step_fn)(float *, const float *, const float *, const float *,
                            double, double, float *, int);
typedef void (*orc_conv_fn)(float *, const float *, const float *, float *, int, int);
typedef void (*orc_gate_fn)(double, double, double, double, double *, double *);

void orc_deltanet_decode_batch(float *S, float *ring, const void *qkv, const void *a,
                               const void *b, const float *A_log, const float *dt_bias,
                               const float *conv_w, const int *pos, void *o,
                               int B, int nqk, int nv, int hd, int flags);

/* GQA append: QK RMSNorm + partial RoPE at pos[b], BF16 store of K/V at slot pos[b].
 *   q_in [B][nq][hd], k_in/v_in [B][nkv][hd] (act dtype); q_out [B][nq][hd] fp32
 *   kc/vc bf16 [B][nkv][cap][hd].  Follows src/vx27_qfwd.c:339-346. */
void orc_gqa_append(const void *q_in, const void *k_in, const void *v_in,
                    const float *q_norm_w, const float *k_norm_w, const int *pos,
                    uint16_t *kc, uint16_t *vc, int cap, float *q_out,
                    int B, int nq, int nkv, int hd, int rope_dim, float theta,
                    float eps, int flags);

/* GQA decode attention over positions [0, pos[b]] of a BF16 cache, then the sigmoid
 * output gate. out [B][nq][hd] (fp32 or bf16 per flags).  src/vx27_qfwd.c:347-371. */
void orc_gqa_attend(const float *q, const void *gate, const uint16_t *kc,
                    const uint16_t *vc, int cap, const int *pos, void *out,
                    int B, int nq, int nkv, int hd, int flags);

/* Split-KV partial over positions [p0, p1) of one sequence (all nq heads):
 * m = max scaled score, l = sum exp(s - m), o = (sum exp(s - m) v) / l.
 * Record layout per part: o[nq][hd] then ml[nq][2]. Empty range: m=-inf, l=0, o=0. */
void orc_gqa_partial(const float *q, const uint16_t *kc, const uint16_t *vc, int cap,
                     int p0, int p1, float *o_part, float *ml_part,
                     int nq, int nkv, int hd);
/* LSE combine of n_parts partial records + sigmoid gate. */
void orc_gqa_combine(const float *o_parts, const float *ml_parts, int n_parts,
                     const void *gate, void *out, int nq, int hd, int flags);

/* Recurrent (token-by-token) gated delta rule over T tokens for one head; the
 * reference for chunked prefill.  q,k,v [T][hd] (act dtype, row stride ld elems),
 * beta/g_log [T]; S [hd][hd] in/out; o [T][hd] fp32. */
void orc_deltanet_recurrent(float *S, const void *q, const void *k, const void *v,
                            long ld, const double *beta, const double *g_log,
                            float *o, int T, int hd, int flags);

/* Gated RMSNorm output of a DeltaNet layer (src/vx27_qfwd.c:146-151): per head of hd,
 * y = rmsn_std(x) * w * silu(z). */
void orc_gated_rmsnorm(const float *x, const float *w, const float *z, float *y, int n_heads,
                       int hd);

/* gate_params (the selected implementation) over a [T][nv] grid of fp32 logits. */
void orc_gate_params_grid(const float *a, const float *b, const float *A_log,
                          const float *dt_bias, int T, int nv, double *beta, double *g_log);

/* Causal gated GQA prefill reference for selected query rows.
 * q,k,v [T][heads][hd] raw (act dtype); rows[n_rows]; out [n_rows][nq][hd] fp32. */
void orc_gqa_prefill_rows(const void *q, const void *k, const void *v, const void *gate,
                          const float *q_norm_w, const float *k_norm_w,
                          int T, int nq, int nkv, int hd, int rope_dim, float theta,
                          float eps, const int *rows, int n_rows, float *out, int flags);

/* ---- packed-weight matvec (src/vx27_pmat.c) ------------------------------- */
/* yb[b*rows + r] = W[r] . xb[b*cols ..] for b < B, per the reference's arithmetic:
 * dtype 0 F32 rows, double accumulation over columns (src/vx27_pmat.c:96-99, 196-204);
 * dtype 2 Q8_K blocks of 256 (float d, int8 qs[256], int16 bsums[16]; 292 B): per block
 *   eight fp32 FMA lanes (lane l takes columns l, l+8, ...), lanes summed left to right,
 *   times d in double, accumulated in double (:10-24, :100-105, :187-195);
 * dtype 4 BP3_128 groups of 128 (three planes of 4 u32 + fp16 scale, 52 B in memory):
 *   eight fp32 FMA lanes over the whole row with q*scale formed by one multiply, lanes
 *   summed left to right at the end (:28-63, :133-177).
 * cols must be a multiple of 256 (Q8_K) or 128 (BP3_128). */
float orc_bp3_scale(uint16_t h);  /* the reference's fp16 -> fp32 of the group scale */
void orc_pmat_batch(const void *W, uint32_t dtype, const float *xb, float *yb, int rows,
                    int cols, int B);

/* ---- seeded synthetic inputs (same formula as vx27_b200/csrc/synth.cu) --- */
uint64_t orc_splitmix64(uint64_t x);
void orc_fill_normal_f32(float *x, size_t n, uint64_t seed, uint64_t stream,
                         float mean, float std);
void orc_fill_normal_bf16(uint16_t *x, size_t n, uint64_t seed, uint64_t stream,
                          float mean, float std);
void orc_fill_uniform_f32(float *x, size_t n, uint64_t seed, uint64_t stream,
                          float lo, float hi);

/* ---- CPU baseline (threaded; reference functions when available) -------- */
/* Selects the implementation of step_exact / conv1d_step / gate_params / rmsnorm /
 * rope used by the drivers above: NULL path -> this restatement; otherwise the
 * shared library built from the reference's own sources (oracle/_ref). Returns 0 on
 * success, -1 if the library or a symbol is missing. */
int  orc_use_reference(const char *ref_so_path);
int  orc_impl_is_reference(void);
/* Threaded variants: work items are (sequence, head) pairs spread over n_threads. */
void orc_deltanet_decode_batch_mt(float *S, float *ring, const void *qkv, const void *a,
                                  const void *b, const float *A_log, const float *dt_bias,
                                  const float *conv_w, const int *pos, void *o,
                                  int B, int nqk, int nv, int hd, int flags, int n_threads);
void orc_gqa_attend_mt(const float *q, const void *gate, const uint16_t *kc,
                       const uint16_t *vc, int cap, const int *pos, void *out,
                       int B, int nq, int nkv, int hd, int flags, int n_threads);

#ifdef __cplusplus
}
#endif
#endif
