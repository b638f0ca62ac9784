/*
 * vx27 oracle -- TEST INFRASTRUCTURE ONLY (see vx27_oracle.h).
 * CPU restatement of the vx27 attention hot path; each function cites the reference
 * file:line (DavidPandleton/vx27) whose arithmetic it restates, in the same operation
 * order, so that with the reference's build flags (-std=c11: no FP contraction) it is
 * bit-identical to the reference where the reference has a callable function.
 */
#define _GNU_SOURCE
#include "vx27_oracle.h"
#include "threadpool.h"
#include <dlfcn.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------- formats */
uint16_t orc_f32_to_bf16(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
float orc_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float x;
    memcpy(&x, &u, 4);
    return x;
}
static inline float act_load(const void *p, size_t i, int bf16) {
    return bf16 ? orc_bf16_to_f32(((const uint16_t *)p)[i]) : ((const float *)p)[i];
}
static inline void act_store(void *p, size_t i, float x, int bf16) {
    if (bf16) ((uint16_t *)p)[i] = orc_f32_to_bf16(x);
    else ((float *)p)[i] = x;
}

/* ------------------------------------------------------- Gated DeltaNet */
/* src/vx27_deltanet.c:15-20 */
void orc_update_ref(float *S, const float *k, const float *v, float decay, int hd) {
    for (int i = 0; i < hd; i++)
        for (int j = 0; j < hd; j++) {
            float t = decay * S[i * hd + j];
            S[i * hd + j] = t + k[i] * v[j];
        }
}
/* src/vx27_deltanet.c:21-28 */
void orc_retrieve_ref(const float *S, const float *q, float *o, int hd) {
    for (int j = 0; j < hd; j++) {
        float acc = 0.0f;
        for (int i = 0; i < hd; i++) acc += S[i * hd + j] * q[i];
        o[j] = acc;
    }
}
/* src/vx27_deltanet.c:51-56: sum of squares in double, eps 1e-6 inside the sqrt, no /n */
void orc_l2norm(const float *x, float *y, int n) {
    double ss = 0.0;
    for (int i = 0; i < n; i++) ss += (double)x[i] * (double)x[i];
    float r = 1.0f / sqrtf((float)ss + 1e-6f);
    for (int i = 0; i < n; i++) y[i] = x[i] * r;
}
/* src/vx27_deltanet.c:58-63: three-regime softplus */
double orc_softplus(double x) {
    if (x > 20.0) return x;
    if (x < -20.0) return exp(x);
    return log(1.0 + exp(x));
}
/* src/vx27_deltanet.c:65-69: beta = sigmoid(b) (no dt_bias); g = -exp(A_log)*softplus(a+dt) */
void orc_gate_params(double a, double A_log, double b, double dt_bias,
                     double *beta, double *g_log) {
    if (beta) *beta = 1.0 / (1.0 + exp(-b));
    if (g_log) *g_log = -exp(A_log) * orc_softplus(a + dt_bias);
}
/* src/vx27_deltanet.c:71-102: one exact gated delta-rule step for one V head.
 * Column sums accumulate in double; S is rounded to float after the decay and after
 * the rank-1 update, exactly as the reference stores it. */
void orc_step_exact(float *S, const float *q, const float *k, const float *v,
                    double beta, double g_log, float *o, int hd) {
    float qn[256], kn[256];
    double kv[256];
    orc_l2norm(q, qn, hd);
    orc_l2norm(k, kn, hd);
    const float qscale = 1.0f / sqrtf((float)hd);
    for (int i = 0; i < hd; i++) qn[i] *= qscale;
    const double decay = exp(g_log);
    for (int e = 0; e < hd * hd; e++) S[e] = (float)((double)S[e] * decay);
    for (int j = 0; j < hd; j++) {
        double acc = 0.0;
        for (int i = 0; i < hd; i++) acc += (double)S[i * hd + j] * kn[i];
        kv[j] = acc;
    }
    for (int i = 0; i < hd; i++) {
        const double ki = kn[i];
        for (int j = 0; j < hd; j++) {
            double d = ((double)v[j] - kv[j]) * beta;
            S[i * hd + j] = (float)((double)S[i * hd + j] + ki * d);
        }
    }
    for (int j = 0; j < hd; j++) {
        double acc = 0.0;
        for (int i = 0; i < hd; i++) acc += (double)S[i * hd + j] * qn[i];
        o[j] = (float)acc;
    }
}
/* src/vx27_deltanet.c:104-122: depthwise causal conv, width 4, tap 0 = oldest sample */
void orc_conv1d_step(float *state, const float *x, const float *w, float *y,
                     int C, int apply_silu) {
    for (int c = 0; c < C; c++) {
        const float *wc = w + (size_t)c * 4;
        float *st = state + (size_t)c * 3;
        float acc = wc[0] * st[0];
        acc = acc + wc[1] * st[1];
        acc = acc + wc[2] * st[2];
        acc = acc + wc[3] * x[c];
        y[c] = apply_silu ? acc / (1.0f + expf(-acc)) : acc;
        st[0] = st[1];
        st[1] = st[2];
        st[2] = x[c];
    }
}

/* ------------------------------------------------------------- GQA/RoPE */
/* src/vx27_gqa.c:6-8 */
int orc_kv_for_q(int q_head, int n_q, int n_kv) { return q_head * n_kv / n_q; }
/* src/vx27_gqa.c:10-15 (one_plus=0); zero-centred form of src/vx27_qfwd.c:32-39 (one_plus=1) */
void orc_rmsnorm(const float *x, const float *w, float *y, int n, float eps, int one_plus) {
    double ss = 0.0;
    for (int i = 0; i < n; i++) ss += (double)x[i] * (double)x[i];
    float r = 1.0f / sqrtf((float)(ss / n) + eps);
    for (int i = 0; i < n; i++) {
        float wi = one_plus ? w[i] + 1.0f : w[i];
        y[i] = x[i] * r * wi;
    }
}
/* src/vx27_rope.c:5-16: powf/cosf/sinf in float, linear YaRN position scaling */
void orc_rope_cos_sin(int pos, float *cosv, float *sinv, int rope_dim, float theta,
                      float yarn_factor) {
    if (yarn_factor < 1.0f) yarn_factor = 1.0f;
    const float p = (float)pos / yarn_factor;
    const int half = rope_dim / 2;
    for (int i = 0; i < half; i++) {
        float freq = powf(theta, -2.0f * (float)i / (float)rope_dim);
        float ang = p * freq;
        cosv[i] = cosf(ang);
        sinv[i] = sinf(ang);
    }
}
/* src/vx27_rope.c:18-29: NeoX half-split rotation of the first rope_dim dims */
void orc_rope_apply(float *v, int n_heads, int head_dim, int rope_dim,
                    const float *cosv, const float *sinv) {
    const int half = rope_dim / 2;
    for (int h = 0; h < n_heads; h++) {
        float *x = v + (size_t)h * head_dim;
        for (int i = 0; i < half; i++) {
            float a = x[i], b = x[i + half];
            x[i] = a * cosv[i] - b * sinv[i];
            x[i + half] = a * sinv[i] + b * cosv[i];
        }
    }
}
/* src/vx27_gqa.c:17-45 without the 1024-position static buffer */
void orc_attn_1q(const float *q, const float *kcache, const float *vcache, int n_pos,
                 int n_q, int n_kv, int hd, float *out) {
    const float scale = 1.0f / sqrtf((float)hd);
    float *sc = (float *)malloc((size_t)(n_pos > 0 ? n_pos : 1) * sizeof(float));
    for (int h = 0; h < n_q; h++) {
        const int kvh = orc_kv_for_q(h, n_q, n_kv);
        const float *qh = q + (size_t)h * hd;
        float smax = -1e30f, ssum = 0.0f;
        for (int p = 0; p < n_pos; p++) {
            const float *kh = kcache + ((size_t)p * n_kv + kvh) * hd;
            float s = 0.0f;
            for (int i = 0; i < hd; i++) s += qh[i] * kh[i];
            s *= scale;
            sc[p] = s;
            if (s > smax) smax = s;
        }
        for (int p = 0; p < n_pos; p++) { sc[p] = expf(sc[p] - smax); ssum += sc[p]; }
        float *oh = out + (size_t)h * hd;
        for (int i = 0; i < hd; i++) oh[i] = 0.0f;
        for (int p = 0; p < n_pos; p++) {
            const float a = sc[p] / ssum;
            const float *vh = vcache + ((size_t)p * n_kv + kvh) * hd;
            for (int i = 0; i < hd; i++) oh[i] += a * vh[i];
        }
    }
    free(sc);
}
/* src/vx27_kv.c:4-9 */
uint64_t orc_kv_elems(int ctx) { return (uint64_t)32768 * (uint64_t)ctx; }
double orc_kv_gb(int ctx, double bytes_per_elem) {
    return (double)orc_kv_elems(ctx) * bytes_per_elem / 1e9;
}

/* --------------------------------------- implementation selection (baseline) */
static orc_step_fn g_step = orc_step_exact;
static orc_conv_fn g_conv = orc_conv1d_step;
static orc_gate_fn g_gate = orc_gate_params;
typedef void (*orc_rms_fn)(const float *, const float *, float *, int, float);
typedef void (*orc_rcs_fn)(int, float *, float *, int, float, float);
typedef void (*orc_rap_fn)(float *, int, int, int, const float *, const float *);
static orc_rms_fn g_rms = NULL; /* NULL: restatement */
static orc_rcs_fn g_rcs = orc_rope_cos_sin;
static orc_rap_fn g_rap = orc_rope_apply;
static int g_is_ref = 0;

int orc_use_reference(const char *path) {
    if (!path) {
        g_step = orc_step_exact; g_conv = orc_conv1d_step; g_gate = orc_gate_params;
        g_rms = NULL; g_rcs = orc_rope_cos_sin; g_rap = orc_rope_apply; g_is_ref = 0;
        return 0;
    }
    void *h = dlopen(path, RTLD_NOW | RTLD_LOCAL);
    if (!h) return -1;
    void *s = dlsym(h, "vx27_deltanet_step_exact"), *c = dlsym(h, "vx27_conv1d_step");
    void *g = dlsym(h, "vx27_deltanet_gate_params"), *r = dlsym(h, "vx27_rmsnorm");
    void *rc = dlsym(h, "vx27_rope_cos_sin"), *ra = dlsym(h, "vx27_rope_apply");
    if (!s || !c || !g || !r || !rc || !ra) return -1;
    g_step = (orc_step_fn)s; g_conv = (orc_conv_fn)c; g_gate = (orc_gate_fn)g;
    g_rms = (orc_rms_fn)r; g_rcs = (orc_rcs_fn)rc; g_rap = (orc_rap_fn)ra;
    g_is_ref = 1;
    return 0;
}
int orc_impl_is_reference(void) { return g_is_ref; }

static void rms_dispatch(const float *x, const float *w, float *y, int n, float eps,
                         int one_plus) {
    if (g_rms && !one_plus) g_rms(x, w, y, n, eps);
    else orc_rmsnorm(x, w, y, n, eps, one_plus);
}

/* ------------------------------------------------------ batched DeltaNet */
/* One sequence of orc_deltanet_decode_batch; heads [h0, h1). The conv of all C
 * channels runs when h0 == 0 (the ring slot write happens exactly once). */
typedef struct {
    float *S, *ring;
    const void *qkv, *a, *b;
    const float *A_log, *dt_bias, *conv_w;
    const int *pos;
    void *o;
    int B, nqk, nv, hd, flags;
} dn_job;

static void dn_conv_seq(const dn_job *j, int bi, float *y) {
    const int C = (2 * j->nqk + j->nv) * j->hd;
    const int bf = j->flags & ORC_F_ACT_BF16;
    const int t = j->pos[bi];
    float *ring = j->ring + (size_t)bi * 4 * C;
    float *st = (float *)malloc((size_t)C * 3 * sizeof(float));
    float *x = (float *)calloc((size_t)C, sizeof(float));
    for (int c = 0; c < C; c++) {
        st[(size_t)c * 3 + 0] = ring[(size_t)((t - 3) & 3) * C + c];
        st[(size_t)c * 3 + 1] = ring[(size_t)((t - 2) & 3) * C + c];
        st[(size_t)c * 3 + 2] = ring[(size_t)((t - 1) & 3) * C + c];
        x[c] = act_load(j->qkv, (size_t)bi * C + c, bf);
    }
    g_conv(st, x, j->conv_w, y, C, 1);
    for (int c = 0; c < C; c++) ring[(size_t)(t & 3) * C + c] = x[c];
    free(st);
    free(x);
}

static void dn_heads_seq(const dn_job *j, int bi, const float *y, int h0, int h1) {
    const int hd = j->hd, nqk = j->nqk, nv = j->nv;
    const int bf = j->flags & ORC_F_ACT_BF16, obf = j->flags & ORC_F_OUT_BF16;
    float ov[256];
    for (int vh = h0; vh < h1; vh++) {
        const int qk = vh * nqk / nv;
        double beta, g;
        g_gate((double)act_load(j->a, (size_t)bi * nv + vh, bf), (double)j->A_log[vh],
               (double)act_load(j->b, (size_t)bi * nv + vh, bf), (double)j->dt_bias[vh],
               &beta, &g);
        float *S = j->S + ((size_t)bi * nv + vh) * hd * hd;
        g_step(S, y + (size_t)qk * hd, y + (size_t)(nqk + qk) * hd,
               y + (size_t)(2 * nqk) * hd + (size_t)vh * hd, beta, g, ov, hd);
        for (int i = 0; i < hd; i++)
            act_store(j->o, ((size_t)bi * nv + vh) * hd + i, ov[i], obf);
    }
}

void orc_deltanet_decode_batch(float *S, float *ring, const void *qkv, const void *a,
                               const void *b, const float *A_log, const float *dt_bias,
                               const float *conv_w, const int *pos, void *o,
                               int B, int nqk, int nv, int hd, int flags) {
    dn_job j = {S, ring, qkv, a, b, A_log, dt_bias, conv_w, pos, o, B, nqk, nv, hd, flags};
    const int C = (2 * nqk + nv) * hd;
    float *y = (float *)malloc((size_t)C * sizeof(float));
    for (int bi = 0; bi < B; bi++) {
        dn_conv_seq(&j, bi, y);
        dn_heads_seq(&j, bi, y, 0, nv);
    }
    free(y);
}

typedef struct { dn_job j; float *ybuf; int C; } dn_mt;
static void dn_conv_worker(void *arg, int tid, int n) {
    dn_mt *m = (dn_mt *)arg;
    for (int bi = tid; bi < m->j.B; bi += n) dn_conv_seq(&m->j, bi, m->ybuf + (size_t)bi * m->C);
}
static void dn_head_worker(void *arg, int tid, int n) {
    dn_mt *m = (dn_mt *)arg;
    const long items = (long)m->j.B * m->j.nv;
    for (long it = tid; it < items; it += n) {
        int bi = (int)(it / m->j.nv), vh = (int)(it % m->j.nv);
        dn_heads_seq(&m->j, bi, m->ybuf + (size_t)bi * m->C, vh, vh + 1);
    }
}
static threadpool *g_tp = NULL;
static int g_tp_n = 0;
static threadpool *pool(int n) {
    if (n < 1) n = 1;
    if (g_tp && g_tp_n == n) return g_tp;
    if (g_tp) tp_free(g_tp);
    char err[128];
    g_tp = tp_create(n, err, sizeof err);
    g_tp_n = g_tp ? n : 0;
    return g_tp;
}
void orc_deltanet_decode_batch_mt(float *S, float *ring, const void *qkv, const void *a,
                                  const void *b, const float *A_log, const float *dt_bias,
                                  const float *conv_w, const int *pos, void *o,
                                  int B, int nqk, int nv, int hd, int flags, int n_threads) {
    dn_mt m = {{S, ring, qkv, a, b, A_log, dt_bias, conv_w, pos, o, B, nqk, nv, hd, flags},
               NULL, (2 * nqk + nv) * hd};
    m.ybuf = (float *)malloc((size_t)B * m.C * sizeof(float));
    threadpool *tp = pool(n_threads);
    tp_run(tp, dn_conv_worker, &m);
    tp_run(tp, dn_head_worker, &m);
    free(m.ybuf);
}

/* ------------------------------------------------------------ batched GQA */
void orc_gqa_append(const void *q_in, const void *k_in, const void *v_in,
                    const float *q_norm_w, const float *k_norm_w, const int *pos,
                    uint16_t *kc, uint16_t *vc, int cap, float *q_out,
                    int B, int nq, int nkv, int hd, int rope_dim, float theta,
                    float eps, int flags) {
    const int bf = flags & ORC_F_ACT_BF16, one_plus = (flags & ORC_F_NORM_1P) ? 1 : 0;
    float cosv[128], sinv[128];
    float *t = (float *)malloc((size_t)hd * sizeof(float));
    float *x = (float *)malloc((size_t)hd * sizeof(float));
    for (int bi = 0; bi < B; bi++) {
        const int p = pos[bi];
        g_rcs(p, cosv, sinv, rope_dim, theta, 1.0f);
        for (int h = 0; h < nq; h++) {
            for (int i = 0; i < hd; i++) x[i] = act_load(q_in, ((size_t)bi * nq + h) * hd + i, bf);
            rms_dispatch(x, q_norm_w, t, hd, eps, one_plus);
            g_rap(t, 1, hd, rope_dim, cosv, sinv);
            memcpy(q_out + ((size_t)bi * nq + h) * hd, t, (size_t)hd * sizeof(float));
        }
        for (int h = 0; h < nkv; h++) {
            for (int i = 0; i < hd; i++) x[i] = act_load(k_in, ((size_t)bi * nkv + h) * hd + i, bf);
            rms_dispatch(x, k_norm_w, t, hd, eps, one_plus);
            g_rap(t, 1, hd, rope_dim, cosv, sinv);
            size_t base = (((size_t)bi * nkv + h) * cap + p) * hd;
            for (int i = 0; i < hd; i++) {
                kc[base + i] = orc_f32_to_bf16(t[i]);
                vc[base + i] = orc_f32_to_bf16(act_load(v_in, ((size_t)bi * nkv + h) * hd + i, bf));
            }
        }
    }
    free(t);
    free(x);
}

/* One (sequence, Q head) of the decode attention: src/vx27_qfwd.c:350-371 with a heap
 * score buffer; scores use a double dot product rounded to float, as the reference. */
static void attend_one(const float *q, const void *gate, const uint16_t *kc,
                       const uint16_t *vc, int cap, const int *pos, void *out, int nq,
                       int nkv, int hd, int flags, int bi, int h, float *sc) {
    const int bf = flags & ORC_F_ACT_BF16, obf = flags & ORC_F_OUT_BF16;
    const int kvh = orc_kv_for_q(h, nq, nkv);
    const int n = pos[bi] + 1;
    const float scl = 1.0f / sqrtf((float)hd);
    const float *qh = q + ((size_t)bi * nq + h) * hd;
    const uint16_t *K = kc + ((size_t)bi * nkv + kvh) * cap * hd;
    const uint16_t *V = vc + ((size_t)bi * nkv + kvh) * cap * hd;
    float smax = -1e30f, ssum = 0.0f;
    for (int p = 0; p < n; p++) {
        double s = 0.0;
        for (int i = 0; i < hd; i++) s += (double)qh[i] * (double)orc_bf16_to_f32(K[(size_t)p * hd + i]);
        sc[p] = (float)(s * scl);
        if (sc[p] > smax) smax = sc[p];
    }
    for (int p = 0; p < n; p++) { sc[p] = expf(sc[p] - smax); ssum += sc[p]; }
    float oh[512];
    for (int i = 0; i < hd; i++) oh[i] = 0.0f;
    for (int p = 0; p < n; p++) {
        const float a = sc[p] / ssum;
        for (int i = 0; i < hd; i++) oh[i] += a * orc_bf16_to_f32(V[(size_t)p * hd + i]);
    }
    for (int i = 0; i < hd; i++) {
        size_t idx = ((size_t)bi * nq + h) * hd + i;
        /* gate NULL: no output gate (src/vx27_mtp.c:249, use_gate = 0) */
        const float gf = gate ? 1.0f / (1.0f + expf(-act_load(gate, idx, bf))) : 1.0f;
        act_store(out, idx, gate ? oh[i] * gf : oh[i], obf);
    }
}

void orc_gqa_attend(const float *q, const void *gate, const uint16_t *kc,
                    const uint16_t *vc, int cap, const int *pos, void *out,
                    int B, int nq, int nkv, int hd, int flags) {
    float *sc = (float *)malloc((size_t)cap * sizeof(float));
    for (int bi = 0; bi < B; bi++)
        for (int h = 0; h < nq; h++)
            attend_one(q, gate, kc, vc, cap, pos, out, nq, nkv, hd, flags, bi, h, sc);
    free(sc);
}

typedef struct {
    const float *q; const void *gate; const uint16_t *kc, *vc; int cap; const int *pos;
    void *out; int B, nq, nkv, hd, flags;
} at_job;
static void at_worker(void *arg, int tid, int n) {
    at_job *j = (at_job *)arg;
    float *sc = (float *)malloc((size_t)j->cap * sizeof(float));
    const long items = (long)j->B * j->nq;
    for (long it = tid; it < items; it += n)
        attend_one(j->q, j->gate, j->kc, j->vc, j->cap, j->pos, j->out, j->nq, j->nkv,
                   j->hd, j->flags, (int)(it / j->nq), (int)(it % j->nq), sc);
    free(sc);
}
void orc_gqa_attend_mt(const float *q, const void *gate, const uint16_t *kc,
                       const uint16_t *vc, int cap, const int *pos, void *out,
                       int B, int nq, int nkv, int hd, int flags, int n_threads) {
    at_job j = {q, gate, kc, vc, cap, pos, out, B, nq, nkv, hd, flags};
    tp_run(pool(n_threads), at_worker, &j);
}

void orc_gqa_partial(const float *q, const uint16_t *kc, const uint16_t *vc, int cap,
                     int p0, int p1, float *o_part, float *ml_part,
                     int nq, int nkv, int hd) {
    const float scl = 1.0f / sqrtf((float)hd);
    const int n = p1 > p0 ? p1 - p0 : 0;
    float *sc = (float *)malloc((size_t)(n > 0 ? n : 1) * sizeof(float));
    for (int h = 0; h < nq; h++) {
        const int kvh = orc_kv_for_q(h, nq, nkv);
        const float *qh = q + (size_t)h * hd;
        const uint16_t *K = kc + (size_t)kvh * cap * hd, *V = vc + (size_t)kvh * cap * hd;
        float *oh = o_part + (size_t)h * hd;
        for (int i = 0; i < hd; i++) oh[i] = 0.0f;
        if (n == 0) { ml_part[2 * h] = -INFINITY; ml_part[2 * h + 1] = 0.0f; continue; }
        float smax = -INFINITY, ssum = 0.0f;
        for (int p = 0; p < n; p++) {
            double s = 0.0;
            for (int i = 0; i < hd; i++)
                s += (double)qh[i] * (double)orc_bf16_to_f32(K[(size_t)(p0 + p) * hd + i]);
            sc[p] = (float)(s * scl);
            if (sc[p] > smax) smax = sc[p];
        }
        for (int p = 0; p < n; p++) { sc[p] = expf(sc[p] - smax); ssum += sc[p]; }
        for (int p = 0; p < n; p++) {
            const float a = sc[p] / ssum;
            for (int i = 0; i < hd; i++) oh[i] += a * orc_bf16_to_f32(V[(size_t)(p0 + p) * hd + i]);
        }
        ml_part[2 * h] = smax;
        ml_part[2 * h + 1] = ssum;
    }
    free(sc);
}

/* m* = max m_i; l* = sum l_i e^{m_i - m*}; o = sum o_i l_i e^{m_i - m*} / l*; then gate */
void orc_gqa_combine(const float *o_parts, const float *ml_parts, int n_parts,
                     const void *gate, void *out, int nq, int hd, int flags) {
    const int bf = flags & ORC_F_ACT_BF16, obf = flags & ORC_F_OUT_BF16;
    for (int h = 0; h < nq; h++) {
        double m = -INFINITY;
        for (int r = 0; r < n_parts; r++) {
            const float *ml = ml_parts + (size_t)r * nq * 2;
            if (ml[2 * h + 1] > 0.0f && ml[2 * h] > m) m = ml[2 * h];
        }
        double L = 0.0, w[1024];
        for (int r = 0; r < n_parts && r < 1024; r++) {
            const float *ml = ml_parts + (size_t)r * nq * 2;
            w[r] = ml[2 * h + 1] > 0.0f ? (double)ml[2 * h + 1] * exp((double)ml[2 * h] - m) : 0.0;
            L += w[r];
        }
        for (int i = 0; i < hd; i++) {
            double acc = 0.0;
            for (int r = 0; r < n_parts && r < 1024; r++)
                acc += w[r] * o_parts[((size_t)r * nq + h) * hd + i];
            float oi = L > 0.0 ? (float)(acc / L) : 0.0f;
            size_t idx = (size_t)h * hd + i;
            const float gf = gate ? 1.0f / (1.0f + expf(-act_load(gate, idx, bf))) : 1.0f;
            act_store(out, idx, gate ? oi * gf : oi, obf);
        }
    }
}

/* Gated RMSNorm output of a DeltaNet layer, src/vx27_qfwd.c:146-151 with rmsn_std
 * (:42-46, sum of squares in double, eps 1e-6 inside the sqrt, /n) and silu1 (:48):
 * y[i] = (x[i] * s * w[i]) * (z[i] / (1 + expf(-z[i]))), for each of n_heads heads of hd. */
void orc_gated_rmsnorm(const float *x, const float *w, const float *z, float *y, int n_heads,
                       int hd) {
    for (int h = 0; h < n_heads; h++) {
        const float *xh = x + (size_t)h * hd, *zh = z + (size_t)h * hd;
        float *yh = y + (size_t)h * hd;
        double ss = 0;
        for (int i = 0; i < hd; i++) ss += (double)xh[i] * xh[i];
        const float s = 1.0f / sqrtf((float)(ss / hd) + 1e-6f);
        for (int i = 0; i < hd; i++) {
            const float tn = xh[i] * s * w[i];
            yh[i] = tn * (zh[i] / (1.0f + expf(-zh[i])));
        }
    }
}

/* gate_params over a [T][nv] grid of logits (fp32 values); beta/g_log [T][nv] */
void orc_gate_params_grid(const float *a, const float *b, const float *A_log,
                          const float *dt_bias, int T, int nv, double *beta, double *g_log) {
    for (long i = 0; i < (long)T * nv; i++) {
        const int vh = (int)(i % nv);
        g_gate((double)a[i], (double)A_log[vh], (double)b[i], (double)dt_bias[vh], beta + i,
               g_log + i);
    }
}

/* ------------------------------------------------------------- prefill refs */
void orc_deltanet_recurrent(float *S, const void *q, const void *k, const void *v,
                            long ld, const double *beta, const double *g_log,
                            float *o, int T, int hd, int flags) {
    const int bf = flags & ORC_F_ACT_BF16;
    float qb[256], kb[256], vb[256];
    for (int t = 0; t < T; t++) {
        for (int i = 0; i < hd; i++) {
            qb[i] = act_load(q, (size_t)t * ld + i, bf);
            kb[i] = act_load(k, (size_t)t * ld + i, bf);
            vb[i] = act_load(v, (size_t)t * ld + i, bf);
        }
        g_step(S, qb, kb, vb, beta[t], g_log[t], o + (size_t)t * hd, hd);
    }
}

void orc_gqa_prefill_rows(const void *q, const void *k, const void *v, const void *gate,
                          const float *q_norm_w, const float *k_norm_w,
                          int T, int nq, int nkv, int hd, int rope_dim, float theta,
                          float eps, const int *rows, int n_rows, float *out, int flags) {
    const int bf = flags & ORC_F_ACT_BF16, one_plus = (flags & ORC_F_NORM_1P) ? 1 : 0;
    int tmax = 0;
    for (int r = 0; r < n_rows; r++) if (rows[r] + 1 > tmax) tmax = rows[r] + 1;
    /* normalised, rotated K (rounded to bf16 like the cache) and V for positions < tmax */
    uint16_t *kc = (uint16_t *)malloc((size_t)nkv * tmax * hd * 2);
    uint16_t *vc = (uint16_t *)malloc((size_t)nkv * tmax * hd * 2);
    float cosv[128], sinv[128], x[512], t[512];
    for (int p = 0; p < tmax; p++) {
        g_rcs(p, cosv, sinv, rope_dim, theta, 1.0f);
        for (int h = 0; h < nkv; h++) {
            for (int i = 0; i < hd; i++) x[i] = act_load(k, ((size_t)p * nkv + h) * hd + i, bf);
            rms_dispatch(x, k_norm_w, t, hd, eps, one_plus);
            g_rap(t, 1, hd, rope_dim, cosv, sinv);
            for (int i = 0; i < hd; i++) {
                kc[((size_t)h * tmax + p) * hd + i] = orc_f32_to_bf16(t[i]);
                vc[((size_t)h * tmax + p) * hd + i] =
                    orc_f32_to_bf16(act_load(v, ((size_t)p * nkv + h) * hd + i, bf));
            }
        }
    }
    float *qn = (float *)malloc((size_t)nq * hd * sizeof(float));
    for (int r = 0; r < n_rows; r++) {
        const int p = rows[r];
        g_rcs(p, cosv, sinv, rope_dim, theta, 1.0f);
        for (int h = 0; h < nq; h++) {
            for (int i = 0; i < hd; i++) x[i] = act_load(q, ((size_t)p * nq + h) * hd + i, bf);
            rms_dispatch(x, q_norm_w, qn + (size_t)h * hd, hd, eps, one_plus);
            g_rap(qn + (size_t)h * hd, 1, hd, rope_dim, cosv, sinv);
        }
        int pos1 = p;
        /* the gate slice of this row: [nq][hd] at row p */
        const void *gate_row = bf ? (const void *)((const uint16_t *)gate + (size_t)p * nq * hd)
                                  : (const void *)((const float *)gate + (size_t)p * nq * hd);
        orc_gqa_attend(qn, gate_row, kc, vc, tmax, &pos1, out + (size_t)r * nq * hd, 1, nq,
                       nkv, hd, flags & ~ORC_F_OUT_BF16);
    }
    free(qn);
    free(kc);
    free(vc);
}

/* ------------------------------------------------------ synthetic inputs */
/* splitmix64 (Steele, Lea & Flood 2014), used as a counter-based generator */
/* ---- packed-weight matvec ------------------------------------------------ */
/* The group scale's fp16 -> fp32 as src/vx27_pmat.c:38-41 forms it: exponent rebased by
 * 112, subnormal fp16 values mapped with exponent 1 (not scaled as IEEE would). */
float orc_bp3_scale(uint16_t h) {
    const uint32_t u = h, sign = (u & 0x8000u) << 16, ex = (u >> 10) & 0x1Fu, man = u & 0x3FFu;
    uint32_t bits;
    if (ex == 0) bits = man ? (sign | ((ex + 1 + 112u) << 23) | (man << 13)) : sign;
    else if (ex == 31) bits = sign | 0x7F800000u | (man << 13);
    else bits = sign | ((ex + 112u) << 23) | (man << 13);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* One BP3_128 row against one vector: eight lanes, lane l = columns l mod 8 of each group
 * in increasing order, q*scale then fused multiply-add (src/vx27_pmat.c:28-63). */
static float orc_bp3_row(const uint8_t *row, int ng, const float *x) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int k = 0; k < ng; k++) {
        const uint8_t *g = row + (size_t)k * 52;
        uint32_t p[12];
        uint16_t h;
        memcpy(p, g, 48);
        memcpy(&h, g + 48, 2);
        const float sc = orc_bp3_scale(h);
        for (int i = 0; i < 128; i += 8)
            for (int l = 0; l < 8; l++) {
                const int e = i + l, w = e >> 5, bit = e & 31;
                const uint32_t u = ((p[w] >> bit) & 1u) | (((p[4 + w] >> bit) & 1u) << 1) |
                                   (((p[8 + w] >> bit) & 1u) << 2);
                const int q = u >= 4 ? (int)u - 8 : (int)u;
                const float qv = (float)q * sc;
                acc[l] = fmaf(qv, x[k * 128 + e], acc[l]);
            }
    }
    return acc[0] + acc[1] + acc[2] + acc[3] + acc[4] + acc[5] + acc[6] + acc[7];
}

/* One Q8_K row: per block eight FMA lanes summed left to right, times d in double
 * (src/vx27_pmat.c:10-24, 100-105). */
static float orc_q8k_row(const uint8_t *row, int nb, const float *x) {
    double s = 0;
    for (int k = 0; k < nb; k++) {
        const uint8_t *blk = row + (size_t)k * 292;
        float d;
        memcpy(&d, blk, 4);
        const int8_t *qs = (const int8_t *)(blk + 4);
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int i = 0; i < 256; i += 8)
            for (int l = 0; l < 8; l++) acc[l] = fmaf((float)qs[i + l], x[k * 256 + i + l], acc[l]);
        const float t = acc[0] + acc[1] + acc[2] + acc[3] + acc[4] + acc[5] + acc[6] + acc[7];
        s += (double)t * d;
    }
    return (float)s;
}

void orc_pmat_batch(const void *W, uint32_t dtype, const float *xb, float *yb, int rows,
                    int cols, int B) {
    const uint8_t *w8 = (const uint8_t *)W;
    const size_t rb = dtype == 0 ? (size_t)cols * 4
                    : dtype == 2 ? (size_t)(cols / 256) * 292 : (size_t)(cols / 128) * 52;
    for (int r = 0; r < rows; r++) {
        const uint8_t *row = w8 + (size_t)r * rb;
        for (int b = 0; b < B; b++) {
            const float *x = xb + (size_t)b * cols;
            float y;
            if (dtype == 0) {
                const float *wr = (const float *)row;
                double s = 0;
                for (int c = 0; c < cols; c++) s += (double)wr[c] * (double)x[c];
                y = (float)s;
            } else if (dtype == 2) {
                y = orc_q8k_row(row, cols / 256, x);
            } else {
                y = orc_bp3_row(row, cols / 128, x);
            }
            yb[(size_t)b * rows + r] = y;
        }
    }
}

uint64_t orc_splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}
static uint64_t stream_key(uint64_t seed, uint64_t stream) {
    return orc_splitmix64(orc_splitmix64(seed) ^ (stream * 0xD1B54A32D192ED03ull));
}
/* Box-Muller on the pair (2j, 2j+1): even index -> cos branch, odd -> sin branch */
static double normal_at(uint64_t key, uint64_t i) {
    const uint64_t j = i >> 1;
    const uint64_t r1 = orc_splitmix64(key + 2 * j), r2 = orc_splitmix64(key + 2 * j + 1);
    const double u1 = (double)((r1 >> 11) + 1) * 0x1.0p-53;
    const double u2 = (double)(r2 >> 11) * 0x1.0p-53;
    const double rad = sqrt(-2.0 * log(u1));
    const double th = 6.283185307179586 * u2;
    return (i & 1) ? rad * sin(th) : rad * cos(th);
}
void orc_fill_normal_f32(float *x, size_t n, uint64_t seed, uint64_t stream, float mean,
                         float std) {
    const uint64_t key = stream_key(seed, stream);
    for (size_t i = 0; i < n; i++) x[i] = (float)((double)mean + (double)std * normal_at(key, i));
}
void orc_fill_normal_bf16(uint16_t *x, size_t n, uint64_t seed, uint64_t stream, float mean,
                          float std) {
    const uint64_t key = stream_key(seed, stream);
    for (size_t i = 0; i < n; i++)
        x[i] = orc_f32_to_bf16((float)((double)mean + (double)std * normal_at(key, i)));
}
void orc_fill_uniform_f32(float *x, size_t n, uint64_t seed, uint64_t stream, float lo,
                          float hi) {
    const uint64_t key = stream_key(seed, stream);
    for (size_t i = 0; i < n; i++) {
        double u = (double)(orc_splitmix64(key + i) >> 11) * 0x1.0p-53;
        x[i] = (float)((double)lo + ((double)hi - (double)lo) * u);
    }
}
