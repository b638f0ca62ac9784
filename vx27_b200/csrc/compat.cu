// The reference's own entry points (src/vx27_deltanet.h, src/vx27_gqa.h,
// src/vx27_rope.h) with their host-pointer, synchronous semantics, run on the GPU:
// copy in, launch, copy out, synchronise. Each kernel reproduces the rounding and the
// summation order of the reference function it replaces (separate multiply and add
// where the reference, compiled as ISO C11, has no contraction; fused where the
// reference uses FMA intrinsics; sequential sums where the reference sums
// sequentially), so results are bit-identical to the reference wherever the reference
// calls no libm function. Where it does (expf in SiLU and softmax, exp for the decay),
// the device computes the correctly rounded value (ddmath.h) or the host supplies it.
// Performance lives in the batched tier; these calls exist so that unmodified reference
// callers (src/vx27_block.c, src/vx27_qfwd.c) link against this library.
#include <math.h>
#include "common.cuh"
#include "ddmath.h"
#include "../../include/vx27_deltanet.h"
#include "../../include/vx27_gqa.h"
#include "../../include/vx27_rope.h"

namespace vx27 {
namespace {

// Per-thread device staging buffer (grow-only) and the per-thread default stream,
// so concurrent host threads can call the reentrant entry points.
thread_local void *t_buf = nullptr;
thread_local size_t t_cap = 0;

bool ensure(size_t bytes, const char *fn) {
    if (bytes <= t_cap) return true;
    if (t_buf) cudaFree(t_buf);
    t_buf = nullptr;
    t_cap = 0;
    size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
    cudaError_t e = cudaMalloc(&t_buf, want);
    if (e != cudaSuccess) {
        compat_fail(fn, cudaGetErrorString(e));
        return false;
    }
    t_cap = want;
    return true;
}

struct Stage {
    const char *fn;
    char *base;
    size_t off = 0;
    bool ok = true;
    explicit Stage(const char *f, size_t total) : fn(f) {
        ok = ensure(total + 64 * 16, f);
        base = (char *)t_buf;
    }
    template <class T>
    T *put(const T *host, size_t n) {  // allocate + copy host->device
        T *d = (T *)(base + off);
        off += (n * sizeof(T) + 255) & ~(size_t)255;
        if (ok && host && n) ok = check(cudaMemcpyAsync(d, host, n * sizeof(T),
                                                        cudaMemcpyHostToDevice,
                                                        cudaStreamPerThread));
        return d;
    }
    template <class T>
    T *take(size_t n) { return put<T>(nullptr, n); }
    template <class T>
    void get(T *host, const T *d, size_t n) {
        if (ok && n) ok = check(cudaMemcpyAsync(host, d, n * sizeof(T), cudaMemcpyDeviceToHost,
                                                cudaStreamPerThread));
    }
    bool check(cudaError_t e) {
        if (e != cudaSuccess) { compat_fail(fn, cudaGetErrorString(e)); return false; }
        return true;
    }
    bool launched() { return ok && (ok = check(cudaGetLastError())); }
    void finish() { if (ok) ok = check(cudaStreamSynchronize(cudaStreamPerThread)); }
};

inline size_t fbytes(size_t n) { return ((n * 4 + 255) & ~(size_t)255); }

// Correctly rounded float exp via the double-double exp (see ddmath.h).
__device__ __forceinline__ float expf_cr(float x) { return (float)vx_exp((double)x); }

// ---- DeltaNet update / retrieve (src/vx27_deltanet.c:15-48, _avx2.c:6-45) --------
__global__ void update_k(float *S, const float *k, const float *v, float decay, int hd,
                         int fused) {
    const size_t n = (size_t)hd * hd;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < n;
         e += (size_t)gridDim.x * blockDim.x) {
        const int i = (int)(e / hd), j = (int)(e % hd);
        const float kv = __fmul_rn(k[i], v[j]);
        S[e] = fused ? __fmaf_rn(S[e], decay, kv) : __fadd_rn(__fmul_rn(decay, S[e]), kv);
    }
}
// mode 0: sequential separate mul+add; 1: 16-row blocks summed then accumulated;
// 2: sequential fused multiply-add.
__global__ void retrieve_k(const float *S, const float *q, float *o, int hd, int mode) {
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < hd; j += gridDim.x * blockDim.x) {
        float acc = 0.0f;
        if (mode == 0) {
            for (int i = 0; i < hd; i++) acc = __fadd_rn(acc, __fmul_rn(S[(size_t)i * hd + j], q[i]));
        } else if (mode == 1) {
            for (int i0 = 0; i0 < hd; i0 += 16) {
                float s = 0.0f;
                const int i1 = i0 + 16 < hd ? i0 + 16 : hd;
                for (int i = i0; i < i1; i++) s = __fadd_rn(s, __fmul_rn(S[(size_t)i * hd + j], q[i]));
                acc = __fadd_rn(acc, s);
            }
        } else {
            for (int i = 0; i < hd; i++) acc = __fmaf_rn(S[(size_t)i * hd + j], q[i], acc);
        }
        o[j] = acc;
    }
}

// Sequential double sum of squares (terms are exact in double), as the reference.
__device__ double seq_sumsq(const float *x, int n) {
    double ss = 0.0;
    for (int i = 0; i < n; i++) ss = __dadd_rn(ss, __dmul_rn((double)x[i], (double)x[i]));
    return ss;
}

// src/vx27_deltanet.c:51-56
__global__ void l2norm_k(const float *x, float *y, int n) {
    __shared__ float r;
    if (threadIdx.x == 0) {
        const double ss = seq_sumsq(x, n);
        r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)ss, 1e-6f)));
    }
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) y[i] = __fmul_rn(x[i], r);
}

// src/vx27_deltanet.c:71-102, one block; decay = exp(g_log) computed on the host.
__global__ void step_exact_k(float *S, const float *q, const float *k, const float *v,
                             double beta, double decay, float *o, int hd) {
    __shared__ float qn[256], kn[256];
    __shared__ double kv[256];
    __shared__ float rq, rk;
    const int t = threadIdx.x;
    if (t == 0) rq = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)seq_sumsq(q, hd), 1e-6f)));
    if (t == 32) rk = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)seq_sumsq(k, hd), 1e-6f)));
    __syncthreads();
    const float qs = __fdiv_rn(1.0f, __fsqrt_rn((float)hd));
    for (int i = t; i < hd; i += blockDim.x) {
        qn[i] = __fmul_rn(__fmul_rn(q[i], rq), qs);
        kn[i] = __fmul_rn(k[i], rk);
    }
    const size_t n = (size_t)hd * hd;
    for (size_t e = t; e < n; e += blockDim.x)
        S[e] = __double2float_rn(__dmul_rn((double)S[e], decay));
    __syncthreads();
    for (int j = t; j < hd; j += blockDim.x) {
        double acc = 0.0;
        for (int i = 0; i < hd; i++)
            acc = __dadd_rn(acc, __dmul_rn((double)S[(size_t)i * hd + j], (double)kn[i]));
        kv[j] = acc;
    }
    __syncthreads();
    for (size_t e = t; e < n; e += blockDim.x) {
        const int i = (int)(e / hd), j = (int)(e % hd);
        const double d = __dmul_rn(__dsub_rn((double)v[j], kv[j]), beta);
        S[e] = __double2float_rn(__dadd_rn((double)S[e], __dmul_rn((double)kn[i], d)));
    }
    __syncthreads();
    for (int j = t; j < hd; j += blockDim.x) {
        double acc = 0.0;
        for (int i = 0; i < hd; i++)
            acc = __dadd_rn(acc, __dmul_rn((double)S[(size_t)i * hd + j], (double)qn[i]));
        o[j] = __double2float_rn(acc);
    }
}

// src/vx27_deltanet.c:104-122
__global__ void conv1d_k(float *state, const float *x, const float *w, float *y, int C,
                         int apply_silu) {
    for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < C; c += gridDim.x * blockDim.x) {
        const float *wc = w + (size_t)c * 4;
        float *st = state + (size_t)c * 3;
        const float s0 = st[0], s1 = st[1], s2 = st[2], xc = x[c];
        float acc = __fmul_rn(wc[0], s0);
        acc = __fadd_rn(acc, __fmul_rn(wc[1], s1));
        acc = __fadd_rn(acc, __fmul_rn(wc[2], s2));
        acc = __fadd_rn(acc, __fmul_rn(wc[3], xc));
        y[c] = apply_silu ? __fdiv_rn(acc, __fadd_rn(1.0f, expf_cr(-acc))) : acc;
        st[0] = s1;
        st[1] = s2;
        st[2] = xc;
    }
}

// src/vx27_gqa.c:10-15
__global__ void rmsnorm_k(const float *x, const float *w, float *y, int n, float eps) {
    __shared__ float r;
    if (threadIdx.x == 0) {
        const double ss = seq_sumsq(x, n);
        r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)__ddiv_rn(ss, (double)n), eps)));
    }
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) y[i] = __fmul_rn(__fmul_rn(x[i], r), w[i]);
}

// src/vx27_rope.c:18-29
__global__ void rope_apply_k(float *v, int n_heads, int head_dim, int rope_dim,
                             const float *cs, const float *sn) {
    const int half = rope_dim / 2;
    const int total = n_heads * half;
    for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < total; e += gridDim.x * blockDim.x) {
        const int h = e / half, i = e % half;
        float *p = v + (size_t)h * head_dim;
        const float x0 = p[i], x1 = p[i + half];
        p[i] = __fsub_rn(__fmul_rn(x0, cs[i]), __fmul_rn(x1, sn[i]));
        p[i + half] = __fadd_rn(__fmul_rn(x0, sn[i]), __fmul_rn(x1, cs[i]));
    }
}

// src/vx27_gqa.c:17-45: one block per Q head; sc is a [n_q][n_pos] device buffer.
__global__ void attn_1q_k(const float *q, const float *kc, const float *vc, int n_pos,
                          int n_q, int n_kv, int hd, float *sc, float *out) {
    const int h = blockIdx.x;
    const int kvh = h * n_kv / n_q;
    const float *qh = q + (size_t)h * hd;
    float *s = sc + (size_t)h * n_pos;
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)hd));
    __shared__ float red[32];
    __shared__ float smax_s, ssum_s;
    float mx = -1e30f;
    for (int p = threadIdx.x; p < n_pos; p += blockDim.x) {
        const float *kh = kc + ((size_t)p * n_kv + kvh) * hd;
        float acc = 0.0f;
        for (int i = 0; i < hd; i++) acc = __fadd_rn(acc, __fmul_rn(qh[i], kh[i]));
        acc = __fmul_rn(acc, scale);
        s[p] = acc;
        mx = fmaxf(mx, acc);
    }
    mx = warp_max(mx);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x == 0) {
        float m = -1e30f;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) m = fmaxf(m, red[w]);
        smax_s = m;
    }
    __syncthreads();
    for (int p = threadIdx.x; p < n_pos; p += blockDim.x) s[p] = expf_cr(__fsub_rn(s[p], smax_s));
    __syncthreads();
    if (threadIdx.x == 0) {
        float sum = 0.0f;
        for (int p = 0; p < n_pos; p++) sum = __fadd_rn(sum, s[p]);
        ssum_s = sum;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < hd; i += blockDim.x) {
        float acc = 0.0f;
        for (int p = 0; p < n_pos; p++) {
            const float a = __fdiv_rn(s[p], ssum_s);
            acc = __fadd_rn(acc, __fmul_rn(a, vc[((size_t)p * n_kv + kvh) * hd + i]));
        }
        out[(size_t)h * hd + i] = acc;
    }
}

void run_update(const char *fn, float *S, const float *k, const float *v, float decay, int hd,
                int fused) {
    if (hd <= 0) return;
    const size_t n = (size_t)hd * hd;
    Stage st(fn, fbytes(n) + 2 * fbytes(hd));
    float *dS = st.put(S, n), *dk = st.put(k, hd), *dv = st.put(v, hd);
    if (!st.ok) return;
    update_k<<<(unsigned)((n + 255) / 256), 256, 0, cudaStreamPerThread>>>(dS, dk, dv, decay, hd, fused);
    if (!st.launched()) return;
    st.get(S, dS, n);
    st.finish();
}

void run_retrieve(const char *fn, const float *S, const float *q, float *o, int hd, int mode) {
    if (hd <= 0) return;
    const size_t n = (size_t)hd * hd;
    Stage st(fn, fbytes(n) + 2 * fbytes(hd));
    float *dS = st.put(S, n), *dq = st.put(q, hd), *dout = st.take<float>(hd);
    if (!st.ok) return;
    retrieve_k<<<(hd + 127) / 128, 128, 0, cudaStreamPerThread>>>(dS, dq, dout, hd, mode);
    if (!st.launched()) return;
    st.get(o, dout, hd);
    st.finish();
}

}  // namespace
}  // namespace vx27

using namespace vx27;

extern "C" {

void vx27_deltanet_update_ref(float *S, const float *k, const float *v, float decay, int hd) {
    run_update("vx27_deltanet_update_ref", S, k, v, decay, hd, 0);
}
void vx27_deltanet_update_tiled(float *S, const float *k, const float *v, float decay, int hd) {
    run_update("vx27_deltanet_update_tiled", S, k, v, decay, hd, 0);
}
void vx27_deltanet_update_avx2(float *S, const float *k, const float *v, float decay, int hd) {
    run_update("vx27_deltanet_update_avx2", S, k, v, decay, hd, 1);
}
void vx27_deltanet_retrieve_ref(const float *S, const float *q, float *o, int hd) {
    run_retrieve("vx27_deltanet_retrieve_ref", S, q, o, hd, 0);
}
void vx27_deltanet_retrieve_tiled(const float *S, const float *q, float *o, int hd) {
    run_retrieve("vx27_deltanet_retrieve_tiled", S, q, o, hd, 1);
}
void vx27_deltanet_retrieve_avx2(const float *S, const float *q, float *o, int hd) {
    run_retrieve("vx27_deltanet_retrieve_avx2", S, q, o, hd, 2);
}

void vx27_deltanet_l2norm(const float *x, float *y, int n) {
    if (n <= 0) return;
    Stage st("vx27_deltanet_l2norm", 2 * fbytes(n));
    float *dx = st.put(x, n), *dy = st.take<float>(n);
    if (!st.ok) return;
    l2norm_k<<<1, 256, 0, cudaStreamPerThread>>>(dx, dy, n);
    if (!st.launched()) return;
    st.get(y, dy, n);
    st.finish();
}

void vx27_deltanet_step_exact(float *S, const float *q, const float *k, const float *v,
                              double beta, double g_log, float *o, int hd) {
    if (hd <= 0) return;
    if (hd > 256) {
        compat_fail("vx27_deltanet_step_exact", "hd > 256 (the reference's buffers hold 256)");
        return;
    }
    const size_t n = (size_t)hd * hd;
    const double decay = exp(g_log);  // host libm, as the reference
    Stage st("vx27_deltanet_step_exact", fbytes(n) + 4 * fbytes(hd));
    float *dS = st.put(S, n), *dq = st.put(q, hd), *dk = st.put(k, hd), *dv = st.put(v, hd);
    float *dout = st.take<float>(hd);
    if (!st.ok) return;
    step_exact_k<<<1, 256, 0, cudaStreamPerThread>>>(dS, dq, dk, dv, beta, decay, dout, hd);
    if (!st.launched()) return;
    st.get(S, dS, n);
    st.get(o, dout, hd);
    st.finish();
}

void vx27_conv1d_step(float *state, const float *x, const float *w, float *y, int C,
                      int apply_silu) {
    if (C <= 0) return;
    Stage st("vx27_conv1d_step", fbytes((size_t)C * 3) + fbytes((size_t)C * 4) + 2 * fbytes(C));
    float *ds = st.put(state, (size_t)C * 3), *dx = st.put(x, C), *dw = st.put(w, (size_t)C * 4);
    float *dy = st.take<float>(C);
    if (!st.ok) return;
    conv1d_k<<<(C + 255) / 256, 256, 0, cudaStreamPerThread>>>(ds, dx, dw, dy, C, apply_silu);
    if (!st.launched()) return;
    st.get(y, dy, C);
    st.get(state, ds, (size_t)C * 3);
    st.finish();
}

void vx27_rmsnorm(const float *x, const float *w, float *y, int n, float eps) {
    if (n <= 0) return;
    Stage st("vx27_rmsnorm", 3 * fbytes(n));
    float *dx = st.put(x, n), *dw = st.put(w, n), *dy = st.take<float>(n);
    if (!st.ok) return;
    rmsnorm_k<<<1, 256, 0, cudaStreamPerThread>>>(dx, dw, dy, n, eps);
    if (!st.launched()) return;
    st.get(y, dy, n);
    st.finish();
}

void vx27_rope_apply(float *v, int n_heads, int head_dim, int rope_dim, const float *cosv,
                     const float *sinv) {
    if (n_heads <= 0 || rope_dim <= 1) return;
    const size_t n = (size_t)n_heads * head_dim;
    const int half = rope_dim / 2;
    Stage st("vx27_rope_apply", fbytes(n) + 2 * fbytes(half));
    float *dv = st.put(v, n), *dc = st.put(cosv, half), *ds = st.put(sinv, half);
    if (!st.ok) return;
    rope_apply_k<<<(n_heads * half + 255) / 256, 256, 0, cudaStreamPerThread>>>(
        dv, n_heads, head_dim, rope_dim, dc, ds);
    if (!st.launched()) return;
    st.get(v, dv, n);
    st.finish();
}

void vx27_attn_1q(const float *q, const float *kcache, const float *vcache, int n_pos,
                  float *out) {
    const int nq = 24, nkv = 4, hd = 256;  // src/vx27_config.h:21-23
    if (n_pos <= 0) return;
    const size_t nkvp = (size_t)n_pos * nkv * hd;
    Stage st("vx27_attn_1q", 2 * fbytes((size_t)nq * hd) + 2 * fbytes(nkvp) +
                                 fbytes((size_t)nq * n_pos));
    float *dq = st.put(q, (size_t)nq * hd), *dk = st.put(kcache, nkvp), *dv = st.put(vcache, nkvp);
    float *dsc = st.take<float>((size_t)nq * n_pos), *dout = st.take<float>((size_t)nq * hd);
    if (!st.ok) return;
    attn_1q_k<<<nq, 256, 0, cudaStreamPerThread>>>(dq, dk, dv, n_pos, nq, nkv, hd, dsc, dout);
    if (!st.launched()) return;
    st.get(out, dout, (size_t)nq * hd);
    st.finish();
}

}  // extern "C"
