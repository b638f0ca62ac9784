// K3: chunked gated delta rule for prefill (config 4), chunks of 64 tokens.
//
// Token-by-token, per V head (src/vx27_deltanet.c:71-102):
//   S <- g_t S;  u_t = beta_t (v_t - S^T k_t);  S <- S + k_t u_t^T;  o_t = S^T q_t
// with q, k l2-normalised and q scaled by 1/sqrt(128). Within a chunk starting from S0,
// with gamma_t the product of the chunk's decays up to t (G_t = log gamma_t, summed in
// double):
//   (I + L) U = diag(beta) (V - diag(gamma) K S0),  L_ts = beta_t (gamma_t/gamma_s) k_t.k_s, s < t
//   so U = Wv - Wk S0 with T = (I + L)^-1 diag(beta), Wv = T V, Wk = T diag(gamma) K;
//   O   = diag(gamma) Q S0 + Pm U,   Pm_ts = (gamma_t/gamma_s) q_t.k_s for s <= t
//   S_C = gamma_C S0 + K^T diag(gamma_C/gamma) U
// Three kernels:
//   dn_chunk_prep   one CTA per (V head, chunk), all chunks in parallel: norms, gates,
//                   K K^T and Q K^T, the unit lower-triangular solve for T, Wv, Wk
//   dn_chunk_scan   one CTA per (V head, 16 state columns): the only sequential part,
//                   U_c = Wv - Wk S_c and S_{c+1} = gamma_C S_c + Kr^T U_c over the chunks
//                   (state columns are independent, so a head's state is split over 8 CTAs)
//   dn_chunk_out    one CTA per (V head, chunk): O = Qg S_c + Pm U
// All arithmetic fp32 (fp64 for the decay sums), so the result stays within 1e-3 of the
// token-by-token reference over 32768 tokens.
#include <math.h>
#include "common.cuh"
#include "../../include/vx27_deltanet.h"

namespace vx27 {
namespace {

constexpr int CK = 64;    // chunk
constexpr int D = 128;    // head dim
constexpr int CB = 16;    // state columns per scan CTA
constexpr int LDS = D + 1;

struct Ws {  // workspace views; blk = vh * n_chunks + chunk
    float *Wk, *Wv, *Qg, *Kr, *Pm, *U, *Sc, *g63;
};
__host__ __device__ inline size_t ws_floats_per_blk() {
    return 4 * (size_t)CK * D + (size_t)CK * CK + (size_t)CK * D + (size_t)D * D + 4;
}
__host__ __device__ inline Ws ws_views(float *base, size_t nblk) {
    Ws w;
    w.Wk = base;
    w.Wv = w.Wk + nblk * CK * D;
    w.Qg = w.Wv + nblk * CK * D;
    w.Kr = w.Qg + nblk * CK * D;
    w.Pm = w.Kr + nblk * CK * D;
    w.U = w.Pm + nblk * CK * CK;
    w.Sc = w.U + nblk * CK * D;
    w.g63 = w.Sc + nblk * D * D;
    return w;
}

__device__ __forceinline__ void gates_dev(double a, double A_log, double b, double dt,
                                          double *beta, double *g_log) {
    *beta = 1.0 / (1.0 + exp(-b));
    const double x = a + dt;
    const double sp = x > 20.0 ? x : (x < -20.0 ? exp(x) : log(1.0 + exp(x)));
    *g_log = -exp(A_log) * sp;
}

// ---- phase 1: per-chunk preparation ----------------------------------------------------
template <bool ACT_BF16, bool GATES_F64>
__global__ void __launch_bounds__(256)
dn_chunk_prep(const void *__restrict__ q, const void *__restrict__ k, const void *__restrict__ v,
              const void *__restrict__ ga, const void *__restrict__ gb,
              const float *__restrict__ A_log, const float *__restrict__ dt_bias, Ws ws, int T,
              int nqk, int nv, int n_chunks) {
    extern __shared__ float psm[];
    float *Kh = psm;                 // [CK][LDS] normalised k
    float *Qh = Kh + CK * LDS;       // [CK][LDS] normalised, scaled q
    float *Vs = Qh + CK * LDS;       // [CK][LDS] v
    float *Lm = Vs + CK * LDS;       // [CK][CK+1] L, then T
    float *Xs = Lm + CK * (CK + 1);  // [CK][CK+1] T
    double *G = reinterpret_cast<double *>(Xs + CK * (CK + 1));  // [CK]
    float *beta = reinterpret_cast<float *>(G + CK);             // [CK]
    float *gam = beta + CK;                                      // [CK] exp(G)
    const int vh = blockIdx.x, c = blockIdx.y, tid = threadIdx.x, warp = tid >> 5,
              lane = tid & 31;
    const int qk = vh * nqk / nv;
    const int t0 = c * CK;
    const size_t blk = (size_t)vh * n_chunks + c;
    // 1. load (tokens past T are identity steps: zero q/k/v, beta = 0, g = 0)
    for (int e = tid; e < CK * D; e += 256) {
        const int t = e / D, d = e % D, tt = t0 + t;
        float qv = 0.f, kv = 0.f, vv = 0.f;
        if (tt < T) {
            qv = act_ld<ACT_BF16>(q, ((size_t)tt * nqk + qk) * D + d);
            kv = act_ld<ACT_BF16>(k, ((size_t)tt * nqk + qk) * D + d);
            vv = act_ld<ACT_BF16>(v, ((size_t)tt * nv + vh) * D + d);
        }
        Qh[t * LDS + d] = qv;
        Kh[t * LDS + d] = kv;
        Vs[t * LDS + d] = vv;
    }
    if (tid < CK) {
        const int tt = t0 + tid;
        double bt = 0.0, gl = 0.0;
        if (tt < T) {
            const size_t gi = (size_t)tt * nv + vh;
            if constexpr (GATES_F64) {
                bt = ((const double *)ga)[gi];
                gl = ((const double *)gb)[gi];
            } else {
                gates_dev((double)act_ld<ACT_BF16>(ga, gi), (double)A_log[vh],
                          (double)act_ld<ACT_BF16>(gb, gi), (double)dt_bias[vh], &bt, &gl);
            }
        }
        beta[tid] = (float)bt;
        G[tid] = gl;
    }
    __syncthreads();
    // 2. l2 norms (double sums as src/vx27_deltanet.c:51) and the decay prefix sum
    for (int row = warp; row < 2 * CK; row += 8) {
        float *x = row < CK ? Qh + row * LDS : Kh + (row - CK) * LDS;
        double ss = 0.0;
        for (int d = lane; d < D; d += 32) ss += (double)x[d] * (double)x[d];
        ss = warp_sum_d(ss);
        const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)ss, 1e-6f)));
        for (int d = lane; d < D; d += 32) {
            float y = __fmul_rn(x[d], r);
            if (row < CK) y = __fmul_rn(y, __fdiv_rn(1.0f, __fsqrt_rn((float)D)));
            x[d] = y;
        }
    }
    if (tid == 0) {
        double acc = 0.0;
        for (int t = 0; t < CK; t++) { acc += G[t]; G[t] = acc; }
    }
    __syncthreads();
    if (tid < CK) gam[tid] = (float)exp(G[tid]);
    // 3. L (strictly lower, with beta and decay) and Pm (lower incl. diagonal)
    float *Pm = ws.Pm + blk * CK * CK;
    for (int e = tid; e < CK * CK; e += 256) {
        const int t = e / CK, s = e % CK;
        float kk = 0.f, qkv = 0.f;
        if (s <= t) {
            const float *kt = Kh + t * LDS, *ks = Kh + s * LDS, *qt = Qh + t * LDS;
#pragma unroll 8
            for (int d = 0; d < D; d++) {
                kk = fmaf(kt[d], ks[d], kk);
                qkv = fmaf(qt[d], ks[d], qkv);
            }
        }
        const float dec = s <= t ? (float)exp(G[t] - G[s]) : 0.f;
        Lm[t * (CK + 1) + s] = s < t ? beta[t] * dec * kk : 0.f;
        Pm[e] = s <= t ? dec * qkv : 0.f;
    }
    __syncthreads();
    // 4. T = (I + L)^-1 diag(beta), row by row: T_t = beta_t e_t - sum_{r<t} L_tr T_r
    for (int t = 0; t < CK; t++) {
        // 64 columns x 4 partial sums per column
        const int s = tid >> 2, part = tid & 3;
        float acc = 0.f;
        if (s < t)
            for (int r = s + part; r < t; r += 4) acc = fmaf(Lm[t * (CK + 1) + r], Xs[r * (CK + 1) + s], acc);
        acc += __shfl_xor_sync(0xffffffffu, acc, 1);
        acc += __shfl_xor_sync(0xffffffffu, acc, 2);
        if (part == 0) Xs[t * (CK + 1) + s] = s < t ? -acc : (s == t ? beta[t] : 0.f);
        __syncthreads();
    }
    // 5. Wv = T V, Wk = T diag(gamma) K; Qg = diag(gamma) Q; Kr = diag(gamma_C/gamma) K
    float *Wv = ws.Wv + blk * CK * D, *Wk = ws.Wk + blk * CK * D;
    float *Qg = ws.Qg + blk * CK * D, *Kr = ws.Kr + blk * CK * D;
    for (int e = tid; e < CK * D; e += 256) {
        const int t = e / D, d = e % D;
        float av = 0.f, ak = 0.f;
        for (int s = 0; s <= t; s++) {
            const float x = Xs[t * (CK + 1) + s];
            av = fmaf(x, Vs[s * LDS + d], av);
            ak = fmaf(x * gam[s], Kh[s * LDS + d], ak);
        }
        Wv[e] = av;
        Wk[e] = ak;
        Qg[e] = gam[t] * Qh[t * LDS + d];
        Kr[e] = (float)exp(G[CK - 1] - G[t]) * Kh[t * LDS + d];
    }
    if (tid == 0) ws.g63[blk] = (float)exp(G[CK - 1]);
}

// ---- phase 2: the sequential state scan --------------------------------------------------
struct ScanSmem {
    float Wk_s[CK][D + 1];
    float Kr_s[CK][D + 1];
    float S_s[D][CB + 1];
    float U_s[CK][CB + 1];
};

__global__ void __launch_bounds__(256)
dn_chunk_scan(Ws ws, float *__restrict__ S, int nv, int n_chunks) {
    extern __shared__ float ssm_raw[];
    ScanSmem &sm = *reinterpret_cast<ScanSmem *>(ssm_raw);
    auto &Wk_s = sm.Wk_s;
    auto &Kr_s = sm.Kr_s;
    auto &S_s = sm.S_s;
    auto &U_s = sm.U_s;
    const int vh = blockIdx.x, cb = blockIdx.y, tid = threadIdx.x;
    float *Sh = S + (size_t)vh * D * D;
    // thread owns state rows tid/2 and 8 of the CB columns
    const int r = tid >> 1, j0 = (tid & 1) * 8;
    float s[8];
#pragma unroll
    for (int j = 0; j < 8; j++) s[j] = Sh[r * D + cb * CB + j0 + j];
    for (int c = 0; c < n_chunks; c++) {
        const size_t blk = (size_t)vh * n_chunks + c;
        const float *Wk = ws.Wk + blk * CK * D, *Kr = ws.Kr + blk * CK * D;
        const float *Wv = ws.Wv + blk * CK * D;
        float *Sc = ws.Sc + blk * D * D, *U = ws.U + blk * CK * D;
        for (int e = tid; e < CK * D; e += 256) {
            Wk_s[e / D][e % D] = Wk[e];
            Kr_s[e / D][e % D] = Kr[e];
        }
#pragma unroll
        for (int j = 0; j < 8; j++) {
            S_s[r][j0 + j] = s[j];
            Sc[r * D + cb * CB + j0 + j] = s[j];  // state at the chunk start, for the output
        }
        __syncthreads();
        // U = Wv - Wk S  (64 x CB): 4 outputs per thread
        for (int e = tid; e < CK * CB; e += 256) {
            const int t = e / CB, j = e % CB;
            float acc = 0.f;
#pragma unroll 8
            for (int d = 0; d < D; d++) acc = fmaf(Wk_s[t][d], S_s[d][j], acc);
            const float u = Wv[t * D + cb * CB + j] - acc;
            U_s[t][j] = u;
            U[t * D + cb * CB + j] = u;
        }
        __syncthreads();
        // S = gamma_C S + Kr^T U
        const float g = ws.g63[blk];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            float acc = 0.f;
#pragma unroll 8
            for (int t = 0; t < CK; t++) acc = fmaf(Kr_s[t][r], U_s[t][j0 + j], acc);
            s[j] = fmaf(g, s[j], acc);
        }
        __syncthreads();
    }
#pragma unroll
    for (int j = 0; j < 8; j++) Sh[r * D + cb * CB + j0 + j] = s[j];
}

// ---- phase 3: outputs ---------------------------------------------------------------------
template <bool OUT_BF16>
__global__ void __launch_bounds__(256)
dn_chunk_out(Ws ws, void *__restrict__ o, int T, int nv, int n_chunks) {
    extern __shared__ float osm[];
    float *Qg = osm;                 // [CK][D+1]
    float *Pm = Qg + CK * (D + 1);   // [CK][CK+1]
    float *Sc = Pm + CK * (CK + 1);  // [D][64+1]  (one half of the columns)
    float *Us = Sc + D * 65;         // [CK][64+1]
    const int vh = blockIdx.x, c = blockIdx.y, tid = threadIdx.x;
    const size_t blk = (size_t)vh * n_chunks + c;
    const float *gQg = ws.Qg + blk * CK * D, *gPm = ws.Pm + blk * CK * CK;
    const float *gSc = ws.Sc + blk * D * D, *gU = ws.U + blk * CK * D;
    for (int e = tid; e < CK * D; e += 256) Qg[(e / D) * (D + 1) + e % D] = gQg[e];
    for (int e = tid; e < CK * CK; e += 256) Pm[(e / CK) * (CK + 1) + e % CK] = gPm[e];
    for (int half = 0; half < 2; half++) {
        for (int e = tid; e < D * 64; e += 256)
            Sc[(e / 64) * 65 + e % 64] = gSc[(e / 64) * D + half * 64 + e % 64];
        for (int e = tid; e < CK * 64; e += 256)
            Us[(e / 64) * 65 + e % 64] = gU[(e / 64) * D + half * 64 + e % 64];
        __syncthreads();
        // 64 x 64 outputs: thread -> 4 rows x 4 columns
        const int tr = (tid >> 4) * 4, tc = (tid & 15) * 4;
        float acc[4][4] = {};
        for (int d = 0; d < D; d++) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; i++) { a[i] = Qg[(tr + i) * (D + 1) + d]; b[i] = Sc[d * 65 + tc + i]; }
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int jj = 0; jj < 4; jj++) acc[i][jj] = fmaf(a[i], b[jj], acc[i][jj]);
        }
        for (int s = 0; s < CK; s++) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; i++) { a[i] = Pm[(tr + i) * (CK + 1) + s]; b[i] = Us[s * 65 + tc + i]; }
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int jj = 0; jj < 4; jj++) acc[i][jj] = fmaf(a[i], b[jj], acc[i][jj]);
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int tt = c * CK + tr + i;
            if (tt >= T) continue;
#pragma unroll
            for (int jj = 0; jj < 4; jj++)
                act_st<OUT_BF16>(o, ((size_t)tt * nv + vh) * D + half * 64 + tc + jj, acc[i][jj]);
        }
        __syncthreads();
    }
}

}  // namespace
}  // namespace vx27

using namespace vx27;

extern "C" size_t vx27_deltanet_prefill_workspace_size(int T, int nqk, int nv, int hd) {
    (void)nqk;
    if (T <= 0 || nv <= 0 || hd != D) return 0;
    const size_t n_chunks = ((size_t)T + CK - 1) / CK;
    return n_chunks * nv * ws_floats_per_blk() * sizeof(float);
}

extern "C" int vx27_deltanet_prefill_chunked(const void *q, const void *k, const void *v,
                                             const void *a, const void *b, const float *A_log,
                                             const float *dt_bias, float *S, void *o,
                                             void *workspace, size_t workspace_bytes, int T,
                                             int nqk, int nv, int hd, int flags, void *stream,
                                             char *err, size_t errlen) {
    const char *fn = "vx27_deltanet_prefill_chunked";
    if (hd != D) return fail(err, errlen, "%s: hd=%d unsupported (128 only)", fn, hd);
    if (T <= 0 || nqk <= 0 || nv < nqk || nv > 65535)
        return fail(err, errlen, "%s: bad shape T=%d nqk=%d nv=%d", fn, T, nqk, nv);
    const bool g64 = flags & VX27_F_GATES_F64;
    if (!q || !k || !v || !a || !b || !S || !o || !workspace || (!g64 && (!A_log || !dt_bias)))
        return fail(err, errlen, "%s: null pointer argument", fn);
    const size_t need = vx27_deltanet_prefill_workspace_size(T, nqk, nv, hd);
    if (workspace_bytes < need)
        return fail(err, errlen, "%s: workspace of %zu bytes, need %zu", fn, workspace_bytes, need);
    const int n_chunks = (T + CK - 1) / CK;
    if (n_chunks > 65535) return fail(err, errlen, "%s: T=%d too long", fn, T);
    cudaStream_t st = (cudaStream_t)stream;
    Ws ws = ws_views((float *)workspace, (size_t)n_chunks * nv);
    const size_t prep_smem = (3 * CK * LDS + 2 * CK * (CK + 1)) * sizeof(float) +
                             CK * sizeof(double) + 2 * CK * sizeof(float);
    const bool bf = flags & VX27_F_ACT_BF16;
#define VX_PREP(A_, G_)                                                                     \
    {                                                                                       \
        static bool attr = false;                                                           \
        if (!attr) {                                                                        \
            VX_CK(cudaFuncSetAttribute(dn_chunk_prep<A_, G_>,                               \
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,         \
                                       (int)prep_smem));                                    \
            attr = true;                                                                    \
        }                                                                                   \
        dn_chunk_prep<A_, G_><<<dim3(nv, n_chunks), 256, prep_smem, st>>>(                  \
            q, k, v, a, b, A_log, dt_bias, ws, T, nqk, nv, n_chunks);                       \
    }
    if (bf && g64) VX_PREP(true, true)
    else if (bf) VX_PREP(true, false)
    else if (g64) VX_PREP(false, true)
    else VX_PREP(false, false)
#undef VX_PREP
    VX_CK(cudaGetLastError());
    {
        static bool attr = false;
        if (!attr) {
            VX_CK(cudaFuncSetAttribute(dn_chunk_scan, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)sizeof(ScanSmem)));
            attr = true;
        }
        dn_chunk_scan<<<dim3(nv, D / CB), 256, sizeof(ScanSmem), st>>>(ws, S, nv, n_chunks);
    }
    VX_CK(cudaGetLastError());
    const size_t out_smem = (CK * (D + 1) + CK * (CK + 1) + D * 65 + CK * 65) * sizeof(float);
    if (flags & VX27_F_OUT_BF16) {
        static bool attr = false;
        if (!attr) {
            VX_CK(cudaFuncSetAttribute(dn_chunk_out<true>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)out_smem));
            attr = true;
        }
        dn_chunk_out<true><<<dim3(nv, n_chunks), 256, out_smem, st>>>(ws, o, T, nv, n_chunks);
    } else {
        static bool attr = false;
        if (!attr) {
            VX_CK(cudaFuncSetAttribute(dn_chunk_out<false>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)out_smem));
            attr = true;
        }
        dn_chunk_out<false><<<dim3(nv, n_chunks), 256, out_smem, st>>>(ws, o, T, nv, n_chunks);
    }
    VX_CK(cudaGetLastError());
    return 0;
}
