// K1: fused Gated DeltaNet decode step for B sequences, one CTA per (sequence, V head).
//
// Per token the reference runs, per V head, conv1d_step -> gate_params -> step_exact
// (src/vx27_qfwd.c:276-297, src/vx27_deltanet.c:51-122). Here one kernel does all of
// it with the 128x128 fp32 state read once and written once:
//   1. the CTA issues its 16 x 16-byte state loads per thread first (64 KB per CTA in
//      flight; a warp reads whole 512-byte rows, so every load is coalesced);
//   2. while they are in flight it runs the width-4 causal conv + SiLU on its 384
//      channels (q and k of its QK head, v of its V head), the l2 norms (double sums
//      as the reference), q/sqrt(128), and the gates (double precision);
//   3. S' = S*decay and the column sums kv = S'^T k (per-thread partials over 16 rows,
//      then an 8-way reduction through shared memory);
//   4. d = (v - kv)*beta, S'' = S' + k d^T, o = S''^T q, and the state store.
// The state never leaves registers between the two reductions. The kernel is bound by
// HBM: 2 x 64 KB of state per (sequence, head) per step.
#include "common.cuh"
#include "../../include/vx27_deltanet.h"

namespace vx27 {
namespace {

constexpr int HD = 128;
constexpr int NT = 256;  // 8 warps; warp w owns rows [16w, 16w+16), lane l columns [4l, 4l+4)

// The gate mapping of src/vx27_deltanet.c:58-69 in double with the device exp/log (a few
// hundred cycles; the correctly rounded ddmath.h versions would put microseconds of
// serial fp64 work on every CTA's critical path). Callers that need the C library's
// exact bits pass host-computed gates (VX27_F_GATES_F64).
__device__ __forceinline__ void gates_device(double a, double A_log, double b, double dt,
                                             double *beta, double *g_log) {
    *beta = 1.0 / (1.0 + exp(-b));
    const double x = a + dt;
    const double sp = x > 20.0 ? x : (x < -20.0 ? exp(x) : log(1.0 + exp(x)));
    *g_log = -exp(A_log) * sp;
}

template <bool ACT_BF16, bool OUT_BF16, bool GATES_F64>
__global__ void __launch_bounds__(NT, 2)
dn_decode_k(float *__restrict__ S, float *__restrict__ ring, const void *__restrict__ qkv,
            const void *__restrict__ ga, const void *__restrict__ gb,
            const float *__restrict__ A_log, const float *__restrict__ dt_bias,
            const float *__restrict__ conv_w, const int *__restrict__ pos, void *__restrict__ o,
            int nqk, int nv) {
    const int vh = blockIdx.x, bi = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int qk = vh * nqk / nv;
    // the first V head of a QK group writes that group's q/k conv history
    const bool qk_owner = (vh == 0) || ((vh - 1) * nqk / nv != qk);
    const int C = (2 * nqk + nv) * HD;

    __shared__ float y_s[3 * HD];  // conv+SiLU output: q | k | v of this head
    __shared__ float qn_s[HD], kn_s[HD], d_s[HD];
    __shared__ __align__(16) float red[8][HD];
    __shared__ float par_s[4];  // 1/|q|, 1/|k|, beta, decay

    // 1. state loads, issued before anything else
    float4 *S4 = reinterpret_cast<float4 *>(S + ((size_t)bi * nv + vh) * HD * HD);
    float4 s[16];
#pragma unroll
    for (int r = 0; r < 16; r++) s[r] = __ldcs(S4 + (warp * 16 + r) * (HD / 4) + lane);

    // 2a. causal conv (tap 0 = oldest) + SiLU; ring slot t&3 receives this token's input
    const int t = pos[bi];
    const int sl0 = (t - 3) & 3, sl1 = (t - 2) & 3, sl2 = (t - 1) & 3, slw = t & 3;
    float *rb = ring + (size_t)bi * 4 * C;
    for (int e = tid; e < 3 * HD; e += NT) {
        const int part = e / HD, d = e % HD;
        const int c = part == 0 ? qk * HD + d
                    : part == 1 ? (nqk + qk) * HD + d
                                : 2 * nqk * HD + vh * HD + d;
        const float x = act_ld<ACT_BF16>(qkv, (size_t)bi * C + c);
        const float4 w = *reinterpret_cast<const float4 *>(conv_w + (size_t)c * 4);
        float acc = __fmul_rn(w.x, rb[(size_t)sl0 * C + c]);
        acc = __fadd_rn(acc, __fmul_rn(w.y, rb[(size_t)sl1 * C + c]));
        acc = __fadd_rn(acc, __fmul_rn(w.z, rb[(size_t)sl2 * C + c]));
        acc = __fadd_rn(acc, __fmul_rn(w.w, x));
        y_s[e] = __fdiv_rn(acc, __fadd_rn(1.0f, expf(-acc)));
        if (part == 2 || qk_owner) rb[(size_t)slw * C + c] = x;
    }
    __syncthreads();

    // 2b. l2 norms (warps 0, 1) and gates (warp 2)
    if (warp < 2) {
        const float *src = y_s + warp * HD;
        double ss = 0.0;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const double x = (double)src[lane * 4 + j];
            ss += x * x;
        }
        ss = warp_sum_d(ss);
        if (lane == 0) par_s[warp] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)ss, 1e-6f)));
    } else if (warp == 2 && lane == 0) {
        double beta, g;
        const size_t gi = (size_t)bi * nv + vh;
        if constexpr (GATES_F64) {
            beta = ((const double *)ga)[gi];
            g = ((const double *)gb)[gi];
        } else {
            gates_device((double)act_ld<ACT_BF16>(ga, gi), (double)A_log[vh],
                         (double)act_ld<ACT_BF16>(gb, gi), (double)dt_bias[vh], &beta, &g);
        }
        par_s[2] = (float)beta;
        par_s[3] = (float)exp(g);
    }
    __syncthreads();
    if (tid < HD) {
        const float qs = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
        qn_s[tid] = __fmul_rn(__fmul_rn(y_s[tid], par_s[0]), qs);
        kn_s[tid] = __fmul_rn(y_s[HD + tid], par_s[1]);
    }
    __syncthreads();

    // 3. decay and column partial sums of S'^T k
    const float decay = par_s[3];
    float4 kv = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < 16; r++) {
        const float k = kn_s[warp * 16 + r];
        s[r].x = __fmul_rn(s[r].x, decay);
        s[r].y = __fmul_rn(s[r].y, decay);
        s[r].z = __fmul_rn(s[r].z, decay);
        s[r].w = __fmul_rn(s[r].w, decay);
        kv.x = fmaf(s[r].x, k, kv.x);
        kv.y = fmaf(s[r].y, k, kv.y);
        kv.z = fmaf(s[r].z, k, kv.z);
        kv.w = fmaf(s[r].w, k, kv.w);
    }
    *reinterpret_cast<float4 *>(&red[warp][lane * 4]) = kv;
    __syncthreads();
    if (tid < HD) {
        float acc = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; w++) acc += red[w][tid];
        d_s[tid] = (y_s[2 * HD + tid] - acc) * par_s[2];
    }
    __syncthreads();

    // 4. rank-1 update, retrieve partials, state store
    const float4 dj = *reinterpret_cast<const float4 *>(&d_s[lane * 4]);
    float4 op = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < 16; r++) {
        const float k = kn_s[warp * 16 + r], q = qn_s[warp * 16 + r];
        s[r].x = fmaf(k, dj.x, s[r].x);
        s[r].y = fmaf(k, dj.y, s[r].y);
        s[r].z = fmaf(k, dj.z, s[r].z);
        s[r].w = fmaf(k, dj.w, s[r].w);
        op.x = fmaf(s[r].x, q, op.x);
        op.y = fmaf(s[r].y, q, op.y);
        op.z = fmaf(s[r].z, q, op.z);
        op.w = fmaf(s[r].w, q, op.w);
        __stcs(S4 + (warp * 16 + r) * (HD / 4) + lane, s[r]);
    }
    *reinterpret_cast<float4 *>(&red[warp][lane * 4]) = op;
    __syncthreads();
    if (tid < HD) {
        float acc = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; w++) acc += red[w][tid];
        act_st<OUT_BF16>(o, ((size_t)bi * nv + vh) * HD + tid, acc);
    }
}

template <bool A, bool O, bool G>
void launch(dim3 grid, cudaStream_t st, float *S, float *ring, const void *qkv, const void *a,
            const void *b, const float *A_log, const float *dt_bias, const float *conv_w,
            const int *pos, void *o, int nqk, int nv) {
    dn_decode_k<A, O, G><<<grid, NT, 0, st>>>(S, ring, qkv, a, b, A_log, dt_bias, conv_w, pos, o,
                                              nqk, nv);
}

}  // namespace
}  // namespace vx27

using namespace vx27;

extern "C" int vx27_deltanet_decode_batch(float *S, float *conv_ring, const void *qkv,
                                          const void *a, const void *b, const float *A_log,
                                          const float *dt_bias, const float *conv_w,
                                          const int *pos, void *o, int B, int nqk, int nv,
                                          int hd, int flags, void *stream, char *err,
                                          size_t errlen) {
    if (hd != HD)
        return fail(err, errlen, "vx27_deltanet_decode_batch: hd=%d unsupported (128 only)", hd);
    if (B <= 0 || B > 65535 || nqk <= 0 || nv <= 0 || nv < nqk || nv > 65535)
        return fail(err, errlen, "vx27_deltanet_decode_batch: bad shape B=%d nqk=%d nv=%d", B,
                    nqk, nv);
    if (!S || !conv_ring || !qkv || !a || !b || !conv_w || !pos || !o)
        return fail(err, errlen, "vx27_deltanet_decode_batch: null pointer argument");
    const bool g64 = flags & VX27_F_GATES_F64;
    if (!g64 && (!A_log || !dt_bias))
        return fail(err, errlen, "vx27_deltanet_decode_batch: A_log/dt_bias required");
    if (((uintptr_t)S & 15) || ((uintptr_t)conv_w & 15))
        return fail(err, errlen, "vx27_deltanet_decode_batch: S and conv_w must be 16-byte aligned");
    const dim3 grid(nv, B);
    cudaStream_t st = (cudaStream_t)stream;
    const int key = (flags & VX27_F_ACT_BF16 ? 1 : 0) | (flags & VX27_F_OUT_BF16 ? 2 : 0) |
                    (g64 ? 4 : 0);
#define VX_L(K, A_, O_, G_) \
    case K: launch<A_, O_, G_>(grid, st, S, conv_ring, qkv, a, b, A_log, dt_bias, conv_w, pos, o, nqk, nv); break;
    switch (key) {
        VX_L(0, false, false, false)
        VX_L(1, true, false, false)
        VX_L(2, false, true, false)
        VX_L(3, true, true, false)
        VX_L(4, false, false, true)
        VX_L(5, true, false, true)
        VX_L(6, false, true, true)
        VX_L(7, true, true, true)
    }
#undef VX_L
    VX_CK(cudaGetLastError());
    return 0;
}
