// K4: causal gated GQA prefill of T prompt tokens on the tensor cores (config 4).
//
//   prep kernel   per token and head: QK RMSNorm, partial RoPE at position p0 + t (host
//                 table), q -> bf16 Qn[nq][T][256], k/v -> the bf16 KV cache slots p0 + t
//                 (the cache the decode continues from); src/vx27_qfwd.c:339-346 per token
//   attention     flash-attention forward. By default a 2-CTA cluster per (128-query tile,
//                 two query heads of one KV head) whose M = 256 tcgen05 MMAs span both SMs,
//                 each SM holding half of every K/V chunk (prefill_attn_pair); else one CTA
//                 per (tile, head) (prefill_attn_tc). Warp roles of a CTA:
//     warp 0      TMA: the Q tile (128 x 256, resident); 128-key K tiles as four 64-dim
//                 chunks and V tiles as four 32-key chunks through two rings, one for K
//                 (read by the S-MMA warp) and one for V (the O-MMA warp), each refilled
//                 as soon as a slot frees. A slot has one consumer, which waits for every
//                 phase of its barriers in order; with a shared ring a consumer that ran
//                 ahead of a slot's previous load (the other warp's) could take that load's
//                 pending phase for its own
//     warp 1      tcgen05.mma: S = Q K^T (128 x 128 fp32 in TMEM), issued as soon as the
//                 softmax has read the previous S
//     warp 10     tcgen05.mma: O += P V (128 x 256 fp32 in TMEM), P read from TMEM as the A
//                 operand, V as an MN-major operand from shared memory
//     warps 2-9   two threads per query row (its TMEM lane), one per half of the keys and of
//                 the output columns: causal mask, running max in log2 units (the halves
//                 meet through shared memory), p = 2^(x - m) written to TMEM as bf16 pairs
//                 (two P buffers); O is rescaled in TMEM only when a row's max grows by
//                 more than 2^8 (lazy rescale); epilogue O / l * sigmoid(gate).
// Query tiles are issued longest first; the six query heads of a KV head run on
// neighbouring CTAs so their K/V tiles are served from L2.
#include <math.h>
#include <algorithm>
#include "common.cuh"
#include "tc.cuh"
#include "../../include/vx27_gqa.h"

namespace vx27 {
namespace {

constexpr int HDP = 256;
constexpr int QT = 128;          // queries per CTA
constexpr int KT = 128;          // keys per tile
constexpr int NKS = 5;           // single-SM kernel: K ring slots of 16 KB
constexpr int NVS = 4;           // V ring slots of 16 KB
constexpr int NS = NKS + NVS;    // slots 0..NKS-1 hold K chunks, NKS.. V chunks
constexpr int NKS2 = 10;         // CTA pair: K ring slots of 8 KB (this SM's half of a chunk)
constexpr int NVS2 = 9;          // V ring slots of 8 KB
constexpr int NS2 = NKS2 + NVS2;
constexpr int SLOT2 = 8192;
constexpr int PF_THREADS = 352;  // TMA warp, S-MMA warp, 8 softmax warps, O-MMA warp
constexpr float RESCALE_LOG2 = 8.0f;

// Tensor memory (512 columns): S at [0, 128) (fp32), O at [128, 384), and P(j) as bf16
// pairs in buffer j & 1 at [384 + 64 b, 448 + 64 b), the O MMA's A operand from there (so
// P needs no shared memory). S(j + 1) is issued as soon as the softmax has read S(j).
constexpr uint32_t TM_O = 128, TM_P = 384;

template <int NSLOT, int SLOT>
struct AttnSmem {
    uint8_t q[4][QT * 128];      // Q tile, 4 chunks of [128 rows x 64 dims], 128B swizzle
    uint8_t ring[NSLOT][SLOT];   // K chunk [keys x 64 dims] or V chunk [32 keys x dims]
    float xmax[2][2][QT];        // row maxima of the two key halves, by tile parity
    float xsum[2][QT];           // row sums of the two halves
    uint64_t qfull, full[NSLOT], empty[NSLOT], s_full, s_empty, p_full[2], pv_done[2],
        o_final, mma_done, qk_done;
    uint32_t tmem_base;
    int abort;
};
using PfSmem = AttnSmem<NS, 16384>;   // K chunk [128 keys x 64 dims], V [32 keys x 256 dims]
using PairSmem = AttnSmem<NS2, SLOT2>;  // K chunk [64 keys x 64 dims], V [32 keys x 128 dims]
// the fp32-gate epilogue stages O / l (128 rows x 256 fp32) over the ring
static_assert(sizeof(PfSmem::ring) >= QT * HDP * 4, "staging");
static_assert(sizeof(PairSmem::ring) >= QT * HDP * 4, "staging");
static_assert(sizeof(PfSmem) + 1024 <= 232448 && sizeof(PairSmem) + 1024 <= 232448, "smem");

// Chunk c of K(m) is the (4m + c)-th load of the K ring, chunk c of V(t) the (4t + c)-th
// of the V ring: slot i % NKS (NKS + i % NVS), barrier phase i / NKS (i / NVS); the same
// with NKS2/NVS2 in the pair kernel.

// ---- prep ----------------------------------------------------------------------------
// One warp per (token, head) row, 8 consecutive dims per lane (16-byte bf16 accesses), with
// every load of the row issued before any is used (the row, the RoPE cos/sin at its
// position, the V row of a KV head), one memory round trip per row instead of three:
// 0.42 ms at config 4 against 0.47 (ncu); two or four rows per warp and round, with more
// bytes in flight, measured slower (0.53 / 0.56 ms).
// RMSNorm with a double sum of squares, NeoX RoPE on dims [0, rope_dim) (the partner of
// dim d < rope_dim/2 is d + rope_dim/2, held rope_dim/16 lanes away), bf16 stores.
template <bool ACT_BF16>
__device__ __forceinline__ void load8(const void *p, size_t i, float *x) {
    if constexpr (ACT_BF16) {
        const uint4 v = *reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(p) + i);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int k = 0; k < 4; k++) {
            x[2 * k] = bf16_to_f32(w[k] & 0xffffu);
            x[2 * k + 1] = bf16_to_f32(w[k] >> 16);
        }
    } else {
        const float4 *f = reinterpret_cast<const float4 *>(static_cast<const float *>(p) + i);
        const float4 a = f[0], b = f[1];
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
        x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    }
}
__device__ __forceinline__ void store8_bf16(uint16_t *p, const float *x) {
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; k++)
        w[k] = (uint32_t)f32_to_bf16(x[2 * k]) | ((uint32_t)f32_to_bf16(x[2 * k + 1]) << 16);
    *reinterpret_cast<uint4 *>(p) = make_uint4(w[0], w[1], w[2], w[3]);
}

template <bool ACT_BF16, bool ONE_P>
__global__ void __launch_bounds__(256, 5)
prefill_prep_k(const void *__restrict__ q_in, const void *__restrict__ k_in,
               const void *__restrict__ v_in, const float *__restrict__ qw,
               const float *__restrict__ kw, const float *__restrict__ rope, int rope_len,
               int p0, uint16_t *__restrict__ qn, uint16_t *__restrict__ kc,
               uint16_t *__restrict__ vc, int cap, int T, int nq, int nkv, int rope_dim,
               float eps, uint32_t *status) {
    const int lane = threadIdx.x & 31;
    const int nh = nq + nkv;
    const size_t n_rows = (size_t)T * nh;
    const int half = rope_dim / 2, hl = half / 8;  // partner lane distance
    const int d0 = lane * 8;
    const bool rot = d0 < rope_dim;
    const bool lo = d0 < half;
    const int src = lo ? lane + hl : lane - hl;
    const int i0 = lo ? d0 : d0 - half;  // this lane's cos/sin columns (when rot)
    for (size_t item = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; item < n_rows;
         item += ((size_t)gridDim.x * blockDim.x) >> 5) {
        const int t = (int)(item / nh), head = (int)(item % nh);
        const bool is_q = head < nq;
        const int h = is_q ? head : head - nq;
        const int p = p0 + t;
        const size_t row = is_q ? ((size_t)t * nq + h) * HDP : ((size_t)t * nkv + h) * HDP;
        // every load of the row first: the row, the RoPE cos/sin at its position, and for a
        // KV head the V row, which goes straight to the cache
        float x[8], cs[8], sn[8];
        load8<ACT_BF16>(is_q ? q_in : k_in, row + d0, x);
        const bool prot = rot && p >= 0 && p < rope_len;
        if (prot) {
            const float4 *rr = reinterpret_cast<const float4 *>(rope + (size_t)p * rope_dim);
            const float4 c0 = rr[i0 / 4], c1 = rr[i0 / 4 + 1];
            const float4 s0 = rr[(half + i0) / 4], s1 = rr[(half + i0) / 4 + 1];
            cs[0] = c0.x; cs[1] = c0.y; cs[2] = c0.z; cs[3] = c0.w;
            cs[4] = c1.x; cs[5] = c1.y; cs[6] = c1.z; cs[7] = c1.w;
            sn[0] = s0.x; sn[1] = s0.y; sn[2] = s0.z; sn[3] = s0.w;
            sn[4] = s1.x; sn[5] = s1.y; sn[6] = s1.z; sn[7] = s1.w;
        }
        if (!is_q && p < cap) {
            float v[8];
            load8<ACT_BF16>(v_in, row + d0, v);
            store8_bf16(vc + ((size_t)h * cap + p) * HDP + d0, v);
        }
        double ss = 0.0;
#pragma unroll
        for (int e = 0; e < 8; e++) ss += (double)x[e] * (double)x[e];
        ss = warp_sum_d(ss);
        const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)(ss / HDP), eps)));
        const float *wp = (is_q ? qw : kw) + d0;  // L1-resident: every row reads them
        float y[8];
#pragma unroll
        for (int e = 0; e < 8; e++) {
            float w = __ldg(wp + e);
            if (ONE_P) w = __fadd_rn(w, 1.0f);
            y[e] = __fmul_rn(__fmul_rn(x[e], r), w);
        }
        // partner values for the rotation (all lanes take part in the shuffles)
        float yp[8];
#pragma unroll
        for (int e = 0; e < 8; e++) yp[e] = __shfl_sync(0xffffffffu, y[e], (src & 31));
        if (rot) {
            if (!prot) {
                dev_flag(status, VX_DEV_BAD_ARG);
            } else {
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    const float x0 = lo ? y[e] : yp[e], x1 = lo ? yp[e] : y[e];
                    y[e] = lo ? __fsub_rn(__fmul_rn(x0, cs[e]), __fmul_rn(x1, sn[e]))
                              : __fadd_rn(__fmul_rn(x0, sn[e]), __fmul_rn(x1, cs[e]));
                }
            }
        }
        if (is_q) store8_bf16(qn + ((size_t)h * T + t) * HDP + d0, y);
        else if (p < cap) store8_bf16(kc + ((size_t)h * cap + p) * HDP + d0, y);
    }
}

// Zero cache slots [from, to) of every KV head so the last key tile reads finite values.
__global__ void zero_slots_k(uint16_t *kc, uint16_t *vc, int cap, int nkv, int from, int to) {
    const int h = blockIdx.y;
    const size_t n = (size_t)(to - from) * HDP;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < n;
         e += (size_t)gridDim.x * blockDim.x) {
        const size_t o = ((size_t)h * cap + from) * HDP + e;
        kc[o] = 0;
        vc[o] = 0;
    }
}

// ---- main kernels ------------------------------------------------------------------------
// Bounded waits. A wait that times out marks the CTA (and, in a pair, its peer) aborted and
// records the code; every later wait of the CTA returns at once. The waits and the remote
// arrivals of a pair use the default (CTA-scope) semantics: cluster-scope acquires in the
// softmax warps' waits cost ~0.7 us per tile step (15.7 against 12.1 ms at config 4).
__device__ __forceinline__ bool pf_try(uint32_t addr, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; "
        "selp.u32 %0, 1, 0, p; }"
        : "=r"(ok) : "r"(addr), "r"(parity) : "memory");
    return ok;
}
__device__ __forceinline__ bool pf_test(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2; "
        "selp.u32 %0, 1, 0, p; }"
        : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok;
}

// Bounded wait for a phase, without the abort check: for copies and MMAs that must be
// done before the CTA may exit.
__device__ __forceinline__ void pf_drain(uint64_t *bar, uint32_t parity) {
    const uint32_t addr = smem_u32(bar);
    for (int it = 0; it < (1 << 20); it++)
        if (pf_try(addr, parity)) return;
}

__device__ __forceinline__ uint64_t pf_timer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// How the roles of one CTA synchronise, and how the two CTAs of a pair do.
struct SyncOne {
    int *abort;
    uint32_t *status;
    __device__ void fail(uint32_t code) const {
        *(volatile int *)abort = 1;
        dev_flag(status, code);
    }
    __device__ bool aborted() const { return *(volatile int *)abort != 0; }
    // every softmax thread arrives once it has read S (count 256) / written its half row of
    // P (count 256)
    __device__ void s_read(uint64_t *bar) const { mbar_arrive(bar); }
    __device__ void p_written(uint64_t *bar) const { mbar_arrive(bar); }
};
struct SyncPair {
    int *abort;
    uint32_t *status;
    uint32_t peer_abort;  // shared::cluster address of the other CTA's abort word
    __device__ void fail(uint32_t code) const {
        *(volatile int *)abort = 1;
        asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(peer_abort), "r"(1) : "memory");
        dev_flag(status, code);
    }
    __device__ bool aborted() const { return *(volatile int *)abort != 0; }
    // one arrival per softmax warp of either CTA on rank 0's barrier (count 16): the lanes'
    // TMEM reads of S / stores of P (each lane fenced them) are ordered before lane 0's
    // arrival
    __device__ void s_read(uint64_t *bar) const {
        __syncwarp();
        if ((threadIdx.x & 31) == 0) mbar_arrive_cluster(mapa_shared(bar, 0));
    }
    __device__ void p_written(uint64_t *bar) const { s_read(bar); }
};

template <class Sync>
__device__ bool pf_wait(const Sync &sy, uint64_t *bar, uint32_t parity, uint32_t code) {
    const uint32_t addr = smem_u32(bar);
    uint64_t t0 = 0;
    for (uint32_t it = 0;; ++it) {
        if (pf_try(addr, parity)) return true;
        if ((it & 255) == 0) {
            if (sy.aborted()) return false;
            const uint64_t now = pf_timer();
            if (it == 0) t0 = now;
            else if (now - t0 > 2000000000ull) {
                sy.fail(code);
                return false;
            }
        }
    }
}

// Softmax, rescale and epilogue (warps 2-9): two threads per query row r of the tile (its
// TMEM lane), one per half of the 128 keys of a tile and of the 256 output columns.
template <bool ACT_BF16, bool OUT_BF16, class Smem, class Sync>
__device__ __forceinline__ void softmax_role(Smem &sm, const Sync &sy, uint32_t tmem, int warp,
                                             int lane, int h, int t0, int p0, int T, int nq,
                                             int n_kt, const void *__restrict__ gate,
                                             void *__restrict__ out) {
    const uint32_t tO = tmem + TM_O;
    const int q4 = warp & 3;
    const int hf = (warp - 2) >> 2;
    const int r = q4 * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const int qpos = p0 + t0 + r;
    const float sc2 = 1.4426950408889634f * 0.0625f;  // log2(e) / sqrt(256)
    float m_run = -INFINITY, l_run = 0.0f;
    bool ok = true;
    // every softmax warp runs all n_kt iterations and the named barrier of each, also
    // after a failed wait (then skipping the tensor-memory work), so none is left waiting
    for (int j = 0; j < n_kt; j++) {
        const int b = j & 1;
        if (ok) ok = pf_wait(sy, &sm.s_full, j & 1, VX_DEV_TIMEOUT_MMA);
        ok = __all_sync(0xffffffffu, ok);  // warp-uniform: tcgen05.ld/st are warp-wide
        constexpr int HK = KT / 2;
        float s[HK];
        float mloc = -INFINITY;
        if (ok) {
            tc_fence_after();
            tmem_ld64(tmem + lane_off + hf * HK, s);  // four loads in flight, one wait
            tc_fence_before();
            sy.s_read(&sm.s_empty);
            const int kbase = j * KT + hf * HK;
            // causal mask only on tiles reaching past the tile's first query (CTA-uniform)
            if (j * KT + KT - 1 > p0 + t0) {
#pragma unroll
                for (int c = 0; c < HK; c++)
                    if (kbase + c > qpos) s[c] = -INFINITY;
            }
            // row max over this half as a tree
            float mx[16];
#pragma unroll
            for (int i = 0; i < 16; i++)
                mx[i] = fmaxf(fmaxf(s[4 * i], s[4 * i + 1]), fmaxf(s[4 * i + 2], s[4 * i + 3]));
#pragma unroll
            for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
                for (int i = 0; i < w; i++) mx[i] = fmaxf(mx[i], mx[i + w]);
            mloc = mx[0];
        }
        // ... and over both halves (the two threads of a row), through shared memory
        sm.xmax[b][hf][r] = mloc;
        named_bar_sync(1, 256);
        const float mpart = sm.xmax[b][hf ^ 1][r];
        if (!ok) continue;
        const float mt = fmaxf(mloc, mpart) * sc2;
        float alpha = 1.0f;
        const bool grow = mt > m_run + RESCALE_LOG2;
        if (grow) {
            alpha = (m_run == -INFINITY) ? 0.0f : exp2f(m_run - mt);
            m_run = mt;
        }
        // rescale this warp's half of its O rows when one of its rows raised its max (not
        // on the first tile of a row, where O holds nothing yet), once O += P(j-1) V(j-1)
        // is done
        const bool need = grow && alpha > 0.0f;
        if (__any_sync(0xffffffffu, need)) {
            ok = pf_wait(sy, &sm.pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, VX_DEV_TIMEOUT_MMA);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) continue;
            tc_fence_after();
#pragma unroll 1
            for (int i = 0; i < HDP / 32; i++) {
                float o[16];
                const uint32_t ta = tO + lane_off + hf * (HDP / 2) + 16 * i;
                tmem_ld16(ta, o);
#pragma unroll
                for (int e = 0; e < 16; e++) o[e] *= alpha;
                tmem_st16(ta, o);
            }
        }
        // P buffer b is free once O += P(j-2) V(j-2) is done
        if (j >= 2) {
            ok = pf_wait(sy, &sm.pv_done[b], ((j >> 1) - 1) & 1, VX_DEV_TIMEOUT_MMA);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) continue;
            tc_fence_after();
        }
        // P(j): this half's 64 keys as 32 columns of bf16 pairs
        float ls[4] = {0.f, 0.f, 0.f, 0.f};
        const float nm = -m_run;
        uint32_t pw[32];
#pragma unroll
        for (int u = 0; u < 8; u++) {
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float pa = ex2_approx(fmaf(s[u * 8 + 2 * e], sc2, nm));
                const float pb = ex2_approx(fmaf(s[u * 8 + 2 * e + 1], sc2, nm));
                ls[e] += pa + pb;
                pw[4 * u + e] = pack_bf16x2(pa, pb);
            }
        }
        tmem_st32(tmem + TM_P + 64u * b + lane_off + 32 * hf, pw);
        tmem_st_wait();
        tc_fence_before();
        l_run = fmaf(l_run, alpha, (ls[0] + ls[1]) + (ls[2] + ls[3]));
        sy.p_written(&sm.p_full[b]);
    }
    // the row sum is the sum of both halves' partial sums (same maxima, same rescales)
    sm.xsum[hf][r] = l_run;
    named_bar_sync(1, 256);
    const float l_row = l_run + sm.xsum[hf ^ 1][r];
    // bf16 gate: this thread's half row of the gate (128 values, 256 contiguous bytes) is
    // requested before O is final, and the gated row goes from registers straight to the
    // output, with no staging pass through shared memory. The sigmoid uses the SFU's 2^x
    // and reciprocal (a few ulp; the result is rounded to bf16 or compared at 2e-2):
    // with the correctly rounded expf and division the 32K sigmoids of a tile took
    // ~10 us per CTA.
    const int t_row = t0 + r;
    uint4 graw[HDP / 16];
    if constexpr (ACT_BF16) {
        if (t_row < T) {
            const uint4 *gp = reinterpret_cast<const uint4 *>(
                static_cast<const uint16_t *>(gate) + ((size_t)t_row * nq + h) * HDP +
                hf * (HDP / 2));
#pragma unroll
            for (int k = 0; k < HDP / 16; k++) graw[k] = gp[k];
        }
    }
    if (ok) ok = pf_wait(sy, &sm.o_final, 0, VX_DEV_TIMEOUT_MMA);
    ok = __all_sync(0xffffffffu, ok);
    if (ok && ACT_BF16) {
        tc_fence_after();
        const float inv = l_row > 0.0f ? 1.0f / l_row : 0.0f;
        const size_t obase = ((size_t)t_row * nq + h) * HDP + hf * (HDP / 2);
#pragma unroll 1
        for (int i = 0; i < HDP / 128; i++) {  // 64 columns per load round
            float o[64];
            tmem_ld64(tO + lane_off + hf * (HDP / 2) + 64 * i, o);
            if (t_row >= T) continue;
#pragma unroll
            for (int k = 0; k < 8; k++) {  // 8 columns per 16-byte gate word group
                const uint4 gv = graw[8 * i + k];
                const uint32_t gw4[4] = {gv.x, gv.y, gv.z, gv.w};
                float a[8];
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const float g0 = bf16_to_f32(gw4[e] & 0xffffu), g1 = bf16_to_f32(gw4[e] >> 16);
                    a[2 * e] = o[8 * k + 2 * e] * inv * __fdividef(1.0f, 1.0f + __expf(-g0));
                    a[2 * e + 1] = o[8 * k + 2 * e + 1] * inv * __fdividef(1.0f, 1.0f + __expf(-g1));
                }
                const size_t oi = obase + 64 * i + 8 * k;
                if constexpr (OUT_BF16) {
                    *reinterpret_cast<uint4 *>(static_cast<uint16_t *>(out) + oi) =
                        make_uint4(pack_bf16x2(a[0], a[1]), pack_bf16x2(a[2], a[3]),
                                   pack_bf16x2(a[4], a[5]), pack_bf16x2(a[6], a[7]));
                } else {
                    float4 *op = reinterpret_cast<float4 *>(static_cast<float *>(out) + oi);
                    op[0] = make_float4(a[0], a[1], a[2], a[3]);
                    op[1] = make_float4(a[4], a[5], a[6], a[7]);
                }
            }
        }
    } else if (ok) {
        // fp32 gate: O / l into a row-major fp32 staging tile over the (now idle) slot
        // ring and P buffers, 16-byte chunks of a row XOR-swizzled by the row so a warp's
        // stores spread over banks; the gated output follows after the CTA barrier
        tc_fence_after();
        const float inv = l_row > 0.0f ? 1.0f / l_row : 0.0f;
        float4 *row = reinterpret_cast<float4 *>(sm.ring[0]) + r * (HDP / 4);
#pragma unroll 1
        for (int i = 0; i < HDP / 128; i++) {  // 64 columns per load round
            float o[64];
            tmem_ld64(tO + lane_off + hf * (HDP / 2) + 64 * i, o);
#pragma unroll
            for (int k = 0; k < 16; k++) {
                const int ch = (hf * (HDP / 2) + 64 * i) / 4 + k;
                row[ch ^ (r & 7)] = make_float4(o[4 * k] * inv, o[4 * k + 1] * inv,
                                                o[4 * k + 2] * inv, o[4 * k + 3] * inv);
            }
        }
    } else {
        *(volatile int *)sy.abort = 1;
    }
}

// fp32 gate, after the CTA barrier: gated output rows from the staging tile with coalesced
// 16-byte loads of the gate and stores of the output; the gate loads of GB iterations are
// issued together before any is used, so a thread waits for one round trip per GB
// iterations instead of one each (the one-at-a-time form took ~14 us per CTA)
template <bool OUT_BF16>
__device__ __forceinline__ void staged_gate_out(const uint8_t *stage_bytes,
                                                const float *__restrict__ gate,
                                                void *__restrict__ out, int tid, int t0, int T,
                                                int nq, int h) {
    constexpr int VEC = OUT_BF16 ? 8 : 4;
    constexpr int PER_ROW = HDP / VEC;
    constexpr int N_IT = QT * PER_ROW;
    constexpr int GB = 6;
    const float4 *stage = reinterpret_cast<const float4 *>(stage_bytes);
    for (int it0 = tid; it0 < N_IT; it0 += GB * PF_THREADS) {
        uint32_t gw[GB][VEC];
#pragma unroll
        for (int u = 0; u < GB; u++) {
            const int it = it0 + u * PF_THREADS;
            const int rr = it / PER_ROW, c0 = (it % PER_ROW) * VEC;
            if (it >= N_IT || t0 + rr >= T) continue;
            const size_t base = ((size_t)(t0 + rr) * nq + h) * HDP + c0;
            const uint4 *gp = reinterpret_cast<const uint4 *>(gate + base);
#pragma unroll
            for (int k = 0; k < VEC / 4; k++) {
                const uint4 f = gp[k];
                gw[u][4 * k] = f.x; gw[u][4 * k + 1] = f.y; gw[u][4 * k + 2] = f.z; gw[u][4 * k + 3] = f.w;
            }
        }
#pragma unroll
        for (int u = 0; u < GB; u++) {
            const int it = it0 + u * PF_THREADS;
            const int rr = it / PER_ROW, c0 = (it % PER_ROW) * VEC;
            if (it >= N_IT || t0 + rr >= T) continue;
            const size_t base = ((size_t)(t0 + rr) * nq + h) * HDP + c0;
            float o[VEC];
#pragma unroll
            for (int k = 0; k < VEC / 4; k++) {
                const float4 f = stage[rr * (HDP / 4) + ((c0 / 4 + k) ^ (rr & 7))];
                o[4 * k] = f.x; o[4 * k + 1] = f.y; o[4 * k + 2] = f.z; o[4 * k + 3] = f.w;
            }
#pragma unroll
            for (int e = 0; e < VEC; e++)
                o[e] = o[e] * (1.0f / (1.0f + expf(-__uint_as_float(gw[u][e]))));
            if constexpr (OUT_BF16) {
                uint32_t w[4];
#pragma unroll
                for (int k = 0; k < 4; k++)
                    w[k] = (uint32_t)f32_to_bf16(o[2 * k]) | ((uint32_t)f32_to_bf16(o[2 * k + 1]) << 16);
                *reinterpret_cast<uint4 *>(static_cast<uint16_t *>(out) + base) =
                    make_uint4(w[0], w[1], w[2], w[3]);
            } else {
                *reinterpret_cast<float4 *>(static_cast<float *>(out) + base) =
                    make_float4(o[0], o[1], o[2], o[3]);
            }
        }
    }
}

// One CTA per (query tile, query head) on one SM.
template <bool ACT_BF16, bool OUT_BF16>
__global__ void __launch_bounds__(PF_THREADS, 1)
prefill_attn_tc(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                const __grid_constant__ CUtensorMap tmv, const void *__restrict__ gate,
                void *__restrict__ out, int T, int p0, int nq, int nkv, int cap,
                uint32_t *status) {
    extern __shared__ uint8_t pf_smem_raw[];
    PfSmem &sm = *reinterpret_cast<PfSmem *>(((uintptr_t)pf_smem_raw + 1023) & ~(uintptr_t)1023);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n_qt = (T + QT - 1) / QT;
    const int qt = n_qt - 1 - (int)(blockIdx.x / nq);  // longest tiles first
    const int h = blockIdx.x % nq;
    const int kvh = h * nkv / nq;
    const int t0 = qt * QT;
    const int t_end = min(T, t0 + QT);
    const int n_kt = (p0 + t_end + KT - 1) / KT;  // key tiles up to the last query's position

    if (tid == 0) {
        mbar_init(&sm.qfull, 1);
        for (int i = 0; i < NS; i++) {
            mbar_init(&sm.full[i], 1);
            mbar_init(&sm.empty[i], 1);
        }
        mbar_init(&sm.s_full, 1);
        mbar_init(&sm.s_empty, 256);
        for (int i = 0; i < 2; i++) {
            mbar_init(&sm.p_full[i], 256);
            mbar_init(&sm.pv_done[i], 1);
        }
        mbar_init(&sm.o_final, 1);
        mbar_init(&sm.mma_done, 1);
        mbar_init(&sm.qk_done, 1);
        sm.abort = 0;
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc(&sm.tmem_base, 512);
        tmem_relinquish();
        if (lane == 0) { tma_prefetch_desc(&tmq); tma_prefetch_desc(&tmk); tma_prefetch_desc(&tmv); }
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;
    const uint32_t tO = tmem + TM_O;
    const SyncOne sy{&sm.abort, status};

    if (warp == 0) {
        if (lane == 0) {  // ---- TMA producer: each ring refilled as soon as a slot frees
            mbar_arrive_expect_tx(&sm.qfull, 4 * QT * 128);
            for (int c = 0; c < 4; c++) tma_load_2d(sm.q[c], &tmq, c * 64, h * T + t0, &sm.qfull);
            const int krow0 = kvh * cap;  // rows of this KV head in the [nkv*cap][256] maps
            const uint32_t n_all = 4u * n_kt;  // chunks per ring
            uint32_t nk = 0, nv = 0;           // loads issued into the K and V rings
            uint32_t spins = 0;
            uint64_t tw0 = 0;
            while (nk < n_all || nv < n_all) {
                bool did = false;
                if (nk < n_all && (nk < NKS || pf_test(&sm.empty[nk % NKS], ((nk / NKS) - 1) & 1))) {
                    const uint32_t s2 = nk % NKS;  // K(m): dims [64c, 64c + 64) of 128 keys
                    mbar_arrive_expect_tx(&sm.full[s2], 16384);
                    tma_load_2d(sm.ring[s2], &tmk, (nk & 3) * 64, krow0 + (nk >> 2) * KT, &sm.full[s2]);
                    nk++;
                    did = true;
                }
                if (nv < n_all && (nv < NVS || pf_test(&sm.empty[NKS + nv % NVS], ((nv / NVS) - 1) & 1))) {
                    // V(t): keys [32c, 32c + 32), all dims, as four [32 keys x 64 dims] blocks
                    const uint32_t s2 = NKS + nv % NVS;
                    mbar_arrive_expect_tx(&sm.full[s2], 16384);
                    tma_load_3d(sm.ring[s2], &tmv, 0, krow0 + (nv >> 2) * KT + 32 * (nv & 3), 0,
                                &sm.full[s2]);
                    nv++;
                    did = true;
                }
                if (did) {
                    spins = 0;
                } else {  // bounded like every wait: ~2 s without a free slot aborts the CTA
                    if ((spins++ & 255) == 0) {
                        if (sy.aborted()) break;
                        const uint64_t now = pf_timer();
                        if (spins == 1) tw0 = now;
                        else if (now - tw0 > 2000000000ull) {
                            sy.fail(VX_DEV_TIMEOUT_TMA);
                            break;
                        }
                    }
                }
            }
            // every copy issued lands before the CTA can exit, also when a role has aborted
            // (on the normal path all have been consumed, so these return at once)
            for (uint32_t i = nk > NKS ? nk - NKS : 0; i < nk; i++)
                pf_drain(&sm.full[i % NKS], (i / NKS) & 1);
            for (uint32_t i = nv > NVS ? nv - NVS : 0; i < nv; i++)
                pf_drain(&sm.full[NKS + i % NVS], (i / NVS) & 1);
            pf_drain(&sm.qfull, 0);
        }
    } else if (warp == 1) {
        if (lane == 0) {  // ---- MMA issuer, S stream: S = Q K(m)^T once the softmax has read S(m-1)
            const uint32_t id1 = idesc_bf16(128, KT, false, false);
            const uint64_t dq0 = sdesc_sw128(smem_u32(sm.q[0]), 16, 1024);
            const uint64_t dr0 = sdesc_sw128(smem_u32(sm.ring[0]), 16, 1024);
            bool ok = pf_wait(sy, &sm.qfull, 0, VX_DEV_TIMEOUT_TMA);
            for (int m = 0; m < n_kt && ok; m++) {
                if (m >= 1) ok = pf_wait(sy, &sm.s_empty, (m - 1) & 1, VX_DEV_TIMEOUT_MMA);
                for (int c = 0; c < 4 && ok; c++) {
                    const uint32_t i = 4u * m + c, s2 = i % NKS;
                    ok = pf_wait(sy, &sm.full[s2], (i / NKS) & 1, VX_DEV_TIMEOUT_TMA);
                    if (!ok) break;
                    tc_fence_after();
                    const uint64_t dq = sdesc_add(dq0, c * (QT * 128));
                    const uint64_t dk = sdesc_add(dr0, s2 * 16384);
#pragma unroll
                    for (int kk = 0; kk < 4; kk++)
                        mma_bf16(tmem, sdesc_add(dq, kk * 32), sdesc_add(dk, kk * 32), id1,
                                 (c | kk) != 0);
                    mma_commit(&sm.empty[s2]);
                }
                if (!ok) break;
                mma_commit(&sm.s_full);
            }
            mma_commit(&sm.qk_done);
            pf_drain(&sm.qk_done, 0);
        }
    } else if (warp == PF_THREADS / 32 - 1) {
        if (lane == 0) {  // ---- MMA issuer, O stream: O += P(t) V(t) once P(t) is written,
                          // P from tensor memory (buffer t & 1)
            const uint32_t id2 = idesc_bf16(128, HDP, false, true);
            const uint64_t dv0 = sdesc_sw128(smem_u32(sm.ring[0]), 32 * 128, 1024);
            bool ok = true;
            for (int t = 0; t < n_kt && ok; t++) {
                const int pb = t & 1;
                ok = pf_wait(sy, &sm.p_full[pb], (t >> 1) & 1, VX_DEV_TIMEOUT_MMA);
                for (int c = 0; c < 4 && ok; c++) {
                    const uint32_t i = 4u * t + c, s2 = NKS + i % NVS;
                    ok = pf_wait(sy, &sm.full[s2], (i / NVS) & 1, VX_DEV_TIMEOUT_TMA);
                    if (!ok) break;
                    tc_fence_after();
                    const uint64_t dv = sdesc_add(dv0, s2 * 16384);
#pragma unroll
                    for (int k2 = 0; k2 < 2; k2++) {
                        const int kk = 2 * c + k2;  // 16-key step: 8 columns of bf16 pairs
                        mma_bf16_ts(tO, tmem + TM_P + 64u * pb + 8u * kk, sdesc_add(dv, k2 * 2048), id2,
                                    (t > 0 || kk > 0) ? 1u : 0u);
                    }
                    mma_commit(&sm.empty[s2]);
                }
                if (!ok) break;
                mma_commit(&sm.pv_done[pb]);
                if (t == n_kt - 1) mma_commit(&sm.o_final);
            }
            mma_commit(&sm.mma_done);
            pf_drain(&sm.mma_done, 0);
        }
    } else {
        softmax_role<ACT_BF16, OUT_BF16>(sm, sy, tmem, warp, lane, h, t0, p0, T, nq, n_kt, gate,
                                         out);
    }
    // lanes that skipped a lane-0 role wait for it here, so whole warps reach the CTA
    // barrier together (it requires converged warps)
    __syncwarp();
    __syncthreads();
    if (!ACT_BF16 && !sy.aborted())
        staged_gate_out<OUT_BF16>(sm.ring[0], static_cast<const float *>(gate), out, tid, t0, T,
                                  nq, h);
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// A 2-CTA cluster per (query tile, two query heads of one KV head): the two heads' 128
// query rows form one M = 256 tcgen05 MMA over both SMs, each SM holding its head's Q and
// P and HALF of every K/V tile (64 of the 128 keys of a K chunk; 128 of the 256 dims of a
// V chunk), so each SM moves half the K/V bytes of the single-SM kernel from L2 into
// shared memory, and its tensor pipe reads half the B operand. Rank 0 issues the MMAs and
// owns the ring and Q barriers (both CTAs' copies count on them); the MMA completions
// arrive on the barriers of both CTAs; the softmax warps of both CTAs report S read and P
// written to rank 0's barriers, one arrival per warp.
template <bool ACT_BF16, bool OUT_BF16>
__global__ void __launch_bounds__(PF_THREADS, 1)
prefill_attn_pair(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                  const __grid_constant__ CUtensorMap tmv, const void *__restrict__ gate,
                  void *__restrict__ out, int T, int p0, int nq, int nkv, int cap,
                  uint32_t *status) {
    extern __shared__ uint8_t pf_smem_raw[];
    PairSmem &sm = *reinterpret_cast<PairSmem *>(((uintptr_t)pf_smem_raw + 1023) & ~(uintptr_t)1023);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = cluster_rank();
    const int n_qt = (T + QT - 1) / QT;
    const int pairs_per_tile = nq >> 1;
    const int pr = (int)(blockIdx.x >> 1);
    const int qt = n_qt - 1 - pr / pairs_per_tile;  // longest tiles first
    const int h = 2 * (pr % pairs_per_tile) + (int)rank;  // heads 2i, 2i+1: one KV head
    const int kvh = h * nkv / nq;
    const int t0 = qt * QT;
    const int t_end = min(T, t0 + QT);
    const int n_kt = (p0 + t_end + KT - 1) / KT;

    if (tid == 0) {
        mbar_init(&sm.qfull, 1);
        for (int i = 0; i < NS2; i++) {
            mbar_init(&sm.full[i], 1);
            mbar_init(&sm.empty[i], 1);
        }
        mbar_init(&sm.s_full, 1);
        mbar_init(&sm.s_empty, 16);
        for (int i = 0; i < 2; i++) {
            mbar_init(&sm.p_full[i], 16);
            mbar_init(&sm.pv_done[i], 1);
        }
        mbar_init(&sm.o_final, 1);
        mbar_init(&sm.mma_done, 1);
        mbar_init(&sm.qk_done, 1);
        sm.abort = 0;
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc_pair(&sm.tmem_base, 512);
        tmem_relinquish_pair();
        if (lane == 0) { tma_prefetch_desc(&tmq); tma_prefetch_desc(&tmk); tma_prefetch_desc(&tmv); }
    }
    tc_fence_before();
    __syncwarp();
    cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;
    const uint32_t tO = tmem + TM_O;
    const SyncPair sy{&sm.abort, status, mapa_shared(&sm.abort, rank ^ 1u)};
    // MMA completion: one arrival on the barrier of each CTA
    auto commit_both = [](uint64_t *bar) { mma_commit_pair_both(bar); };

    if (warp == 0) {
        if (lane == 0) {  // ---- TMA producer (both CTAs): this CTA's halves of the K/V chunks
            if (rank == 0) mbar_arrive_expect_tx(&sm.qfull, 2 * 4 * QT * 128);
            const uint32_t lq = mapa_shared(&sm.qfull, 0);
            for (int c = 0; c < 4; c++) tma_load_2d_pair(sm.q[c], &tmq, c * 64, h * T + t0, lq);
            const int krow0 = kvh * cap;
            const uint32_t n_all = 4u * n_kt;
            uint32_t nk = 0, nv = 0;
            uint32_t spins = 0;
            uint64_t tw0 = 0;
            while (nk < n_all || nv < n_all) {
                bool did = false;
                if (nk < n_all && (nk < NKS2 || pf_test(&sm.empty[nk % NKS2], ((nk / NKS2) - 1) & 1))) {
                    // K(m) chunk c: dims [64c, 64c + 64) of keys [64 rank, 64 rank + 64)
                    const uint32_t s2 = nk % NKS2;
                    if (rank == 0) mbar_arrive_expect_tx(&sm.full[s2], 2 * SLOT2);
                    tma_load_2d_pair(sm.ring[s2], &tmk, (nk & 3) * 64,
                                     krow0 + (nk >> 2) * KT + 64 * (int)rank,
                                     mapa_shared(&sm.full[s2], 0));
                    nk++;
                    did = true;
                }
                if (nv < n_all && (nv < NVS2 || pf_test(&sm.empty[NKS2 + nv % NVS2], ((nv / NVS2) - 1) & 1))) {
                    // V(t) chunk c: keys [32c, 32c + 32), dims [128 rank, 128 rank + 128)
                    const uint32_t s2 = NKS2 + nv % NVS2;
                    if (rank == 0) mbar_arrive_expect_tx(&sm.full[s2], 2 * SLOT2);
                    tma_load_3d_pair(sm.ring[s2], &tmv, 0, krow0 + (nv >> 2) * KT + 32 * (nv & 3),
                                     2 * (int)rank, mapa_shared(&sm.full[s2], 0));
                    nv++;
                    did = true;
                }
                if (did) {
                    spins = 0;
                } else {
                    if ((spins++ & 255) == 0) {
                        if (sy.aborted()) break;
                        const uint64_t now = pf_timer();
                        if (spins == 1) tw0 = now;
                        else if (now - tw0 > 2000000000ull) {
                            sy.fail(VX_DEV_TIMEOUT_TMA);
                            break;
                        }
                    }
                }
            }
            if (rank == 0) {  // both CTAs' copies count on these barriers
                for (uint32_t i = nk > NKS2 ? nk - NKS2 : 0; i < nk; i++)
                    pf_drain(&sm.full[i % NKS2], (i / NKS2) & 1);
                for (uint32_t i = nv > NVS2 ? nv - NVS2 : 0; i < nv; i++)
                    pf_drain(&sm.full[NKS2 + i % NVS2], (i / NVS2) & 1);
                pf_drain(&sm.qfull, 0);
            }
            if (sy.aborted()) {
                // after an abort the two CTAs may have issued different numbers of copies,
                // which no barrier then tracks: give those in flight 200 us to land
                const uint64_t tw = pf_timer();
                while (pf_timer() - tw < 200000ull) {
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {  // ---- MMA issuer, S stream (rank 0)
            const uint32_t id1 = idesc_bf16(256, KT, false, false);
            const uint64_t dq0 = sdesc_sw128(smem_u32(sm.q[0]), 16, 1024);
            const uint64_t dr0 = sdesc_sw128(smem_u32(sm.ring[0]), 16, 1024);
            bool ok = pf_wait(sy, &sm.qfull, 0, VX_DEV_TIMEOUT_TMA);
            for (int m = 0; m < n_kt && ok; m++) {
                if (m >= 1) ok = pf_wait(sy, &sm.s_empty, (m - 1) & 1, VX_DEV_TIMEOUT_MMA);
                for (int c = 0; c < 4 && ok; c++) {
                    const uint32_t i = 4u * m + c, s2 = i % NKS2;
                    ok = pf_wait(sy, &sm.full[s2], (i / NKS2) & 1, VX_DEV_TIMEOUT_TMA);
                    if (!ok) break;
                    tc_fence_after();
                    const uint64_t dq = sdesc_add(dq0, c * (QT * 128));
                    const uint64_t dk = sdesc_add(dr0, s2 * SLOT2);
#pragma unroll
                    for (int kk = 0; kk < 4; kk++)
                        mma_bf16_pair(tmem, sdesc_add(dq, kk * 32), sdesc_add(dk, kk * 32), id1,
                                      (c | kk) != 0);
                    commit_both(&sm.empty[s2]);
                }
                if (!ok) break;
                commit_both(&sm.s_full);
            }
            mma_commit_pair(mapa_shared(&sm.qk_done, 0));
            pf_drain(&sm.qk_done, 0);
        }
    } else if (warp == PF_THREADS / 32 - 1) {
        if (lane == 0 && rank == 0) {  // ---- MMA issuer, O stream (rank 0)
            const uint32_t id2 = idesc_bf16(256, HDP, false, true);
            const uint64_t dv0 = sdesc_sw128(smem_u32(sm.ring[0]), 32 * 128, 1024);
            bool ok = true;
            for (int t = 0; t < n_kt && ok; t++) {
                const int pb = t & 1;
                ok = pf_wait(sy, &sm.p_full[pb], (t >> 1) & 1, VX_DEV_TIMEOUT_MMA);
                for (int c = 0; c < 4 && ok; c++) {
                    const uint32_t i = 4u * t + c, s2 = NKS2 + i % NVS2;
                    ok = pf_wait(sy, &sm.full[s2], (i / NVS2) & 1, VX_DEV_TIMEOUT_TMA);
                    if (!ok) break;
                    tc_fence_after();
                    const uint64_t dv = sdesc_add(dv0, s2 * SLOT2);
#pragma unroll
                    for (int k2 = 0; k2 < 2; k2++) {
                        const int kk = 2 * c + k2;
                        mma_bf16_pair_ts(tO, tmem + TM_P + 64u * pb + 8u * kk, sdesc_add(dv, k2 * 2048),
                                         id2, (t > 0 || kk > 0) ? 1u : 0u);
                    }
                    commit_both(&sm.empty[s2]);
                }
                if (!ok) break;
                commit_both(&sm.pv_done[pb]);
                if (t == n_kt - 1) commit_both(&sm.o_final);
            }
            mma_commit_pair(mapa_shared(&sm.mma_done, 0));
            pf_drain(&sm.mma_done, 0);
        }
    } else {
        softmax_role<ACT_BF16, OUT_BF16>(sm, sy, tmem, warp, lane, h, t0, p0, T, nq, n_kt, gate,
                                         out);
    }
    __syncwarp();
    __syncthreads();
    if (!ACT_BF16 && !sy.aborted())
        staged_gate_out<OUT_BF16>(sm.ring[0], static_cast<const float *>(gate), out, tid, t0, T,
                                  nq, h);
    // neither CTA leaves (or frees TMEM) while the other may still arrive on its barriers
    // or rank 0's MMAs may still touch its memory: rank 0's issuers waited for their MMAs
    tc_fence_before();
    __syncwarp();
    cluster_sync();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, 512);
    }
}

template <bool A, bool O>
int launch_attn(const CUtensorMap &mq, const CUtensorMap &mk, const CUtensorMap &mv,
                const void *gate, void *out, int T, int p0, int nq, int nkv, int cap, bool pair,
                cudaStream_t st, char *err, size_t errlen) {
    const int n_qt = (T + QT - 1) / QT;
    if (!pair) {
        const size_t smem = sizeof(PfSmem) + 1024;
        if (ensure_smem_attr((const void *)prefill_attn_tc<A, O>, smem, err, errlen)) return -1;
        prefill_attn_tc<A, O><<<n_qt * nq, PF_THREADS, smem, st>>>(mq, mk, mv, gate, out, T, p0,
                                                                     nq, nkv, cap, dev_status());
        VX_CK(cudaGetLastError());
        return 0;
    }
    const size_t smem = sizeof(PairSmem) + 1024;
    if (ensure_smem_attr((const void *)prefill_attn_pair<A, O>, smem, err, errlen)) return -1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n_qt * nq);  // nq even: whole pairs
    cfg.blockDim = dim3(PF_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    VX_CK(cudaLaunchKernelEx(&cfg, prefill_attn_pair<A, O>, mq, mk, mv, gate, out, T, p0, nq, nkv,
                             cap, dev_status()));
    return 0;
}

}  // namespace
}  // namespace vx27

using namespace vx27;

extern "C" size_t vx27_gqa_prefill_workspace_size(int T, int nq, int hd) {
    if (T <= 0 || nq <= 0 || hd <= 0) return 0;
    // normalised, rotated bf16 q [nq][T][hd] plus the TMA boxes' overhang of one tile
    return ((size_t)nq * T + QT) * hd * sizeof(uint16_t);
}

extern "C" int vx27_gqa_prefill(const void *q_in, const void *k_in, const void *v_in,
                                const void *gate, const float *q_norm_w, const float *k_norm_w,
                                const float *rope_table, int rope_table_len, int p0,
                                void *k_cache, void *v_cache, int cap, void *out,
                                void *workspace, size_t workspace_bytes, int T, int nq, int nkv,
                                int hd, int rope_dim, float eps, int flags, void *stream,
                                char *err, size_t errlen) {
    const char *fn = "vx27_gqa_prefill";
    if (hd != HDP) return fail(err, errlen, "%s: hd=%d unsupported (256 only)", fn, hd);
    if (T <= 0 || nq <= 0 || nkv <= 0 || nq % nkv || nq * ((T + QT - 1) / QT) > (1 << 30))
        return fail(err, errlen, "%s: bad shape T=%d nq=%d nkv=%d", fn, T, nq, nkv);
    if (p0 < 0 || p0 + T > cap)
        return fail(err, errlen, "%s: positions [%d, %d) exceed the cache capacity %d", fn, p0,
                    p0 + T, cap);
    if (rope_dim < 0 || rope_dim > hd || (rope_dim & 15) || p0 + T > rope_table_len)
        return fail(err, errlen, "%s: rope_dim=%d / table of %d positions", fn, rope_dim,
                    rope_table_len);
    if (!q_in || !k_in || !v_in || !gate || !q_norm_w || !k_norm_w || !k_cache || !v_cache ||
        !out || !workspace || (rope_dim && !rope_table))
        return fail(err, errlen, "%s: null pointer argument", fn);
    if (((uintptr_t)gate | (uintptr_t)out | (uintptr_t)q_in | (uintptr_t)k_in | (uintptr_t)v_in |
         (uintptr_t)k_cache | (uintptr_t)v_cache) & 15)
        return fail(err, errlen, "%s: activations, caches and out must be 16-byte aligned", fn);
    if (workspace_bytes < vx27_gqa_prefill_workspace_size(T, nq, hd))
        return fail(err, errlen, "%s: workspace of %zu bytes, need %zu", fn, workspace_bytes,
                    vx27_gqa_prefill_workspace_size(T, nq, hd));
    cudaStream_t st = (cudaStream_t)stream;
    uint16_t *qn = (uint16_t *)workspace;
    const bool a = flags & VX27_F_ACT_BF16, one = flags & VX27_F_NORM_1P;
    const size_t prep_rows = (size_t)T * (nq + nkv);
    // one resident wave (five 8-warp blocks per SM at the kernel's 48 registers)
    const int pg = (int)std::min<size_t>((prep_rows + 7) / 8, (size_t)num_sms() * 5);
#define VX_P(A_, O_)                                                                         \
    prefill_prep_k<A_, O_><<<pg, 256, 0, st>>>(q_in, k_in, v_in, q_norm_w, k_norm_w,          \
                                               rope_table, rope_table_len, p0, qn,            \
                                               (uint16_t *)k_cache, (uint16_t *)v_cache, cap, \
                                               T, nq, nkv, rope_dim, eps, dev_status())
    if (a && one) VX_P(true, true);
    else if (a) VX_P(true, false);
    else if (one) VX_P(false, true);
    else VX_P(false, false);
#undef VX_P
    VX_CK(cudaGetLastError());
    // the last key tile may reach past p0 + T: give those slots finite values
    const int tail_end = min(cap, ((p0 + T + KT - 1) / KT) * KT);
    if (tail_end > p0 + T) {
        zero_slots_k<<<dim3(4, nkv), 256, 0, st>>>((uint16_t *)k_cache, (uint16_t *)v_cache,
                                                    cap, nkv, p0 + T, tail_end);
        VX_CK(cudaGetLastError());
    }
    // CTA pairs when two neighbouring query heads always share a KV head (even group size)
    const bool pair = !(flags & VX27_F_PREFILL_CTA1) && (nq / nkv) % 2 == 0;
    CUtensorMap mq, mk, mv;
    if (make_tmap_bf16_2d(&mq, qn, (uint64_t)nq * T, HDP, HDP * 2, 64, QT, err, errlen) ||
        make_tmap_bf16_2d(&mk, k_cache, (uint64_t)nkv * cap, HDP, HDP * 2, 64, pair ? KT / 2 : KT,
                          err, errlen) ||
        // V as [64-dim block][key][64 dims]: one copy brings a chunk's blocks (4, or this
        // SM's 2 in a pair) one after the other, the MN-major operand layout
        make_tmap_bf16_3d(&mv, v_cache, 64, (uint64_t)nkv * cap, HDP / 64, HDP * 2, 128, 64, 32,
                          pair ? 2 : 4, err, errlen))
        return -1;
    const bool o = flags & VX27_F_OUT_BF16;
#define VX_A(A_, O_) \
    launch_attn<A_, O_>(mq, mk, mv, gate, out, T, p0, nq, nkv, cap, pair, st, err, errlen)
    if (a && o) return VX_A(true, true);
    if (a) return VX_A(true, false);
    if (o) return VX_A(false, true);
    return VX_A(false, false);
#undef VX_A
}
