// K2 on the CUDA cores: split-KV flash decoding for small batches, where the work is a
// few (sequence, KV head) streams and the tensor-core kernel's per-CTA pipeline (TMEM
// allocation, q staging, a 12-slot ring ramping up per SM) is latency rather than
// bandwidth. One CTA per (split, KV head, sequence), two CTAs per SM, non-persistent:
//   thread 0      streams the range's cache rows as 32-position sub-tiles of K and V
//                 (16 KB each, one 1-D bulk copy per plane; a (sequence, KV head) keeps its
//                 positions contiguous, src/vx27_qfwd.c:183-184 keeps them per slot) into a
//                 3-stage ring;
//   all 8 warps   scores s[h][p] = q_h . k_p / 16 for the G query heads of the group
//                 (thread = position x 32-dim part, fp32 FMA, parts summed by shuffles);
//                 per head (warp h) the running max and sum, p = e^(s - m); then
//                 o[h][d] += p[h][p] v[p][d] with thread = dimension d.
// The result is the split's partial record (m, l, o) (vx27_gqa_combine merges them), or,
// with one split, the gated output itself. Arithmetic: q fp32, bf16 K/V widened exactly,
// fp32 products and sums (the reference: fp64 dot, fp32 softmax and sums,
// src/vx27_qfwd.c:186-211).
//
// Fused prologue (vx27_gqa_decode_fused): each CTA forms its group's q rows from the raw
// activations (QK RMSNorm with a double sum of squares, NeoX RoPE on dims < rope_dim, the
// rounding of vx27_gqa_append), and the CTA whose range holds the token's slot also forms
// the new K/V row, stores it in the cache and patches it into its staged sub-tile.
//
// With prefetch (VX27_F_PREFETCH_KV) the first sub-tiles are requested before the kernel
// waits for its predecessor on the stream (programmatic dependent launch); the caller
// guarantees that predecessor writes neither pos nor cache rows other than the token's.
// Waits on the ring are bounded (~2 s); a timeout sets the device status word and the CTA
// leaves after its issued copies have landed.
#include <math.h>
#include "common.cuh"
#include "../../include/vx27_gqa.h"

namespace vx27 {

int launch_gqa_combine(const float *parts, int n_parts, const void *gate, void *out, int B,
                       int nq, int flags, cudaStream_t st, char *err, size_t errlen, bool pdl);

namespace {

constexpr int HD = 256;
constexpr int SUB = 32;                     // cache positions per ring stage
constexpr int NST = 3;                      // ring stages
constexpr int CC_THREADS = 256;
constexpr int SUB_BYTES = SUB * HD * 2;     // 16 KB of one plane
constexpr int QPAD = 36;                    // floats per (head, 32-dim part) row of q

struct CcSmem {
    alignas(128) uint8_t k[NST][SUB_BYTES];
    alignas(128) uint8_t v[NST][SUB_BYTES];
    union {
        float y[10][HD];               // fused prologue: normalised rows before RoPE
        struct {
            alignas(16) float q[8][8][QPAD];  // q[h][d / 32][q_slot(d)] (see q_slot)
            float sc[8][SUB];                 // scaled scores of the stage [head][position]
            alignas(16) float p[SUB][8];      // probabilities [position][head]
        };
    };
    float corr[8];                     // max correction of the stage per head
    float m[8], l[8];                  // final running max and sum per head
    double red[10][8];                 // fused prologue: per-warp sums of squares
    alignas(16) uint16_t kvrow[2][HD]; // fused prologue: the new K and V rows (bf16)
    uint64_t full[NST];
    int flag;
};
// two CTAs per SM (228 KB of shared memory, 1 KB of it reserved per CTA)
static_assert(2 * (sizeof(CcSmem) + 128 + 1024) <= 233472, "two CTAs per SM must fit");

// Within its 32-dim part, dim d's slot in the q row: the part's 8-dim chunks are stored in
// the order the score loop visits them (chunk c at step (c - part / 2) mod 4), so step u
// reads slots 8u..8u+7; with rows of 36 floats the 8 parts of a quarter warp then hit 8
// different 16-byte bank groups.
__device__ __forceinline__ int q_slot(int d) {
    const int part = d >> 5, c = (d >> 3) & 3, e = d & 7;
    return ((c - (part >> 1)) & 3) * 8 + e;
}

struct CcArgs {
    const uint16_t *kc, *vc;   // caches [B][nkv][cap][HD] bf16 (fused: the new row is written)
    const float *q;            // normalised q [B][nq][HD] (not fused)
    const int *pos;
    float *parts;              // partial records (n_splits > 1)
    const void *gate;
    void *out;                 // gated output (n_splits == 1)
    int cap, B, nq, nkv, n_splits, prefetch;
    // fused prologue
    const void *q_in, *k_in, *v_in;
    const float *qw, *kw, *rope;
    int rope_len, rope_dim, one_p;
    float eps;
    uint32_t *status;
};

__device__ __forceinline__ uint64_t cc_timer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Thread 0 waits for a stage (bounded, ~2 s), the CTA learns the outcome together.
__device__ __forceinline__ bool cc_wait_all(uint64_t *bar, uint32_t parity, CcSmem &sm,
                                            uint32_t *status) {
    if (threadIdx.x == 0) {
        const uint32_t addr = smem_u32(bar);
        uint64_t t0 = 0;
        int ok = 0;
        for (uint32_t it = 0;; ++it) {
            uint32_t done;
            asm volatile(
                "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; "
                "selp.u32 %0, 1, 0, p; }"
                : "=r"(done) : "r"(addr), "r"(parity) : "memory");
            if (done) { ok = 1; break; }
            if ((it & 255) == 0) {
                const uint64_t now = cc_timer();
                if (it == 0) t0 = now;
                else if (now - t0 > 2000000000ull) break;
            }
        }
        if (!ok) dev_flag(status, VX_DEV_TIMEOUT_TMA);
        sm.flag = ok;
    }
    __syncwarp();  // converged warps at the CTA barrier
    __syncthreads();
    return sm.flag != 0;
}

// Split s of sequence b covers sub-tiles [t0, t1) of the positions [0, pos[b]] (capped by
// the cache capacity), cut into n_splits nearly equal pieces.
struct CcRange {
    int n_pos, t0, t1;
};
__device__ __forceinline__ CcRange cc_range(int p, int cap, int n_splits, int s) {
    CcRange r;
    r.n_pos = min(p + 1, cap);
    if (r.n_pos < 0) r.n_pos = 0;
    const int subs = (r.n_pos + SUB - 1) / SUB;
    const int per = (subs + n_splits - 1) / n_splits;
    r.t0 = min(subs, s * per);
    r.t1 = min(subs, (s + 1) * per);
    return r;
}

template <int G, bool FUSED, bool ACT_BF16, bool OUT_BF16>
__global__ void __launch_bounds__(CC_THREADS, 2) gqa_split_cc(const __grid_constant__ CcArgs a) {
    extern __shared__ uint8_t cc_smem_raw[];
    CcSmem &sm = *reinterpret_cast<CcSmem *>(((uintptr_t)cc_smem_raw + 127) & ~(uintptr_t)127);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int s = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    if (tid == 0) {
        for (int i = 0; i < NST; i++) mbar_init(&sm.full[i], 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (!a.prefetch) grid_dep_wait();
    const int p_tok = a.pos[b];
    const CcRange r = cc_range(p_tok, a.cap, a.n_splits, s);
    const int n_sub = r.t1 - r.t0;
    const size_t row0 = ((size_t)b * a.nkv + kvh) * a.cap;  // cache row of position 0
    // the sub-tile holding the token's slot: before the predecessor is done (prefetch) it
    // may still be written by it (two-kernel decode), so it is requested after the wait
    const int tok_sub = p_tok / SUB - r.t0;
    auto issue = [&](int i) {  // sub-tile i of the range into stage i % NST (thread 0)
        const int st = i % NST;
        const int base = (r.t0 + i) * SUB;
        const int rows = min(SUB, r.n_pos - base);
        const uint32_t bytes = (uint32_t)rows * HD * 2;
        mbar_arrive_expect_tx(&sm.full[st], 2 * bytes);
        bulk_g2s(sm.k[st], a.kc + (row0 + base) * HD, bytes, &sm.full[st]);
        bulk_g2s(sm.v[st], a.vc + (row0 + base) * HD, bytes, &sm.full[st]);
    };
    int issued = 0;  // sub-tiles requested (thread 0)
    if (tid == 0 && a.prefetch)
        for (; issued < n_sub && issued < NST && (FUSED || issued != tok_sub); issued++) issue(issued);
    if (a.prefetch) grid_dep_wait();
    if (tid == 0) {
        for (; issued < n_sub && issued < NST; issued++) issue(issued);
        grid_dep_launch();  // the combine may be scheduled once every CTA is past here
    }
    __syncwarp();

    // ---- q of the group (and, fused, the new K/V row) ------------------------------
    const size_t qrow = ((size_t)b * a.nq + kvh * G) * HD;
    const bool app = FUSED && p_tok >= r.t0 * SUB && p_tok < r.t1 * SUB && p_tok < a.cap;
    if constexpr (FUSED) {
        // rows 0..G-1: q heads of the group, G: k, G+1: v (RMSNorm + RoPE as gqa_append_k)
        const int d = tid;
        const size_t kvi = ((size_t)b * a.nkv + kvh) * HD + d;
        float x[G + 1];
#pragma unroll
        for (int h = 0; h < G; h++) x[h] = act_ld<ACT_BF16>(a.q_in, qrow + (size_t)h * HD + d);
        x[G] = app ? act_ld<ACT_BF16>(a.k_in, kvi) : 0.0f;
        const float xv = app ? act_ld<ACT_BF16>(a.v_in, kvi) : 0.0f;
#pragma unroll
        for (int h = 0; h <= G; h++) {
            const double ss = warp_sum_d((double)x[h] * (double)x[h]);
            if (lane == 0) sm.red[h][warp] = ss;
        }
        __syncthreads();
        const float wq = a.one_p ? __fadd_rn(a.qw[d], 1.0f) : a.qw[d];
        const float wk = a.one_p ? __fadd_rn(a.kw[d], 1.0f) : a.kw[d];
#pragma unroll
        for (int h = 0; h <= G; h++) {
            double t = 0.0;
#pragma unroll
            for (int w = 0; w < CC_THREADS / 32; w++) t += sm.red[h][w];
            const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)(t / HD), a.eps)));
            sm.y[h][d] = __fmul_rn(__fmul_rn(x[h], rs), h < G ? wq : wk);
        }
        __syncthreads();
        const int half = a.rope_dim / 2;
        const bool p_ok = p_tok >= 0 && p_tok < a.rope_len;
        if (a.rope_dim > 0 && !p_ok && tid == 0) dev_flag(a.status, VX_DEV_BAD_ARG);
        const float *rr = p_ok && a.rope_dim > 0 ? a.rope + (size_t)p_tok * a.rope_dim : nullptr;
        float ro[G + 1];  // rotated rows, held until every thread has read y (q aliases it)
#pragma unroll
        for (int h = 0; h <= G; h++) {
            float o = sm.y[h][d];
            if (rr && d < a.rope_dim) {
                const int i = d < half ? d : d - half;
                const float c = rr[i], sn = rr[half + i];
                const float x0 = sm.y[h][i], x1 = sm.y[h][i + half];
                o = d < half ? __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn))
                             : __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
            }
            ro[h] = o;
        }
        __syncthreads();
#pragma unroll
        for (int h = 0; h < G; h++) sm.q[h][d >> 5][q_slot(d)] = ro[h];
        if (app) sm.kvrow[0][d] = f32_to_bf16(ro[G]);
        if (app) {
            sm.kvrow[1][d] = f32_to_bf16(xv);
            const size_t o = (row0 + p_tok) * HD + d;
            const_cast<uint16_t *>(a.kc)[o] = sm.kvrow[0][d];
            const_cast<uint16_t *>(a.vc)[o] = sm.kvrow[1][d];
        }
    } else {
#pragma unroll
        for (int h = 0; h < G; h++) sm.q[h][tid >> 5][q_slot(tid)] = a.q[qrow + (size_t)h * HD + tid];
    }
    __syncthreads();

    // ---- stream the range -------------------------------------------------------------
    float o[G];
    float m_run = -INFINITY, l_run = 0.0f;  // head `warp` (warps < G)
#pragma unroll
    for (int h = 0; h < G; h++) o[h] = 0.0f;
    const float scale = 1.0f / 16.0f;  // 1/sqrt(hd), exact
    const int pp = tid >> 3, part = tid & 7;
    bool ok = true;
    for (int i = 0; i < n_sub; i++) {
        const int st = i % NST;
        if (!cc_wait_all(&sm.full[st], (i / NST) & 1, sm, a.status)) { ok = false; break; }
        const int base = (r.t0 + i) * SUB;
        const int rows = min(SUB, r.n_pos - base);
        if (app && p_tok >= base && p_tok < base + SUB) {  // the new row, as stored above
            reinterpret_cast<uint16_t *>(sm.k[st])[(p_tok - base) * HD + tid] = sm.kvrow[0][tid];
            reinterpret_cast<uint16_t *>(sm.v[st])[(p_tok - base) * HD + tid] = sm.kvrow[1][tid];
            __syncthreads();
        }
        // scores: thread (position pp, part) sums 32 dims of every head; the parts visit
        // their four 16-byte chunks in a rotated order so a quarter warp reads all banks
        float acc[G];
#pragma unroll
        for (int h = 0; h < G; h++) acc[h] = 0.0f;
        if (pp < rows) {
            const uint8_t *krow = sm.k[st] + pp * (HD * 2) + part * 64;
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int c = (u + (part >> 1)) & 3;
                const uint4 kv = *reinterpret_cast<const uint4 *>(krow + c * 16);
                const uint32_t w4[4] = {kv.x, kv.y, kv.z, kv.w};
                float kf[8];
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    kf[2 * e] = __uint_as_float(w4[e] << 16);
                    kf[2 * e + 1] = __uint_as_float(w4[e] & 0xffff0000u);
                }
#pragma unroll
                for (int h = 0; h < G; h++) {
                    const float4 q0 = *reinterpret_cast<const float4 *>(&sm.q[h][part][u * 8]);
                    const float4 q1 = *reinterpret_cast<const float4 *>(&sm.q[h][part][u * 8 + 4]);
                    acc[h] = fmaf(q0.x, kf[0], acc[h]);
                    acc[h] = fmaf(q0.y, kf[1], acc[h]);
                    acc[h] = fmaf(q0.z, kf[2], acc[h]);
                    acc[h] = fmaf(q0.w, kf[3], acc[h]);
                    acc[h] = fmaf(q1.x, kf[4], acc[h]);
                    acc[h] = fmaf(q1.y, kf[5], acc[h]);
                    acc[h] = fmaf(q1.z, kf[6], acc[h]);
                    acc[h] = fmaf(q1.w, kf[7], acc[h]);
                }
            }
        }
#pragma unroll
        for (int h = 0; h < G; h++) {
            acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], 4);
            acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], 2);
            acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], 1);
        }
        if (part == 0) {
#pragma unroll
            for (int h = 0; h < G; h++) sm.sc[h][pp] = pp < rows ? acc[h] * scale : -INFINITY;
        }
        __syncthreads();
        // softmax statistics: warp h owns head h, lane = position
        if (warp < G) {
            const float sv = sm.sc[warp][lane];
            const float m_new = fmaxf(m_run, warp_max(sv));  // finite: rows >= 1
            const float corr = expf(m_run - m_new);          // 0 on the first stage
            const float pe = expf(sv - m_new);               // 0 for masked positions
            l_run = fmaf(l_run, corr, warp_sum(pe));
            m_run = m_new;
            sm.p[lane][warp] = pe;
            if (lane == 0) sm.corr[warp] = corr;
        }
        __syncthreads();
        // o[h][d] = corr o[h][d] + sum_p p[h][p] v[p][d], thread = dimension d
        {
            const uint16_t *vcol = reinterpret_cast<const uint16_t *>(sm.v[st]) + tid;
#pragma unroll
            for (int h = 0; h < G; h++) o[h] *= sm.corr[h];
#pragma unroll 2
            for (int p = 0; p < rows; p++) {
                const float vv = bf16_to_f32(vcol[p * HD]);
                const float4 pa = *reinterpret_cast<const float4 *>(&sm.p[p][0]);
                const float4 pb = *reinterpret_cast<const float4 *>(&sm.p[p][4]);
                const float pr[8] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
#pragma unroll
                for (int h = 0; h < G; h++) o[h] = fmaf(pr[h], vv, o[h]);
            }
        }
        __syncthreads();  // stage, scores and probabilities free again
        if (tid == 0 && i + NST < n_sub) issue(issued++);
        __syncwarp();
    }
    if (!ok) {
        // let every issued copy land before the CTA exits (bounded)
        if (tid == 0)
            for (int j = max(0, issued - NST); j < issued; j++) {
                const uint32_t addr = smem_u32(&sm.full[j % NST]);
                for (int it = 0; it < (1 << 20); it++) {
                    uint32_t done;
                    asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                                 : "=r"(done) : "r"(addr), "r"((uint32_t)((j / NST) & 1)) : "memory");
                    if (done) break;
                }
            }
        return;
    }
    if (warp < G && lane == 0) {
        sm.m[warp] = m_run;
        sm.l[warp] = l_run;
    }
    __syncthreads();
    const int d = tid;
    if (a.out) {  // one split: the gated output (the combine's arithmetic)
#pragma unroll
        for (int h = 0; h < G; h++) {
            const float L = sm.l[h];
            const float O = L > 0.0f ? o[h] / L : 0.0f;
            const float att = L > 0.0f ? (L * O) / L : 0.0f;
            const size_t oi = qrow + (size_t)h * HD + d;
            if (a.gate) {
                const float g = act_ld<ACT_BF16>(a.gate, oi);
                act_st<OUT_BF16>(a.out, oi, att * (1.0f / (1.0f + expf(-g))));
            } else {
                act_st<OUT_BF16>(a.out, oi, att);
            }
        }
    } else {
        const size_t rec = (size_t)a.B * a.nq * (HD + 2);
        float *pr = a.parts + (size_t)s * rec;
#pragma unroll
        for (int h = 0; h < G; h++) {
            const float L = sm.l[h];
            pr[qrow + (size_t)h * HD + d] = L > 0.0f ? o[h] / L : 0.0f;
        }
        if (d < G) {
            float *ml = pr + (size_t)a.B * a.nq * HD + ((size_t)b * a.nq + kvh * G + d) * 2;
            ml[0] = sm.l[d] > 0.0f ? sm.m[d] : -INFINITY;
            ml[1] = sm.l[d];
        }
    }
}

size_t cc_smem_bytes() { return sizeof(CcSmem) + 128; }

}  // namespace

// Split count of the CUDA-core kernel: two CTAs per SM run at once; a launch takes about
// waves x (sub-tiles per split + 3 of per-CTA prologue and epilogue), plus 3 for the
// combine pass when there is more than one split. Ties: fewer splits.
int cc_auto_splits(int B, int nkv, int max_ctx) {
    const long long blocks = (long long)B * nkv, slots = 2LL * num_sms();
    const int subs = (max_ctx + SUB - 1) / SUB;
    if (subs <= 1) return 1;
    int best = 1;
    long long best_t = -1;
    const int n_max = subs < 1024 ? subs : 1024;
    for (int n = 1; n <= n_max; n++) {
        const int per = (subs + n - 1) / n;
        if ((subs + per - 1) / per < n) continue;  // same as a smaller n
        const long long waves = (blocks * n + slots - 1) / slots;
        const long long t = waves * (per + 3) + (n > 1 ? 3 : 0);
        if (best_t < 0 || t < best_t) { best_t = t; best = n; }
    }
    return best;
}

// The CUDA-core decode: split kernel (+ combine when n_splits > 1). q_in != NULL selects
// the fused prologue (q from raw activations, the new K/V row appended). Returns the
// number of kernels launched, or -1.
int launch_decode_cc(const void *kc, const void *vc, const float *q, const int *pos,
                     float *parts, int cap, int B, int nq, int nkv, int n_splits,
                     const void *gate, void *out, int flags, const void *q_in, const void *k_in,
                     const void *v_in, const float *qw, const float *kw, const float *rope,
                     int rope_len, int rope_dim, float eps, cudaStream_t st, char *err,
                     size_t errlen) {
    const bool fused = q_in != nullptr;
    if (((uintptr_t)kc & 15) || ((uintptr_t)vc & 15))
        return fail(err, errlen, "vx27_gqa: the caches must be 16-byte aligned");
    if (fused && (rope_dim < 0 || rope_dim > HD || (rope_dim & 1)))
        return fail(err, errlen, "vx27_gqa_decode_fused: rope_dim=%d", rope_dim);
    CcArgs a{};
    a.kc = (const uint16_t *)kc;
    a.vc = (const uint16_t *)vc;
    a.q = q;
    a.pos = pos;
    a.parts = parts;
    a.gate = n_splits == 1 ? gate : nullptr;
    a.out = n_splits == 1 ? out : nullptr;
    a.cap = cap;
    a.B = B;
    a.nq = nq;
    a.nkv = nkv;
    a.n_splits = n_splits;
    a.prefetch = (flags & VX27_F_PREFETCH_KV) ? 1 : 0;
    a.q_in = q_in;
    a.k_in = k_in;
    a.v_in = v_in;
    a.qw = qw;
    a.kw = kw;
    a.rope = rope;
    a.rope_len = rope_len;
    a.rope_dim = rope_dim;
    a.one_p = (flags & VX27_F_NORM_1P) ? 1 : 0;
    a.eps = eps;
    a.status = dev_status();
    const size_t smem = cc_smem_bytes();
    const dim3 grid(n_splits, nkv, B);
    const bool ab = flags & VX27_F_ACT_BF16, ob = flags & VX27_F_OUT_BF16;
#define VX_CC(GG, FF, AA, OO)                                                                 \
    {                                                                                         \
        if (ensure_smem_attr((const void *)gqa_split_cc<GG, FF, AA, OO>, smem, err, errlen))  \
            return -1;                                                                        \
        VX_CK(launch_pdl(gqa_split_cc<GG, FF, AA, OO>, grid, dim3(CC_THREADS), smem, st, a)); \
    }
#define VX_CCF(GG)                                                                            \
    case GG:                                                                                  \
        if (fused) {                                                                          \
            if (ab && ob) VX_CC(GG, true, true, true)                                         \
            else if (ab) VX_CC(GG, true, true, false)                                         \
            else if (ob) VX_CC(GG, true, false, true)                                         \
            else VX_CC(GG, true, false, false)                                                \
        } else {                                                                              \
            if (ab && ob) VX_CC(GG, false, true, true)                                        \
            else if (ab) VX_CC(GG, false, true, false)                                        \
            else if (ob) VX_CC(GG, false, false, true)                                        \
            else VX_CC(GG, false, false, false)                                               \
        }                                                                                     \
        break;
    switch (nq / nkv) {
        VX_CCF(1) VX_CCF(2) VX_CCF(4) VX_CCF(6) VX_CCF(8)
        default:
            return fail(err, errlen, "vx27_gqa: group size %d (nq/nkv) unsupported", nq / nkv);
    }
#undef VX_CCF
#undef VX_CC
    VX_CK(cudaGetLastError());
    if (n_splits == 1) return 1;
    // the combine waits for this kernel (programmatic dependent launch)
    if (launch_gqa_combine(parts, n_splits, gate, out, B, nq, flags, st, err, errlen, true))
        return -1;
    return 2;
}

}  // namespace vx27
