// K2: gated GQA decode over a BF16 KV cache.
//   gqa_append_k   per-token prologue: QK RMSNorm, partial RoPE, bf16 K/V store
//                  (src/vx27_qfwd.c:339-346)
//   split kernel   tensor-core split-KV flash decoding (gqa_tc.cu), one CTA per
//                  (sequence, KV head, split) serving the nq/nkv Q heads of the group;
//                  writes one partial record (m, l, o) per split
//   gqa_combine32_k / gqa_combine_k
//                  log-sum-exp merge of the partial records + sigmoid output gate
//                  (src/vx27_qfwd.c:347-371): up to 32 records in one round trip to L2,
//                  more in blocks, the same bits either way
#include <math.h>
#include "common.cuh"
#include "../../include/vx27_gqa.h"

namespace vx27 {

// gqa_tc.cu: the tensor-core split-KV kernel (persistent, one CTA per SM over the
// (sequence, KV head, split) items). With out != NULL and one split it writes the gated
// attention output itself (gate/out dtypes from VX27_F_ACT_BF16 / VX27_F_OUT_BF16).
int launch_split_tc(const void *kc, const void *vc, const float *q, const int *pos, float *parts,
                    int cap, int B, int nq, int nkv, int n_splits, int p_begin, int p_end,
                    cudaStream_t st, char *err, size_t errlen, const void *gate = nullptr,
                    void *out = nullptr, int flags = 0);
int launch_split_tc_fused(const void *q_in, const void *k_in, const void *v_in,
                          const float *qw, const float *kw, const float *rope, int rope_len,
                          int rope_dim, float eps, void *kc, void *vc, int cap, const int *pos,
                          float *parts, int B, int nq, int nkv, int n_splits, const void *gate,
                          void *out, int flags, cudaStream_t st, char *err, size_t errlen);

// gqa_cc.cu: the CUDA-core split-KV kernel for small batches (+ its combine); q_in != NULL
// selects its fused prologue. Returns the kernels launched or -1.
int launch_decode_cc(const void *kc, const void *vc, const float *q, const int *pos,
                     float *parts, int cap, int B, int nq, int nkv, int n_splits,
                     const void *gate, void *out, int flags, const void *q_in, const void *k_in,
                     const void *v_in, const float *qw, const float *kw, const float *rope,
                     int rope_len, int rope_dim, float eps, cudaStream_t st, char *err,
                     size_t errlen);
int cc_auto_splits(int B, int nkv, int max_ctx);

namespace {

constexpr int HD = 256;
constexpr int TILE = 128;  // split boundaries fall on multiples of TILE positions

// ---- append -------------------------------------------------------------------
template <bool ACT_BF16, bool ONE_P>
__global__ void __launch_bounds__(HD)
gqa_append_k(const void *__restrict__ q_in, const void *__restrict__ k_in,
             const void *__restrict__ v_in, const float *__restrict__ qw,
             const float *__restrict__ kw, const float *__restrict__ rope, int rope_len,
             const int *__restrict__ pos, int slot_base, uint16_t *__restrict__ kc,
             uint16_t *__restrict__ vc, int cap, float *__restrict__ q_out, int nq, int nkv,
             int rope_dim, float eps, int w_group, uint32_t *status) {
    grid_dep_wait();  // inputs and positions come from the kernels before this one
    if (threadIdx.x == 0) grid_dep_launch();
    const int head = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
    const bool is_q = head < nq;
    const int h = is_q ? head : head - nq;
    const size_t row = is_q ? ((size_t)b * nq + h) * HD : ((size_t)b * nkv + h) * HD;
    const float x = act_ld<ACT_BF16>(is_q ? q_in : k_in, row + d);
    __shared__ double red[HD / 32];
    __shared__ float r_s;
    __shared__ float y_s[HD];
    double ss = warp_sum_d((double)x * (double)x);
    if ((d & 31) == 0) red[d >> 5] = ss;
    __syncthreads();
    if (d == 0) {
        double t = 0.0;
        for (int w = 0; w < HD / 32; w++) t += red[w];
        r_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)(t / HD), eps)));
    }
    __syncthreads();
    const size_t wrow = (size_t)(b / w_group) * HD;  // norm weights of this sequence's group
    float w = is_q ? qw[wrow + d] : kw[wrow + d];
    if (ONE_P) w = __fadd_rn(w, 1.0f);
    const float y = __fmul_rn(__fmul_rn(x, r_s), w);
    y_s[d] = y;
    __syncthreads();
    const int p = pos[b];
    const int half = rope_dim / 2;
    float out = y;
    if (d < rope_dim) {
        if (p < 0 || p >= rope_len) {
            if (d == 0) dev_flag(status, VX_DEV_BAD_ARG);
        } else {
            const float *rr = rope + (size_t)p * rope_dim;
            const int i = d < half ? d : d - half;
            const float c = rr[i], s = rr[half + i];
            const float x0 = y_s[i], x1 = y_s[i + half];
            out = d < half ? __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s))
                           : __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
        }
    }
    if (is_q) {
        q_out[row + d] = out;
    } else if (kc) {
        const int slot = p - slot_base;
        if (slot >= 0 && slot < cap) {
            const size_t o = (((size_t)b * nkv + h) * cap + slot) * HD + d;
            kc[o] = f32_to_bf16(out);
            vc[o] = f32_to_bf16(act_ld<ACT_BF16>(v_in, row + d));
        }
    }
}

// ---- combine ------------------------------------------------------------------------
// One CTA per (Q head, sequence) merges the split records: m* = max m_i,
// l* = sum l_i e^{m_i - m*}, o = sum o_i l_i e^{m_i - m*} / l* (records with l_i = 0 skipped).
// The records' (m, l) are read in parallel and their weights staged in shared memory in
// blocks of CMB_R, then each thread (one output dim) sums its column with independent
// loads; the sums run in record order, so the result does not depend on the block size.
constexpr int CMB_R = 1024;

struct CmbWeights {
    float w[CMB_R];
    float red[HD / 32];
    float M;
};

// Max of the valid records' m over all n_parts (every thread gets it).
__device__ __forceinline__ float cmb_max(const float *__restrict__ parts, int n_parts, size_t rec,
                                         size_t ml_off, CmbWeights &cw) {
    const int d = threadIdx.x;
    float M = -INFINITY;
    for (int r = d; r < n_parts; r += HD) {
        const float2 ml = *reinterpret_cast<const float2 *>(parts + (size_t)r * rec + ml_off);
        if (ml.y > 0.0f) M = fmaxf(M, ml.x);
    }
    M = warp_max(M);
    if ((d & 31) == 0) cw.red[d >> 5] = M;
    __syncthreads();
    if (d == 0) {
        float t = cw.red[0];
        for (int w = 1; w < HD / 32; w++) t = fmaxf(t, cw.red[w]);
        cw.M = t;
    }
    __syncthreads();
    return cw.M;
}

// (L, O) for output dim threadIdx.x: L = sum w_r, O = sum w_r o_r[d] in record order.
__device__ __forceinline__ void cmb_sum(const float *__restrict__ parts, int n_parts, size_t rec,
                                        size_t ml_off, size_t o_off, float M, CmbWeights &cw,
                                        float &L, float &O) {
    const int d = threadIdx.x;
    L = 0.0f;
    O = 0.0f;
    if (M == -INFINITY) return;
    for (int r0 = 0; r0 < n_parts; r0 += CMB_R) {
        const int n = min(CMB_R, n_parts - r0);
        __syncthreads();
        for (int r = d; r < n; r += HD) {
            const float2 ml = *reinterpret_cast<const float2 *>(parts + (size_t)(r0 + r) * rec + ml_off);
            cw.w[r] = ml.y > 0.0f ? ml.y * expf(ml.x - M) : 0.0f;
        }
        __syncthreads();
        const float *col = parts + (size_t)r0 * rec + o_off + d;
        int r = 0;
        for (; r + 8 <= n; r += 8) {
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; u++) v[u] = col[(size_t)(r + u) * rec];
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const float w = cw.w[r + u];
                if (w != 0.0f) {  // skipped records (w = 0) add nothing
                    L += w;
                    O = fmaf(w, v[u], O);
                }
            }
        }
        for (; r < n; r++) {
            const float w = cw.w[r];
            if (w != 0.0f) {
                L += w;
                O = fmaf(w, col[(size_t)r * rec], O);
            }
        }
    }
}

template <bool ACT_BF16, bool OUT_BF16, bool PDL>
__global__ void __launch_bounds__(HD)
gqa_combine_k(const float *__restrict__ parts, int n_parts, const void *__restrict__ gate,
              void *__restrict__ out, int B, int nq, size_t rec) {
    if constexpr (PDL) grid_dep_wait();
    __shared__ CmbWeights cw;
    const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
    const size_t hq = (size_t)b * nq + h;
    const size_t ml_off = (size_t)B * nq * HD + hq * 2;
    const float M = cmb_max(parts, n_parts, rec, ml_off, cw);
    float L, O;
    cmb_sum(parts, n_parts, rec, ml_off, hq * HD, M, cw, L, O);
    const float att = L > 0.0f ? O / L : 0.0f;
    if (gate) {
        const float g = act_ld<ACT_BF16>(gate, hq * HD + d);
        act_st<OUT_BF16>(out, hq * HD + d, att * (1.0f / (1.0f + expf(-g))));
    } else {  // no output gate (the MTP drafter's use_gate = 0, src/vx27_mtp.c:249)
        act_st<OUT_BF16>(out, hq * HD + d, att);
    }
}

// The combine for at most CMB_FAST records, with one round trip to L2: each thread
// requests its column of every record, and each warp the records' (m, l) (lane r: record
// r) and the gate, all at once. Each warp then forms the max and the weights itself, so
// no shared memory or CTA barrier is on the path. Same arithmetic and record order as
// gqa_combine_k, hence the same bits.
constexpr int CMB_FAST = 32;

template <bool ACT_BF16, bool OUT_BF16, bool PDL>
__global__ void __launch_bounds__(HD)
gqa_combine32_k(const float *__restrict__ parts, int n_parts, const void *__restrict__ gate,
                void *__restrict__ out, int B, int nq, size_t rec) {
    if constexpr (PDL) grid_dep_wait();
    const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x, lane = d & 31;
    const size_t hq = (size_t)b * nq + h;
    const float *col = parts + hq * HD + d;
    const float *mlp = parts + (size_t)B * nq * HD + hq * 2;
    float v[CMB_FAST];
#pragma unroll
    for (int r = 0; r < CMB_FAST; r++) v[r] = r < n_parts ? __ldcg(col + (size_t)r * rec) : 0.0f;
    const float2 ml = lane < n_parts
                          ? __ldcg(reinterpret_cast<const float2 *>(mlp + (size_t)lane * rec))
                          : make_float2(-INFINITY, 0.0f);
    const float g = gate ? act_ld<ACT_BF16>(gate, hq * HD + d) : 0.0f;
    const float M = warp_max(ml.y > 0.0f ? ml.x : -INFINITY);
    const float w = ml.y > 0.0f ? ml.y * expf(ml.x - M) : 0.0f;
    float L = 0.0f, O = 0.0f;
#pragma unroll
    for (int r = 0; r < CMB_FAST; r++) {
        const float wr = __shfl_sync(0xffffffffu, w, r);
        if (wr != 0.0f) {  // skipped records (w = 0) add nothing
            L += wr;
            O = fmaf(wr, v[r], O);
        }
    }
    const float att = L > 0.0f ? O / L : 0.0f;
    if (gate)
        act_st<OUT_BF16>(out, hq * HD + d, att * (1.0f / (1.0f + expf(-g))));
    else
        act_st<OUT_BF16>(out, hq * HD + d, att);
}

// Merges n_parts partial records into one partial record (same layout), for a range
// that was split across CTAs: m = max m_i, l = sum l_i e^{m_i - m}, o = sum o_i l_i
// e^{m_i - m} / l.
__global__ void __launch_bounds__(HD)
gqa_merge_k(const float *__restrict__ parts, int n_parts, float *__restrict__ rec_out, int B,
            int nq) {
    __shared__ CmbWeights cw;
    const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
    const size_t rec = (size_t)B * nq * (HD + 2);
    const size_t hq = (size_t)b * nq + h;
    const size_t ml_off = (size_t)B * nq * HD + hq * 2;
    const float M = cmb_max(parts, n_parts, rec, ml_off, cw);
    float L, O;
    cmb_sum(parts, n_parts, rec, ml_off, hq * HD, M, cw, L, O);
    rec_out[hq * HD + d] = L > 0.0f ? O / L : 0.0f;
    if (d == 0) {
        float *ml = rec_out + (size_t)B * nq * HD + hq * 2;
        ml[0] = L > 0.0f ? M : -INFINITY;
        ml[1] = L;
    }
}

// Split count for B*nkv (sequence, KV head) blocks over max_ctx positions. The split
// kernel is persistent (one CTA per SM, items streamed back to back), so a launch takes
// about ceil(items / SMs) x (tiles per split + 1/4 tile of per-item epilogue) plus ~2
// tiles of pipeline fill and drain; pick the count that minimises that estimate (ties:
// fewer splits, i.e. fewer partial records to merge).
int auto_splits(int B, int nkv, int max_ctx) {
    const long long blocks = (long long)B * nkv;
    const long long sms = num_sms();
    const int tiles = (max_ctx + TILE - 1) / TILE;
    if (tiles <= 1 || blocks >= 8 * sms) return 1;
    int best = 1;
    long long best_t = -1;
    const int n_max = tiles < 512 ? tiles : 512;
    for (int n = 1; n <= n_max; n++) {
        const int per = (tiles + n - 1) / n;          // tiles per split
        const int active = (tiles + per - 1) / per;   // splits that get work
        if (active < n) continue;                     // same as a smaller n
        const long long waves = (blocks * n + sms - 1) / sms;
        const long long t = waves * (4LL * per + 1) + 8;  // quarter tiles
        if (best_t < 0 || t < best_t) { best_t = t; best = n; }
    }
    return best;
}

// Which decode kernel a call uses: the tensor-core kernel unless the flags ask for the
// CUDA-core one. Measured on a B200 (graph-replayed, events): the CUDA-core kernel is the
// slower at every shape tried, 1.5x at one sequence of 8192 positions and 2.8x at 256
// sequences of 4096 (its fp32 FMA work per cache byte, not HBM, bounds it).
bool use_cc(int B, int nkv, int flags) {
    (void)B;
    (void)nkv;
    return (flags & VX27_F_DECODE_CC) && !(flags & VX27_F_DECODE_TC);
}

// The split count a decode call runs with: n_splits when given, else the chosen kernel's
// own count capped by the workspace (fit records).
int plan_splits(int B, int nkv, int cap, int n_splits, int fit, bool cc) {
    if (n_splits > 0) return n_splits;
    n_splits = cc ? cc_auto_splits(B, nkv, cap) : auto_splits(B, nkv, cap);
    return n_splits > fit ? fit : n_splits;
}

int launch_split(const float *q, const void *kc, const void *vc, int cap, const int *pos,
                 float *parts, int B, int nq, int nkv, int n_splits, int p_begin, int p_end,
                 cudaStream_t st, char *err, size_t errlen) {
    return launch_split_tc(kc, vc, q, pos, parts, cap, B, nq, nkv, n_splits, p_begin, p_end, st,
                           err, errlen);
}

// pdl: launched with programmatic dependent launch (the kernel waits for its predecessor,
// so its launch overlaps the split kernel's tail)
int launch_combine(const float *parts, int n_parts, const void *gate, void *out, int B, int nq,
                   int flags, cudaStream_t st, char *err, size_t errlen, size_t stride = 0,
                   bool pdl = false) {
    const dim3 grid(nq, B);
    const bool a = flags & VX27_F_ACT_BF16, o = flags & VX27_F_OUT_BF16;
    const size_t rec = stride ? stride : (size_t)B * nq * (HD + 2);
#define VX_CMB1(K_, A_, O_)                                                                \
    if (pdl)                                                                               \
        VX_CK(launch_pdl(K_<A_, O_, true>, grid, dim3(HD), 0, st, parts, n_parts, gate, out, \
                         B, nq, rec));                                                     \
    else                                                                                   \
        K_<A_, O_, false><<<grid, HD, 0, st>>>(parts, n_parts, gate, out, B, nq, rec);
#define VX_CMB(A_, O_)                                                                     \
    if (n_parts <= CMB_FAST) { VX_CMB1(gqa_combine32_k, A_, O_) }                          \
    else { VX_CMB1(gqa_combine_k, A_, O_) }
    if (a && o) { VX_CMB(true, true) }
    else if (a) { VX_CMB(true, false) }
    else if (o) { VX_CMB(false, true) }
    else { VX_CMB(false, false) }
#undef VX_CMB
#undef VX_CMB1
    VX_CK(cudaGetLastError());
    return 0;
}

int check_shape(const char *fn, int B, int nq, int nkv, int hd, char *err, size_t errlen) {
    if (hd != HD) return fail(err, errlen, "%s: hd=%d unsupported (256 only)", fn, hd);
    if (B <= 0 || B > 65535 || nq <= 0 || nkv <= 0 || nkv > 65535 || nq % nkv)
        return fail(err, errlen, "%s: bad shape B=%d nq=%d nkv=%d", fn, B, nq, nkv);
    return 0;
}

}  // namespace

// The decode's split-count choice and its launches after the argument checks, for
// vx27_gqa_decode_batch and the entry point without a workspace (gqa_noalloc.cu): the
// kernel by use_cc, n_splits records at parts. Allocates nothing.
int gqa_plan_splits(int B, int nkv, int cap, int n_splits, int fit, int flags) {
    return plan_splits(B, nkv, cap, n_splits, fit, use_cc(B, nkv, flags));
}

int gqa_decode_dispatch(const float *q, const void *gate, const void *k_cache,
                        const void *v_cache, int cap, const int *pos, void *out, float *parts,
                        int B, int nq, int nkv, int n_splits, int flags, cudaStream_t st,
                        char *err, size_t errlen) {
    if (use_cc(B, nkv, flags))
        return launch_decode_cc(k_cache, v_cache, q, pos, parts, cap, B, nq, nkv, n_splits, gate,
                                out, flags, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                                0, 0, 0.0f, st, err, errlen) < 0 ? -1 : 0;
    if (n_splits == 1)  // the split kernel applies the gate and writes out; no combine pass
        return launch_split_tc(k_cache, v_cache, q, pos, parts, cap, B, nq, nkv, 1, 0, -1, st,
                               err, errlen, gate, out, flags);
    if (launch_split(q, k_cache, v_cache, cap, pos, parts, B, nq, nkv, n_splits, 0, -1, st, err,
                     errlen))
        return -1;
    return launch_combine(parts, n_splits, gate, out, B, nq, flags, st, err, errlen, 0, true);
}

int launch_gqa_combine(const float *parts, int n_parts, const void *gate, void *out, int B,
                       int nq, int flags, cudaStream_t st, char *err, size_t errlen, bool pdl) {
    return launch_combine(parts, n_parts, gate, out, B, nq, flags, st, err, errlen, 0, pdl);
}

}  // namespace vx27

using namespace vx27;

extern "C" {

int vx27_gqa_append(const void *q_in, const void *k_in, const void *v_in,
                    const float *q_norm_w, const float *k_norm_w, const float *rope_table,
                    int rope_table_len, const int *pos, int slot_base, void *k_cache,
                    void *v_cache, int cap, float *q_out, int B, int nq, int nkv, int hd,
                    int rope_dim, float eps, int flags, void *stream, char *err,
                    size_t errlen) {
    return vx27_gqa_append_grouped(q_in, k_in, v_in, q_norm_w, k_norm_w, B, rope_table,
                                   rope_table_len, pos, slot_base, k_cache, v_cache, cap, q_out,
                                   B, nq, nkv, hd, rope_dim, eps, flags, stream, err, errlen);
}

int vx27_gqa_append_grouped(const void *q_in, const void *k_in, const void *v_in,
                            const float *q_norm_w, const float *k_norm_w, int seqs_per_weight,
                            const float *rope_table, int rope_table_len, const int *pos,
                            int slot_base, void *k_cache, void *v_cache, int cap, float *q_out,
                            int B, int nq, int nkv, int hd, int rope_dim, float eps, int flags,
                            void *stream, char *err, size_t errlen) {
    if (check_shape("vx27_gqa_append", B, nq, nkv, hd, err, errlen)) return -1;
    if (seqs_per_weight <= 0 || B % seqs_per_weight)
        return fail(err, errlen, "vx27_gqa_append: %d sequences per weight row does not divide B=%d",
                    seqs_per_weight, B);
    if (rope_dim < 0 || rope_dim > hd || (rope_dim & 1))
        return fail(err, errlen, "vx27_gqa_append: rope_dim=%d", rope_dim);
    if (!q_in || !k_in || !v_in || !q_norm_w || !k_norm_w || !pos || !q_out ||
        (rope_dim && !rope_table))
        return fail(err, errlen, "vx27_gqa_append: null pointer argument");
    if ((k_cache == nullptr) != (v_cache == nullptr))
        return fail(err, errlen, "vx27_gqa_append: k_cache and v_cache must both be set or both NULL");
    const dim3 grid(nq + nkv, B);
    cudaStream_t st = (cudaStream_t)stream;
    const bool a = flags & VX27_F_ACT_BF16, one = flags & VX27_F_NORM_1P;
#define VX_A(A_, O_)                                                                    \
    VX_CK(launch_pdl(gqa_append_k<A_, O_>, grid, dim3(HD), 0, st, q_in, k_in, v_in, q_norm_w, \
                     k_norm_w, rope_table, rope_table_len, pos, slot_base,                 \
                     (uint16_t *)k_cache, (uint16_t *)v_cache, cap, q_out, nq, nkv, rope_dim, \
                     eps, seqs_per_weight, dev_status()))
    if (a && one) VX_A(true, true);
    else if (a) VX_A(true, false);
    else if (one) VX_A(false, true);
    else VX_A(false, false);
#undef VX_A
    VX_CK(cudaGetLastError());
    return 0;
}

size_t vx27_gqa_decode_workspace_size(int B, int nq, int nkv, int hd, int max_ctx,
                                      int n_splits) {
    if (B <= 0 || nq <= 0 || nkv <= 0 || hd <= 0) return 0;
    if (n_splits <= 0) n_splits = auto_splits(B, nkv, max_ctx);
    return (size_t)n_splits * B * nq * (hd + 2) * sizeof(float);
}

int vx27_gqa_decode_plan(int B, int nq, int nkv, int hd, int cap, size_t workspace_bytes,
                         int n_splits, int flags, int *kernel, int *splits) {
    if (B <= 0 || nq <= 0 || nkv <= 0 || hd != HD || cap <= 0) return -1;
    const bool cc = use_cc(B, nkv, flags);
    const size_t rec = (size_t)B * nq * (hd + 2) * sizeof(float);
    const int n = plan_splits(B, nkv, cap, n_splits, (int)(workspace_bytes / rec), cc);
    if (n < 1) return -1;
    if (kernel) *kernel = cc ? 1 : 0;
    if (splits) *splits = n;
    return n == 1 ? 1 : 2;
}

int vx27_gqa_decode_batch(const float *q, const void *gate, const void *k_cache,
                          const void *v_cache, int cap, const int *pos, void *out,
                          void *workspace, size_t workspace_bytes, int B, int nq, int nkv,
                          int hd, int n_splits, int flags, void *stream, char *err,
                          size_t errlen) {
    if (check_shape("vx27_gqa_decode_batch", B, nq, nkv, hd, err, errlen)) return -1;
    if (!q || !k_cache || !v_cache || !pos || !out || !workspace || cap <= 0)
        return fail(err, errlen, "vx27_gqa_decode_batch: null pointer argument");
    const size_t rec = (size_t)B * nq * (hd + 2) * sizeof(float);
    const int fit = (int)(workspace_bytes / rec);
    n_splits = plan_splits(B, nkv, cap, n_splits, fit, use_cc(B, nkv, flags));
    if (n_splits < 1 || n_splits > fit || n_splits > 65535)
        return fail(err, errlen,
                    "vx27_gqa_decode_batch: workspace of %zu bytes holds %d splits, need %d",
                    workspace_bytes, fit, n_splits < 1 ? 1 : n_splits);
    return gqa_decode_dispatch(q, gate, k_cache, v_cache, cap, pos, out, (float *)workspace, B,
                               nq, nkv, n_splits, flags, (cudaStream_t)stream, err, errlen);
}

int vx27_gqa_decode_fused(const void *q_in, const void *k_in, const void *v_in,
                          const float *q_norm_w, const float *k_norm_w, const float *rope_table,
                          int rope_table_len, const void *gate, void *k_cache, void *v_cache,
                          int cap, const int *pos, void *out, void *workspace,
                          size_t workspace_bytes, int B, int nq, int nkv, int hd, int rope_dim,
                          float eps, int n_splits, int flags, void *stream, char *err,
                          size_t errlen) {
    if (check_shape("vx27_gqa_decode_fused", B, nq, nkv, hd, err, errlen)) return -1;
    if (!q_in || !k_in || !v_in || !q_norm_w || !k_norm_w || !k_cache || !v_cache || !pos ||
        !out || !workspace || cap <= 0 || (rope_dim && !rope_table))
        return fail(err, errlen, "vx27_gqa_decode_fused: null pointer argument");
    const size_t rec = (size_t)B * nq * (hd + 2) * sizeof(float);
    const int fit = (int)(workspace_bytes / rec);
    const bool cc = use_cc(B, nkv, flags);
    n_splits = plan_splits(B, nkv, cap, n_splits, fit, cc);
    if (n_splits < 1 || n_splits > fit || n_splits > 65535)
        return fail(err, errlen,
                    "vx27_gqa_decode_fused: workspace of %zu bytes holds %d splits, need %d",
                    workspace_bytes, fit, n_splits < 1 ? 1 : n_splits);
    cudaStream_t st = (cudaStream_t)stream;
    float *parts = (float *)workspace;
    if (cc)
        return launch_decode_cc(k_cache, v_cache, nullptr, pos, parts, cap, B, nq, nkv, n_splits,
                                gate, out, flags, q_in, k_in, v_in, q_norm_w, k_norm_w,
                                rope_table, rope_table_len, rope_dim, eps, st, err, errlen) < 0
                   ? -1 : 0;
    const bool direct = n_splits == 1;  // the split kernel applies the gate and writes out
    if (launch_split_tc_fused(q_in, k_in, v_in, q_norm_w, k_norm_w, rope_table, rope_table_len,
                              rope_dim, eps, k_cache, v_cache, cap, pos, parts, B, nq, nkv,
                              n_splits, direct ? gate : nullptr, direct ? out : nullptr, flags,
                              st, err, errlen))
        return -1;
    if (direct) return 0;
    return launch_combine(parts, n_splits, gate, out, B, nq, flags, st, err, errlen, 0, true);
}

size_t vx27_gqa_partial_workspace_size(int B, int nq, int nkv, int hd, int max_range) {
    if (B <= 0 || nq <= 0 || nkv <= 0 || hd <= 0) return 0;
    const int n = auto_splits(B, nkv, max_range);
    return n > 1 ? (size_t)n * B * nq * (hd + 2) * sizeof(float) : 0;
}

int vx27_gqa_partial(const float *q, const void *k_cache, const void *v_cache, int cap,
                     int p_begin, int p_end, float *part, int B, int nq, int nkv, int hd,
                     void *workspace, size_t workspace_bytes, void *stream, char *err,
                     size_t errlen) {
    if (check_shape("vx27_gqa_partial", B, nq, nkv, hd, err, errlen)) return -1;
    if (!q || !k_cache || !v_cache || !part)
        return fail(err, errlen, "vx27_gqa_partial: null pointer argument");
    if (p_begin < 0 || p_end < p_begin || p_end > cap)
        return fail(err, errlen, "vx27_gqa_partial: range [%d, %d) outside cache of %d", p_begin,
                    p_end, cap);
    cudaStream_t st = (cudaStream_t)stream;
    const size_t rec = (size_t)B * nq * (hd + 2) * sizeof(float);
    int n = auto_splits(B, nkv, p_end - p_begin);
    const int fit = workspace ? (int)(workspace_bytes / rec) : 0;
    if (n > fit) n = fit;
    if (n <= 1)  // one CTA per (sequence, KV head) writes the record directly
        return launch_split(q, k_cache, v_cache, cap, nullptr, part, B, nq, nkv, 1, p_begin,
                            p_end, st, err, errlen);
    float *sub = (float *)workspace;
    if (launch_split(q, k_cache, v_cache, cap, nullptr, sub, B, nq, nkv, n, p_begin, p_end, st,
                     err, errlen))
        return -1;
    gqa_merge_k<<<dim3(nq, B), HD, 0, st>>>(sub, n, part, B, nq);
    VX_CK(cudaGetLastError());
    return 0;
}

int vx27_gqa_combine(const float *parts, int n_parts, size_t part_stride, const void *gate,
                     void *out, int B, int nq, int hd, int flags, void *stream, char *err,
                     size_t errlen) {
    if (hd != HD) return fail(err, errlen, "vx27_gqa_combine: hd=%d unsupported (256 only)", hd);
    if (!parts || !out || n_parts < 1 || B <= 0 || nq <= 0)
        return fail(err, errlen, "vx27_gqa_combine: bad arguments");
    const size_t rec = (size_t)B * nq * (hd + 2);
    if (part_stride && part_stride < rec)
        return fail(err, errlen, "vx27_gqa_combine: part_stride %zu < record size %zu",
                    part_stride, rec);
    // each record's (m, l) pairs are read as 8-byte vectors
    if (((uintptr_t)parts & 7) || (part_stride & 1))
        return fail(err, errlen,
                    "vx27_gqa_combine: parts must be 8-byte aligned and part_stride even");
    return launch_combine(parts, n_parts, gate, out, B, nq, flags, (cudaStream_t)stream, err,
                          errlen, part_stride);
}

}  // extern "C"
