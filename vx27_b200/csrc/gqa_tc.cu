// K2 main loop on the 5th-generation tensor cores: split-KV flash decoding of work items
// (sequence, KV head, split), each serving the G = nq/nkv query heads of its group, by a
// persistent grid of one CTA per SM. A staging warp does the CTA's global loads and stores
// (q of the next item, gate values, the gated output or the partial record).
//
// Data flow per tile of 128 cache positions:
//   TMA (warp 0)   K and V tiles, bf16 [128 positions x 256 dims], fetched as 16 KB chunks
//                  of 64 dims with 128-byte swizzle into a 12-slot ring (192 KB)
//   MMA (warp 1)   S^T[128 x 16] = K[128 x 256] . Q^T[256 x 16]      (TMEM, fp32)
//                  O^T[256 x 16] = V^T[256 x 128] . P^T[128 x 16]    (TMEM, fp32, per tile)
//   softmax        warps 2-5, one thread per position (= TMEM lane): scaled scores, running
//                  max per head, p = 2^(x - m), P^T written to shared memory; then the
//                  previous tile's O^T is read back (one thread per head dimension) and
//                  folded into fp32 register accumulators with the max correction.
// The 16 MMA columns carry each query head twice: rows 0..G-1 hold the bf16-rounded q
// (and p), rows G..2G-1 the bf16 rounding residual, so q and p enter the tensor core with
// ~16 significant bits and the result is close to an fp32 dot product.
// Every mbarrier wait is bounded (~2 s); a timeout sets the device status word and makes
// all roles leave their loops.
#include <math.h>
#include "common.cuh"
#include "tc.cuh"

namespace vx27 {

constexpr int TC_TILE = 128;
constexpr int NSLOT = 12;
constexpr int SLOT_BYTES = 16384;      // 128 rows x 128 bytes
constexpr int TC_THREADS = 224;     // TMA, MMA, 4 softmax warps, staging warp
constexpr int HDIM = 256;
constexpr uint32_t TMEM_COLS = 128;    // S[2] at 0,16; O[2] (two halves) at 32..95

struct TcSmem {
    uint8_t ring[NSLOT][SLOT_BYTES];
    uint8_t q[2][4][2048];             // Q^T operand per item buffer: 4 chunks of [16 rows x 128 B]
    uint8_t p[2][2][2048];             // P^T operand per buffer: 2 chunks of 64 positions
    uint64_t full[NSLOT], empty[NSLOT];
    uint64_t s_full[2], s_empty[2], p_full[2], o_full[2], o_empty[2], q_full[2], q_empty[2];
    uint64_t ob_full, ob_empty, mma_done;
    uint64_t kv_ready[2];              // fused prologue: an item's new K/V row is in the cache
    alignas(16) uint8_t kvrow[2][HDIM * 2];  // ... staged here, stored by a bulk copy
    uint64_t grp[2], grp_end[2];       // softmax-group rendezvous (bounded, unlike bar.sync)
    float red_max[2][4][8];
    float red_sum[2][4][8];
    float ob[8][HDIM];                 // an item's normalised output rows, for the staging warp
    float ml[8][2];                    // and its (m, l) per head
    uint32_t tmem_base;
    int abort;
};

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait: false when the CTA has aborted or ~2 s passed (then the CTA aborts).
__device__ __forceinline__ bool tc_wait(uint64_t *bar, uint32_t parity, TcSmem &sm,
                                        uint32_t *status, uint32_t code) {
    const uint32_t addr = smem_u32(bar);
    uint64_t t0 = 0;
    for (uint32_t it = 0;; ++it) {
        uint32_t ok;
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; "
            "selp.u32 %0, 1, 0, p; }"
            : "=r"(ok) : "r"(addr), "r"(parity) : "memory");
        if (ok) return true;
        if ((it & 255) == 0) {
            if (*(volatile int *)&sm.abort) return false;
            const uint64_t now = globaltimer();
            if (it == 0) t0 = now;
            else if (now - t0 > 2000000000ull) {
                *(volatile int *)&sm.abort = 1;
                dev_flag(status, code);
                return false;
            }
        }
    }
}

// Non-blocking test: has the phase with this parity completed?
__device__ __forceinline__ bool mbar_test(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2; "
        "selp.u32 %0, 1, 0, p; }"
        : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}

// Byte offset of element (row, col) of a K-major operand stored as 128-byte swizzled
// rows: col in [0, 64) within one chunk.
__device__ __forceinline__ uint32_t sw128(int row, int col) {
    return (uint32_t)(row * 128 + ((((col >> 3) ^ (row & 7)) & 7) << 4) + (col & 7) * 2);
}

__device__ __forceinline__ uint16_t bf16_bits(float x) { return f32_to_bf16(x); }

// The token prologue fused into the split kernel (decode): the staging warp forms each
// item's q from the raw activations, and the CTA whose range ends at the token's slot
// appends its K/V row to the cache (the arithmetic of gqa_append_k: QK RMSNorm with a
// double sum of squares, NeoX RoPE on dims < rope_dim, bf16 store). q_in == NULL: q is the
// normalised q of vx27_gqa_append instead.
struct TcAppend {
    const void *q_in, *k_in, *v_in;   // [B][nq][hd], [B][nkv][hd] (act dtype)
    const float *qw, *kw, *rope;      // norm weights [hd]; rope table [rope_len][rope_dim]
    uint16_t *kc, *vc;                // the caches the tensor maps read
    int rope_len, rope_dim;
    float eps;
    int one_p;                        // zero-centred (1 + w) norm weights
};

__device__ __forceinline__ void load8f(const void *p, size_t i, bool bf, float (&x)[8]) {
    if (bf) {
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
__device__ __forceinline__ uint4 pack8_bf16(const float (&x)[8]) {
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; k++)
        w[k] = (uint32_t)f32_to_bf16(x[2 * k]) | ((uint32_t)f32_to_bf16(x[2 * k + 1]) << 16);
    return make_uint4(w[0], w[1], w[2], w[3]);
}

// A lane's 8 norm weights (dims 8*lane ..), with the zero-centred form's 1 + w applied.
__device__ __forceinline__ void tc_norm_w8(float (&wv)[8], const float *w, const TcAppend &ap,
                                           int lane) {
#pragma unroll
    for (int e = 0; e < 8; e++) {
        const float v = w[8 * lane + e];
        wv[e] = ap.one_p ? __fadd_rn(v, 1.0f) : v;
    }
}
// A lane's cos / sin entries of the position's rope row rr (NULL: none), for the dims it
// rotates (zero for dims past rope_dim).
__device__ __forceinline__ void tc_rope8(float (&c)[8], float (&sn)[8], const float *rr,
                                         const TcAppend &ap, int lane) {
    const int d0 = 8 * lane, half = ap.rope_dim / 2;
    const int i0 = d0 < half ? d0 : d0 - half;
#pragma unroll
    for (int e = 0; e < 8; e++) {
        const bool on = rr && d0 < ap.rope_dim;
        c[e] = on ? rr[i0 + e] : 0.f;
        sn[e] = on ? rr[half + i0 + e] : 0.f;
    }
}

// One 256-dim row held 8 dims per lane (dims 8*lane ..): RMSNorm then the rotation, as
// gqa_append_k rounds them; wv = the lane's norm weights (tc_norm_w8), c / sn = its rope
// entries (tc_rope8), rot = whether the position's rope row exists (false for a bad
// position). The per-row inputs are loaded once per item, so a row costs no memory round
// trip. Inlined into a row loop that is not unrolled: one copy of the code serves all
// rows, so the staging warp's code does not crowd the instruction cache the other roles'
// loops share (inlined and unrolled eight times it slowed a config 2 layer by 1.5%), and no
// call saves and restores registers (as a called function it took ~14 us per item).
__device__ __forceinline__ void tc_norm_rope(float (&y)[8], const float (&x)[8],
                                             const float (&wv)[8], const float (&c)[8],
                                             const float (&sn)[8], bool rot,
                                             const TcAppend &ap, int lane) {
    double ss = 0.0;
#pragma unroll
    for (int e = 0; e < 8; e++) ss += (double)x[e] * (double)x[e];
    ss = warp_sum_d(ss);
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)(ss / HDIM), ap.eps)));
    const int d0 = 8 * lane;
#pragma unroll
    for (int e = 0; e < 8; e++) y[e] = __fmul_rn(__fmul_rn(x[e], r), wv[e]);
    // the partner of dim d < half is d + half, held half / 8 lanes away
    const int half = ap.rope_dim / 2, hl = half / 8;
    const bool lo = d0 < half;
    float yp[8];
#pragma unroll
    for (int e = 0; e < 8; e++)
        yp[e] = __shfl_sync(0xffffffffu, y[e], (lo ? lane + hl : lane - hl) & 31);
    if (rot && d0 < ap.rope_dim) {
#pragma unroll
        for (int e = 0; e < 8; e++) {
            const float x0 = lo ? y[e] : yp[e], x1 = lo ? yp[e] : y[e];
            y[e] = lo ? __fsub_rn(__fmul_rn(x0, c[e]), __fmul_rn(x1, sn[e]))
                      : __fadd_rn(__fmul_rn(x0, sn[e]), __fmul_rn(x1, c[e]));
        }
    }
}

// One work item = (split s, KV head, sequence b), numbered w = s + n_splits * (kvh + nkv * b).
struct TcItem {
    int b, kvh, s, p0, p1, n_tiles, row0;
};

// Range of an item: [p_begin, p_end) (decode: [0, pos[b]]) cut into n_splits pieces on
// 128-position boundaries, clipped to the cache capacity.
__device__ __forceinline__ TcItem tc_item(int w, const int *__restrict__ pos, int cap, int nkv,
                                          int n_splits, int p_begin, int p_end) {
    TcItem it;
    it.s = w % n_splits;
    it.kvh = (w / n_splits) % nkv;
    it.b = w / (n_splits * nkv);
    const int rb = p_end >= 0 ? p_begin : 0;
    const int re = p_end >= 0 ? p_end : pos[it.b] + 1;
    const int tiles = (re - rb + TC_TILE - 1) / TC_TILE;
    const int per = (tiles + n_splits - 1) / n_splits;
    int p0 = rb + it.s * per * TC_TILE;
    int p1 = min(re, rb + (it.s + 1) * per * TC_TILE);
    if (p1 < p0) p1 = p0;
    p0 = max(p0, 0);
    p1 = min(p1, cap);
    it.p0 = p0;
    it.p1 = p1;
    it.n_tiles = p1 > p0 ? (p1 - p0 + TC_TILE - 1) / TC_TILE : 0;
    it.row0 = (it.b * nkv + it.kvh) * cap + p0;
    return it;
}

// Persistent: CTA c serves items c, c + gridDim.x, ... (one CTA per SM). The three roles
// walk the same item sequence with CTA-wide counters (ring slot j, tile g, non-empty item
// k), so the TMA ring keeps streaming across item boundaries; the softmax warps stage the
// next item's q in the second Q buffer while the current item runs.
template <int G, bool FUSED>
__global__ void __launch_bounds__(TC_THREADS, 1)
gqa_split_tc(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
             const __grid_constant__ CUtensorMap tmk32, const __grid_constant__ CUtensorMap tmv32,
             const float *__restrict__ q, const int *__restrict__ pos, float *__restrict__ parts,
             int cap, int B, int nq, int nkv, int n_splits, int p_begin, int p_end,
             const void *__restrict__ gate, void *__restrict__ out, int flags,
             const __grid_constant__ TcAppend ap, uint32_t *status) {
    extern __shared__ uint8_t smem_raw[];
    TcSmem &sm = *reinterpret_cast<TcSmem *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    constexpr bool fused = FUSED;  // the token prologue runs in this kernel (ap is set)
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n_items = n_splits * nkv * B, stride = gridDim.x;
    const size_t rec = (size_t)B * nq * (HDIM + 2);
    auto item = [&](int w) { return tc_item(w, pos, cap, nkv, n_splits, p_begin, p_end); };
    auto next_work = [&](int w) {  // first item >= w (in this CTA's sequence) with work
        for (; w < n_items; w += stride)
            if (item(w).n_tiles > 0) return w;
        return n_items;
    };
    // q rows of item w as bf16 hi (rows 0..G-1) and lo (rows G..2G-1) into Q buffer qb, by
    // the staging warp: all loads first, then the conversions
    auto stage_q_plain = [&](int w, int qb) {
        const TcItem it = item(w);
        const float2 *src = reinterpret_cast<const float2 *>(q + ((size_t)it.b * nq + it.kvh * G) * HDIM);
        float2 v[4 * G];
#pragma unroll
        for (int u = 0; u < 4 * G; u++) v[u] = src[lane + 32 * u];
#pragma unroll
        for (int u = 0; u < 4 * G; u++) {
            const int e = lane + 32 * u, g = e / (HDIM / 2), d = (e % (HDIM / 2)) * 2;
            const uint16_t hx = bf16_bits(v[u].x), hy = bf16_bits(v[u].y);
            const uint16_t lx = bf16_bits(v[u].x - bf16_to_f32(hx)), ly = bf16_bits(v[u].y - bf16_to_f32(hy));
            const int c = d >> 6, col = d & 63;
            *reinterpret_cast<uint32_t *>(&sm.q[qb][c][sw128(g, col)]) = hx | ((uint32_t)hy << 16);
            *reinterpret_cast<uint32_t *>(&sm.q[qb][c][sw128(g + G, col)]) = lx | ((uint32_t)ly << 16);
        }
        fence_proxy_async();
    };
    // fused prologue: q of item w normalised and rotated from q_in into Q buffer qb (then
    // q_full[qb]); the new token's K/V row into the cache when its slot ends this item's
    // range, then kv_ready[qb] (after a proxy fence: the TMA loads read that row). All rows
    // are loaded before any arithmetic, so their latencies overlap.
    auto stage_q_fused = [&](int w, int qb) {
        const TcItem it = item(w);
        const int p = pos[it.b];
        const bool bf = flags & VX27_F_ACT_BF16;
        const bool p_ok = p >= 0 && p < ap.rope_len;
        const float *rr = ap.rope_dim > 0 && p_ok ? ap.rope + (size_t)p * ap.rope_dim : nullptr;
        if (ap.rope_dim > 0 && !p_ok && lane == 0) dev_flag(status, VX_DEV_BAD_ARG);
        const bool app = p >= it.p0 && p < it.p1;  // this item's range ends at the token's slot
        const int d0 = 8 * lane, c = d0 >> 6, col = d0 & 63;
        const size_t q_row = ((size_t)it.b * nq + it.kvh * G) * HDIM + d0;
        const size_t kv_row = ((size_t)it.b * nkv + it.kvh) * HDIM + d0;
        float x[G + 2][8];  // q rows of the group, then k and v
        if (bf) {
            uint4 raw[G + 2];
#pragma unroll
            for (int h = 0; h < G; h++)
                raw[h] = *reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(ap.q_in) +
                                                          q_row + (size_t)h * HDIM);
            if (app) {
                raw[G] = *reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(ap.k_in) + kv_row);
                raw[G + 1] = *reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(ap.v_in) + kv_row);
            } else {
                raw[G] = raw[G + 1] = make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int h = 0; h < G + 2; h++) {
                const uint32_t wv[4] = {raw[h].x, raw[h].y, raw[h].z, raw[h].w};
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    x[h][2 * k] = bf16_to_f32(wv[k] & 0xffffu);
                    x[h][2 * k + 1] = bf16_to_f32(wv[k] >> 16);
                }
            }
        } else {
            float4 raw[G + 2][2];
#pragma unroll
            for (int h = 0; h < G; h++) {
                const float4 *f = reinterpret_cast<const float4 *>(static_cast<const float *>(ap.q_in) +
                                                                   q_row + (size_t)h * HDIM);
                raw[h][0] = f[0];
                raw[h][1] = f[1];
            }
            if (app) {
                const float4 *fk = reinterpret_cast<const float4 *>(static_cast<const float *>(ap.k_in) + kv_row);
                const float4 *fv = reinterpret_cast<const float4 *>(static_cast<const float *>(ap.v_in) + kv_row);
                raw[G][0] = fk[0]; raw[G][1] = fk[1];
                raw[G + 1][0] = fv[0]; raw[G + 1][1] = fv[1];
            } else {
                raw[G][0] = raw[G][1] = raw[G + 1][0] = raw[G + 1][1] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int h = 0; h < G + 2; h++) {
                x[h][0] = raw[h][0].x; x[h][1] = raw[h][0].y; x[h][2] = raw[h][0].z; x[h][3] = raw[h][0].w;
                x[h][4] = raw[h][1].x; x[h][5] = raw[h][1].y; x[h][6] = raw[h][1].z; x[h][7] = raw[h][1].w;
            }
        }
        // the item's norm weights and rope entries, once for all its rows
        float wq[8], wk[8], rc[8], rs[8];
        tc_norm_w8(wq, ap.qw, ap, lane);
        if (app) tc_norm_w8(wk, ap.kw, ap, lane);
        tc_rope8(rc, rs, rr, ap, lane);
#pragma unroll 1
        for (int h = 0; h < G; h++) {
            float y[8], lo8[8];
            tc_norm_rope(y, x[h], wq, rc, rs, rr != nullptr, ap, lane);
#pragma unroll
            for (int e = 0; e < 8; e++) lo8[e] = y[e] - bf16_to_f32(f32_to_bf16(y[e]));
            *reinterpret_cast<uint4 *>(&sm.q[qb][c][sw128(h, col)]) = pack8_bf16(y);
            *reinterpret_cast<uint4 *>(&sm.q[qb][c][sw128(h + G, col)]) = pack8_bf16(lo8);
        }
        fence_proxy_async();
        mbar_arrive(&sm.q_full[qb]);
        if (app) {
            // the rows go out as bulk copies (async proxy, like the TMA loads that read them
            // back), staged in shared memory
            float y[8];
            tc_norm_rope(y, x[G], wk, rc, rs, rr != nullptr, ap, lane);
            *reinterpret_cast<uint4 *>(&sm.kvrow[0][16 * lane]) = pack8_bf16(y);
            *reinterpret_cast<uint4 *>(&sm.kvrow[1][16 * lane]) = pack8_bf16(x[G + 1]);
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) {
                const size_t o = (((size_t)it.b * nkv + it.kvh) * cap + p) * HDIM;
                asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;"
                             ::"l"(ap.kc + o), "r"(smem_u32(sm.kvrow[0])), "r"(HDIM * 2) : "memory");
                asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;"
                             ::"l"(ap.vc + o), "r"(smem_u32(sm.kvrow[1])), "r"(HDIM * 2) : "memory");
                asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");  // stores complete
            }
            __syncwarp();
        }
        mbar_arrive(&sm.kv_ready[qb]);
    };
    // q of item w into Q buffer qb, then q_full[qb]
    auto stage_q = [&](int w, int qb) {
        if constexpr (FUSED) {
            stage_q_fused(w, qb);
        } else {
            stage_q_plain(w, qb);
            mbar_arrive(&sm.q_full[qb]);
        }
    };
    const int w_first = next_work(blockIdx.x);

    // ---- prologue --------------------------------------------------------------
    if (tid == 0) {
        for (int i = 0; i < NSLOT; i++) { mbar_init(&sm.full[i], 1); mbar_init(&sm.empty[i], 1); }
        for (int i = 0; i < 2; i++) {
            mbar_init(&sm.s_full[i], 1);
            mbar_init(&sm.s_empty[i], 128);
            mbar_init(&sm.p_full[i], 128);
            mbar_init(&sm.o_full[i], 1);
            mbar_init(&sm.o_empty[i], 128);
            mbar_init(&sm.q_full[i], 32);
            mbar_init(&sm.q_empty[i], 1);
            mbar_init(&sm.grp[i], 128);
            mbar_init(&sm.grp_end[i], 128);
            mbar_init(&sm.kv_ready[i], 32);
        }
        mbar_init(&sm.ob_full, 128);
        mbar_init(&sm.ob_empty, 1);
        mbar_init(&sm.mma_done, 1);
        sm.abort = 0;
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc(&sm.tmem_base, TMEM_COLS);
        tmem_relinquish();
        if (lane == 0) { tma_prefetch_desc(&tmk); tma_prefetch_desc(&tmv); }
    }
    if (warp >= 2 && warp < 6) {
        // zero both Q buffers and both P operands (rows >= 2G stay zero)
        uint4 z = make_uint4(0, 0, 0, 0);
        for (int e = tid - 64; e < (int)(sizeof(sm.q) + sizeof(sm.p)) / 16; e += 128)
            reinterpret_cast<uint4 *>(&sm.q[0][0][0])[e] = z;  // q and p are contiguous
        fence_proxy_async();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;
    // Issues ring chunk j (tile jj / 8 of item it, K for jj % 8 < 4, V otherwise).
    auto issue_chunk = [&](const TcItem &it, int jj, int j) {
        const int slot = j % NSLOT;
        const int tile = jj >> 3, r = jj & 7;
        // the last tile fetches only the 32-row boxes that hold positions of the range
        // (the rows past it are masked, and V's are zeroed, by the softmax warps)
        const int rows_left = it.p1 - (it.p0 + tile * TC_TILE);
        if (rows_left < TC_TILE) {
            const int nsub = (rows_left + 31) / 32;
            mbar_arrive_expect_tx(&sm.full[slot], nsub * (SLOT_BYTES / 4));
            for (int k = 0; k < nsub; k++)
                tma_load_2d(sm.ring[slot] + k * (SLOT_BYTES / 4), r < 4 ? &tmk32 : &tmv32,
                            (r & 3) * 64, it.row0 + tile * TC_TILE + 32 * k, &sm.full[slot]);
        } else {
            mbar_arrive_expect_tx(&sm.full[slot], SLOT_BYTES);
            tma_load_2d(sm.ring[slot], r < 4 ? &tmk : &tmv, (r & 3) * 64,
                        it.row0 + tile * TC_TILE, &sm.full[slot]);
        }
    };
    // VX27_F_PREFETCH_KV: the first ring round of the first item is requested before the
    // wait for the previous kernel (which, by the flag's contract, writes neither pos nor
    // any cache row but the token's), except the tile that holds the token's row
    int j_pre = 0;
    if ((flags & VX27_F_PREFETCH_KV) && warp == 0 && lane == 0 && w_first < n_items) {
        const TcItem it = item(w_first);
        const int p_tok = p_end >= 0 ? -1 : pos[it.b];
        const int tok_tile = (p_tok >= it.p0 && p_tok < it.p1) ? (p_tok - it.p0) / TC_TILE : -1;
        for (; j_pre < NSLOT && j_pre < it.n_tiles * 8 && (j_pre >> 3) != tok_tile; j_pre++)
            issue_chunk(it, j_pre, j_pre);
    }
    // q, gate, positions and the newest cache rows come from the kernels before this one
    grid_dep_wait();
    if (tid == 0) grid_dep_launch();

    if (warp == 0) {
        // ---- TMA producer --------------------------------------------------------
        if (lane == 0) {
            int j = 0;   // ring items issued by this CTA
            int kp = 0;  // items with work seen
            bool ok = true;
            for (int w = w_first; w < n_items && ok; w = next_work(w + stride), kp++) {
                const TcItem it = item(w);
                for (int jj = 0; jj < it.n_tiles * 8; jj++, j++) {
                    // fused prologue: the last tile may hold the new token's row, written by
                    // the staging warp when it staged this item's q
                    if (fused && jj == (it.n_tiles - 1) * 8 &&
                        !tc_wait(&sm.kv_ready[kp & 1], (kp >> 1) & 1, sm, status, VX_DEV_TIMEOUT_TMA)) {
                        ok = false;
                        break;
                    }
                    if (j < j_pre) continue;  // requested before the dependency wait
                    const int slot = j % NSLOT, round = j / NSLOT;
                    if (round > 0 &&
                        !tc_wait(&sm.empty[slot], (round - 1) & 1, sm, status, VX_DEV_TIMEOUT_TMA)) {
                        ok = false;
                        break;
                    }
                    issue_chunk(it, jj, j);
                }
            }
            if (sm.abort) {  // let the copies already issued land before the CTA exits
                const int jn = max(j, j_pre);
                for (int k = max(0, jn - NSLOT); k < jn; k++) {
                    const uint32_t addr = smem_u32(&sm.full[k % NSLOT]);
                    for (int it = 0; it < (1 << 20); it++) {
                        uint32_t ok2;
                        asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                                     : "=r"(ok2) : "r"(addr), "r"((uint32_t)((k / NSLOT) & 1)) : "memory");
                        if (ok2) break;
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ---- MMA issuer: S(g) = K_g Q^T, then O(g-1) = V_{g-1}^T P_{g-1}^T -----------
        if (lane == 0) {
            const uint32_t id1 = idesc_bf16(128, 16, false, false);
            const uint32_t id2 = idesc_bf16(128, 16, true, false);
            const uint32_t ring0 = smem_u32(sm.ring[0]);
            // Non-blocking schedule of the two MMA streams: S(gs) chunk by chunk as its K
            // chunks land, O(go) half by half as P(go) and its V chunks are ready, each
            // issued as soon as its inputs are there. (Waiting for S(g+1)'s K chunks before
            // issuing O(g) held V(g)'s ring slots for most of a tile and gated the
            // producer.) S runs at most one tile ahead of O: S(gs)'s K chunks reuse the
            // slots of O(gs-2)'s V chunks and O(go)'s V chunks those of S(go-1)'s K
            // chunks, so every slot's phases are awaited in order.
            bool ok = true;
            int ws = w_first, n_ts = ws < n_items ? item(ws).n_tiles : 0, is = 0, kqs = 0;
            int gs = 0, cs = 0, go = 0, ho = 0;
            bool s_started = false, o_started = false;
            uint32_t spins = 0;
            uint64_t t_idle = 0;
            while (ok && (ws < n_items || go < gs)) {
                bool progressed = false;
                if (go < gs) {  // ---- O(go) = V(go)^T P(go)^T, two halves of 4 V chunks
                    const int bb = go & 1;
                    if (!o_started &&
                        mbar_test(&sm.p_full[bb], (go >> 1) & 1) &&
                        (go < 2 || mbar_test(&sm.o_empty[bb], ((go >> 1) - 1) & 1)))
                        o_started = true;
                    if (o_started) {
                        const int j0 = 8 * go + 4 + 2 * ho, s0 = j0 % NSLOT, s1 = (j0 + 1) % NSLOT;
                        if (mbar_test(&sm.full[s0], (j0 / NSLOT) & 1) &&
                            mbar_test(&sm.full[s1], ((j0 + 1) / NSLOT) & 1)) {
                            tc_fence_after();
                            const uint32_t pb = smem_u32(sm.p[bb][0]);
#pragma unroll
                            for (int kk = 0; kk < 8; kk++)
                                mma_bf16(tmem + 32 + bb * 32 + ho * 16,
                                         sdesc_sw128(ring0 + s0 * SLOT_BYTES + kk * 2048, SLOT_BYTES, 1024),
                                         sdesc_sw128(pb + (kk >> 2) * 2048 + (kk & 3) * 32, 16, 1024),
                                         id2, kk != 0);
                            mma_commit(&sm.empty[s0]);
                            mma_commit(&sm.empty[s1]);
                            progressed = true;
                            if (++ho == 2) {
                                mma_commit(&sm.o_full[bb]);
                                ho = 0;
                                o_started = false;
                                go++;
                            }
                        }
                    }
                }
                if (ws < n_items && gs - go <= 1) {  // ---- S(gs) = K(gs) Q^T, 4 K chunks
                    const int bb = gs & 1;
                    if (!s_started && (is > 0 || mbar_test(&sm.q_full[kqs & 1], (kqs >> 1) & 1)) &&
                        (gs < 2 || mbar_test(&sm.s_empty[bb], ((gs >> 1) - 1) & 1)))
                        s_started = true;
                    if (s_started) {
                        const int j = 8 * gs + cs, slot = j % NSLOT;
                        if (mbar_test(&sm.full[slot], (j / NSLOT) & 1)) {
                            tc_fence_after();
                            const uint32_t q0 = smem_u32(sm.q[kqs & 1][0]);
#pragma unroll
                            for (int kk = 0; kk < 4; kk++)
                                mma_bf16(tmem + bb * 16,
                                         sdesc_sw128(ring0 + slot * SLOT_BYTES + kk * 32, 16, 1024),
                                         sdesc_sw128(q0 + cs * 2048 + kk * 32, 16, 1024), id1,
                                         (cs | kk) != 0);
                            mma_commit(&sm.empty[slot]);
                            progressed = true;
                            if (++cs == 4) {
                                mma_commit(&sm.s_full[bb]);
                                cs = 0;
                                s_started = false;
                                gs++;
                                if (++is == n_ts) {  // the item's S MMAs are all issued
                                    mma_commit(&sm.q_empty[kqs & 1]);
                                    is = 0;
                                    kqs++;
                                    ws = next_work(ws + stride);
                                    n_ts = ws < n_items ? item(ws).n_tiles : 0;
                                }
                            }
                        }
                    }
                }
                if (progressed) {
                    spins = 0;
                } else if ((++spins & 255) == 0) {  // bounded like every wait (~2 s idle)
                    if (*(volatile int *)&sm.abort) ok = false;
                    const uint64_t now = globaltimer();
                    if (spins == 256) t_idle = now;
                    else if (now - t_idle > 2000000000ull) {
                        *(volatile int *)&sm.abort = 1;
                        dev_flag(status, VX_DEV_TIMEOUT_MMA);
                        ok = false;
                    }
                }
            }
            mma_commit(&sm.mma_done);
            tc_wait(&sm.mma_done, 0, sm, status, VX_DEV_TIMEOUT_MMA);
        }
    } else if (warp < 6) {
        // ---- softmax / correction / epilogue (warps 2..5); no global memory traffic --
        const int q4 = warp & 3;               // TMEM lane quarter of this warp
        const int r = q4 * 32 + lane;          // position within a tile; output dim r, r+128
        const uint32_t lane_addr = tmem + ((uint32_t)(q4 * 32) << 16);
        const float sc2 = 1.4426950408889634f * 0.0625f;  // log2(e) / sqrt(256)
        bool ok = true;
        int g = 0, kq = 0;  // tiles and items with work done so far
        for (int w = w_first; w < n_items && ok; w = next_work(w + stride)) {
            const TcItem it = item(w);
            float m2[8], l[8], acc_a[8], acc_b[8], al[8], al_prev[8];
#pragma unroll
            for (int h = 0; h < 8; h++) {
                m2[h] = -INFINITY; l[h] = 0.f; acc_a[h] = 0.f; acc_b[h] = 0.f; al_prev[h] = 0.f;
            }
            auto correction = [&](int t) {  // folds O(t) in with alpha_t = al_prev
                const int bb = t & 1;
                ok = ok && tc_wait(&sm.o_full[bb], (t >> 1) & 1, sm, status, VX_DEV_TIMEOUT_MMA);
                ok = __all_sync(0xffffffffu, ok);  // warp-uniform: tcgen05.ld is warp-wide
                if (!ok) return;
                tc_fence_after();
                float oa[16], ob[16];
                tmem_ld16(lane_addr + 32 + bb * 32, oa);
                tmem_ld16(lane_addr + 48 + bb * 32, ob);
                tc_fence_before();
                mbar_arrive(&sm.o_empty[bb]);
#pragma unroll
                for (int h = 0; h < 8; h++) {
                    if (h < G) {
                        acc_a[h] = fmaf(acc_a[h], al_prev[h], oa[h] + oa[h + G]);
                        acc_b[h] = fmaf(acc_b[h], al_prev[h], ob[h] + ob[h + G]);
                    }
                }
            };
            for (int i = 0; i < it.n_tiles && ok; i++) {
                const int gi = g + i, bb = gi & 1;
                ok = tc_wait(&sm.s_full[bb], (gi >> 1) & 1, sm, status, VX_DEV_TIMEOUT_MMA);
                ok = __all_sync(0xffffffffu, ok);
                if (!ok) break;
                tc_fence_after();
                float v[16];
                tmem_ld16(lane_addr + bb * 16, v);
                tc_fence_before();
                mbar_arrive(&sm.s_empty[bb]);
                const int pabs = it.p0 + i * TC_TILE + r;
                const bool valid = pabs < it.p1;
                float x[8];
#pragma unroll
                for (int h = 0; h < 8; h++) {
                    x[h] = (h < G && valid) ? (v[h] + v[h + G]) * sc2 : -INFINITY;
                    const float t = warp_max(x[h]);
                    if (lane == 0) sm.red_max[bb][q4][h] = t;
                }
                // every thread of the group must see all four warps' maxima
                mbar_arrive(&sm.grp[bb]);
                ok = tc_wait(&sm.grp[bb], (gi >> 1) & 1, sm, status, VX_DEV_TIMEOUT_MMA);
                if (!ok) break;
#pragma unroll
                for (int h = 0; h < 8; h++) {
                    const float t = fmaxf(fmaxf(sm.red_max[bb][0][h], sm.red_max[bb][1][h]),
                                          fmaxf(sm.red_max[bb][2][h], sm.red_max[bb][3][h]));
                    const float mn = fmaxf(m2[h], t);
                    al[h] = (h < G) ? exp2f(m2[h] - mn) : 0.f;
                    m2[h] = mn;
                }
                uint8_t *pbuf = sm.p[bb][r >> 6];
#pragma unroll
                for (int h = 0; h < 8; h++) {
                    if (h < G) {
                        const float pr = exp2f(x[h] - m2[h]);
                        l[h] = fmaf(l[h], al[h], pr);
                        const uint16_t hi = bf16_bits(pr);
                        const uint16_t lo = bf16_bits(pr - bf16_to_f32(hi));
                        *reinterpret_cast<uint16_t *>(pbuf + sw128(h, r & 63)) = hi;
                        *reinterpret_cast<uint16_t *>(pbuf + sw128(h + G, r & 63)) = lo;
                    }
                }
                if (i == it.n_tiles - 1 && it.p0 + it.n_tiles * TC_TILE > it.p1) {
                    // V rows past the range may hold anything: zero them before V^T P^T reads them
                    for (int c = 0; c < 4 && ok; c++) {
                        const int j = 8 * gi + 4 + c;
                        ok = tc_wait(&sm.full[j % NSLOT], (j / NSLOT) & 1, sm, status, VX_DEV_TIMEOUT_TMA);
                        if (ok && !valid) {
                            uint4 *row = reinterpret_cast<uint4 *>(sm.ring[j % NSLOT] + r * 128);
#pragma unroll
                            for (int u = 0; u < 8; u++) row[u] = make_uint4(0, 0, 0, 0);
                        }
                    }
                }
                fence_proxy_async();
                mbar_arrive(&sm.p_full[bb]);
                if (i >= 1) correction(gi - 1);
#pragma unroll
                for (int h = 0; h < 8; h++) al_prev[h] = al[h];
            }
            if (ok) correction(g + it.n_tiles - 1);
            // epilogue: total l per head; the normalised rows go to the output buffer, which
            // the staging warp has emptied of the previous item
            const int eb = kq & 1;
#pragma unroll
            for (int h = 0; h < 8; h++) {
                const float t = warp_sum(l[h]);
                if (lane == 0) sm.red_sum[eb][q4][h] = t;
            }
            mbar_arrive(&sm.grp_end[eb]);
            ok = tc_wait(&sm.grp_end[eb], (kq >> 1) & 1, sm, status, VX_DEV_TIMEOUT_MMA) && ok;
            if (kq > 0)
                ok = tc_wait(&sm.ob_empty, (kq - 1) & 1, sm, status, VX_DEV_TIMEOUT_MMA) && ok;
#pragma unroll
            for (int h = 0; h < 8; h++) {
                if (h < G) {
                    const float L = sm.red_sum[eb][0][h] + sm.red_sum[eb][1][h] +
                                    sm.red_sum[eb][2][h] + sm.red_sum[eb][3][h];
                    const float inv = L > 0.f ? 1.0f / L : 0.f;
                    sm.ob[h][r] = acc_a[h] * inv;
                    sm.ob[h][r + 128] = acc_b[h] * inv;
                    if (r == 0) {
                        sm.ml[h][0] = L > 0.f ? m2[h] * 0.6931471805599453f : -INFINITY;
                        sm.ml[h][1] = L;
                    }
                }
            }
            mbar_arrive(&sm.ob_full);
            g += it.n_tiles;
            kq++;
        }
    } else {
        // ---- staging warp: every global load and store of the CTA except the TMA ring --
        // (q of the next item, gate values, the output or the partial record), so that no
        // release in the softmax warps waits on an HBM round trip
        const bool bf_gate = flags & VX27_F_ACT_BF16, bf_out = flags & VX27_F_OUT_BF16;
        bool ok = true;
        int kq = 0;  // items with work seen so far
        if (w_first < n_items) {
            stage_q(w_first, 0);
        }
        for (int w = blockIdx.x; w < n_items && ok; w += stride) {
            const TcItem it = item(w);
            const size_t base = ((size_t)it.b * nq + it.kvh * G) * HDIM;  // first of G rows
            float *po = parts + (size_t)it.s * rec;
            float *pml = po + (size_t)B * nq * HDIM;
            float gv[G][8];  // gate of this lane's 8 dims per head
            auto fetch_gate = [&]() {
#pragma unroll
                for (int h = 0; h < G; h++) {
                    const size_t i = base + (size_t)h * HDIM + 8 * lane;
                    if (!gate) {
#pragma unroll
                        for (int u = 0; u < 8; u++) gv[h][u] = 0.f;
                    } else if (bf_gate) {
                        const uint4 raw = *reinterpret_cast<const uint4 *>(
                            reinterpret_cast<const uint16_t *>(gate) + i);
                        const uint32_t wv[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
                        for (int u = 0; u < 4; u++) {
                            gv[h][2 * u] = bf16_to_f32((uint16_t)(wv[u] & 0xffff));
                            gv[h][2 * u + 1] = bf16_to_f32((uint16_t)(wv[u] >> 16));
                        }
                    } else {
                        const float4 a = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(gate) + i);
                        const float4 c = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(gate) + i + 4);
                        gv[h][0] = a.x; gv[h][1] = a.y; gv[h][2] = a.z; gv[h][3] = a.w;
                        gv[h][4] = c.x; gv[h][5] = c.y; gv[h][6] = c.z; gv[h][7] = c.w;
                    }
                }
            };
            // att for this lane's 8 dims of head h -> out (gated, the combine's arithmetic)
            // or the partial record
            auto write_rows = [&](auto att_of) {
#pragma unroll
                for (int h = 0; h < G; h++) {
                    float a[8];
#pragma unroll
                    for (int u = 0; u < 8; u++) {
                        a[u] = att_of(h, 8 * lane + u);
                        if (out && gate) a[u] = a[u] * (1.0f / (1.0f + expf(-gv[h][u])));
                    }
                    const size_t i = base + (size_t)h * HDIM + 8 * lane;
                    if (!out) {
                        float4 *d = reinterpret_cast<float4 *>(po + i);
                        d[0] = make_float4(a[0], a[1], a[2], a[3]);
                        d[1] = make_float4(a[4], a[5], a[6], a[7]);
                    } else if (bf_out) {
                        uint4 o;
                        o.x = f32_to_bf16(a[0]) | ((uint32_t)f32_to_bf16(a[1]) << 16);
                        o.y = f32_to_bf16(a[2]) | ((uint32_t)f32_to_bf16(a[3]) << 16);
                        o.z = f32_to_bf16(a[4]) | ((uint32_t)f32_to_bf16(a[5]) << 16);
                        o.w = f32_to_bf16(a[6]) | ((uint32_t)f32_to_bf16(a[7]) << 16);
                        *reinterpret_cast<uint4 *>(reinterpret_cast<uint16_t *>(out) + i) = o;
                    } else {
                        float4 *d = reinterpret_cast<float4 *>(reinterpret_cast<float *>(out) + i);
                        d[0] = make_float4(a[0], a[1], a[2], a[3]);
                        d[1] = make_float4(a[4], a[5], a[6], a[7]);
                    }
                }
            };
            if (it.n_tiles == 0) {  // empty range: neutral record, or a zero attention output
                if (out) fetch_gate();
                write_rows([&](int, int) { return 0.0f; });
                if (!out && lane < G) {
                    pml[((size_t)it.b * nq + it.kvh * G + lane) * 2] = -INFINITY;
                    pml[((size_t)it.b * nq + it.kvh * G + lane) * 2 + 1] = 0.0f;
                }
                continue;
            }
            // q of the next item with work into the other buffer, once the S MMAs of the
            // item before this one (its last reader) are complete
            const int wn = next_work(w + stride);
            if (wn < n_items) {
                if (kq >= 1)
                    ok = tc_wait(&sm.q_empty[(kq + 1) & 1], ((kq - 1) >> 1) & 1, sm, status,
                                 VX_DEV_TIMEOUT_MMA);
                if (ok) stage_q(wn, (kq + 1) & 1);
            }
            if (out) fetch_gate();
            ok = ok && tc_wait(&sm.ob_full, kq & 1, sm, status, VX_DEV_TIMEOUT_MMA);
            if (ok) {
                write_rows([&](int h, int d) { return sm.ob[h][d]; });
                if (!out && lane < G) {
                    pml[((size_t)it.b * nq + it.kvh * G + lane) * 2] = sm.ml[lane][0];
                    pml[((size_t)it.b * nq + it.kvh * G + lane) * 2 + 1] = sm.ml[lane][1];
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.ob_empty);
            kq++;
        }
    }
    // lanes that skipped a lane-0 role wait for it here, so whole warps reach the CTA
    // barrier together (it requires converged warps)
    __syncwarp();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

// one CTA per SM: the struct, aligned to 1024 B, within the 227 KB a CTA may opt into
static_assert(sizeof(TcSmem) + 1024 <= 232448, "split kernel shared memory over 227 KB");
size_t tc_smem_bytes() { return sizeof(TcSmem) + 1024; }

// One CTA per SM (fewer when there are fewer items).
static int tc_grid(int B, int nkv, int n_splits) {
    const long long items = (long long)B * nkv * n_splits;
    return (int)(items < num_sms() ? items : num_sms());
}

// The split kernel's launch: tensor maps over both caches, one CTA per SM; with pdl the
// launch may overlap its predecessor's tail (programmatic dependent launch), else a plain
// launch reporting to the status word given.
static int launch_tc(const void *kc, const void *vc, const float *q, const int *pos,
                     float *parts, int cap, int B, int nq, int nkv, int n_splits, int p_begin,
                     int p_end, const void *gate, void *out, int flags, const TcAppend &ap,
                     uint32_t *stw, bool pdl, cudaStream_t st, char *err, size_t errlen) {
    CUtensorMap mk, mv, mk32, mv32;
    const uint64_t rows = (uint64_t)B * nkv * cap;
    if (make_tmap_bf16_2d(&mk, kc, rows, HDIM, HDIM * 2, 64, TC_TILE, err, errlen) ||
        make_tmap_bf16_2d(&mv, vc, rows, HDIM, HDIM * 2, 64, TC_TILE, err, errlen) ||
        make_tmap_bf16_2d(&mk32, kc, rows, HDIM, HDIM * 2, 64, 32, err, errlen) ||
        make_tmap_bf16_2d(&mv32, vc, rows, HDIM, HDIM * 2, 64, 32, err, errlen))
        return -1;
    const size_t smem = tc_smem_bytes();
    const dim3 grid(tc_grid(B, nkv, n_splits));
#define VX_TCK(GG, FF)                                                                    \
    {                                                                                     \
        if (ensure_smem_attr((const void *)gqa_split_tc<GG, FF>, smem, err, errlen))      \
            return -1;                                                                    \
        if (pdl)                                                                          \
            VX_CK(launch_pdl(gqa_split_tc<GG, FF>, grid, dim3(TC_THREADS), smem, st, mk, mv, \
                             mk32, mv32, q, pos, parts, cap, B, nq, nkv, n_splits, p_begin, \
                             p_end, gate, out, flags, ap, stw));                           \
        else                                                                              \
            gqa_split_tc<GG, FF><<<grid, TC_THREADS, smem, st>>>(                          \
                mk, mv, mk32, mv32, q, pos, parts, cap, B, nq, nkv, n_splits, p_begin, p_end, \
                gate, out, flags, ap, stw);                                                \
    }
#define VX_TCG(GG)                                                                        \
    case GG:                                                                              \
        if (ap.q_in) VX_TCK(GG, true) else VX_TCK(GG, false)                              \
        break;
    switch (nq / nkv) {
        VX_TCG(1) VX_TCG(2) VX_TCG(4) VX_TCG(6) VX_TCG(8)
        default:
            return fail(err, errlen, "vx27_gqa: group size %d (nq/nkv) unsupported", nq / nkv);
    }
#undef VX_TCG
#undef VX_TCK
    VX_CK(cudaGetLastError());
    return 0;
}

int launch_split_tc(const void *kc, const void *vc, const float *q, const int *pos, float *parts,
                    int cap, int B, int nq, int nkv, int n_splits, int p_begin, int p_end,
                    cudaStream_t st, char *err, size_t errlen, const void *gate, void *out,
                    int flags) {
    if (out && n_splits != 1)
        return fail(err, errlen, "vx27_gqa: a direct output needs exactly one split");
    // the staging warp moves rows as 16-byte vectors (q as 8-byte pairs)
    if (((uintptr_t)parts & 15) || ((uintptr_t)out & 15) || ((uintptr_t)gate & 15) ||
        ((uintptr_t)q & 7))
        return fail(err, errlen,
                    "vx27_gqa: q must be 8-byte aligned, gate, out and the workspace 16-byte aligned");
    return launch_tc(kc, vc, q, pos, parts, cap, B, nq, nkv, n_splits, p_begin, p_end, gate, out,
                     flags, TcAppend{}, dev_status(), true, st, err, errlen);
}

// Decode with the token prologue fused in (q_in/k_in/v_in raw activations; the new K/V rows
// are appended at slot pos[b] by the kernel itself).
int launch_split_tc_fused(const void *q_in, const void *k_in, const void *v_in,
                          const float *qw, const float *kw, const float *rope, int rope_len,
                          int rope_dim, float eps, void *kc, void *vc, int cap, const int *pos,
                          float *parts, int B, int nq, int nkv, int n_splits, const void *gate,
                          void *out, int flags, cudaStream_t st, char *err, size_t errlen) {
    if (out && n_splits != 1)
        return fail(err, errlen, "vx27_gqa: a direct output needs exactly one split");
    if (((uintptr_t)parts & 15) || ((uintptr_t)out & 15) || ((uintptr_t)gate & 15) ||
        ((uintptr_t)q_in & 15) || ((uintptr_t)k_in & 15) || ((uintptr_t)v_in & 15))
        return fail(err, errlen,
                    "vx27_gqa_decode_fused: q_in, k_in, v_in, gate, out and the workspace must be "
                    "16-byte aligned");
    if (rope_dim < 0 || rope_dim > HDIM || (rope_dim & 15))
        return fail(err, errlen, "vx27_gqa_decode_fused: rope_dim=%d (a multiple of 16 up to 256)",
                    rope_dim);
    TcAppend ap{};
    ap.q_in = q_in;
    ap.k_in = k_in;
    ap.v_in = v_in;
    ap.qw = qw;
    ap.kw = kw;
    ap.rope = rope;
    ap.kc = (uint16_t *)kc;
    ap.vc = (uint16_t *)vc;
    ap.rope_len = rope_len;
    ap.rope_dim = rope_dim;
    ap.eps = eps;
    ap.one_p = (flags & VX27_F_NORM_1P) ? 1 : 0;
    return launch_tc(kc, vc, nullptr, pos, parts, cap, B, nq, nkv, n_splits, 0, -1, gate, out,
                     flags, ap, dev_status(), true, st, err, errlen);
}

// ---- host: tensor maps ---------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int make_tmap_bf16_2d(CUtensorMap *map, const void *base, uint64_t rows, uint64_t cols,
                      uint64_t row_pitch_bytes, uint32_t box_cols, uint32_t box_rows,
                      char *err, size_t errlen) {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
                cudaSuccess || !p)
            return fail(err, errlen, "cuTensorMapEncodeTiled unavailable from the driver");
        fn = (EncodeTiledFn)p;
    }
    if (((uintptr_t)base & 15) || (row_pitch_bytes & 15))
        return fail(err, errlen, "tensor map: base and row pitch must be 16-byte aligned");
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {row_pitch_bytes};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims,
                    strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(err, errlen, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return 0;
}

int make_tmap_bf16_3d(CUtensorMap *map, const void *base, uint64_t n0, uint64_t n1,
                      uint64_t n2, uint64_t s1, uint64_t s2, uint32_t b0, uint32_t b1,
                      uint32_t b2, char *err, size_t errlen) {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
                cudaSuccess || !p)
            return fail(err, errlen, "cuTensorMapEncodeTiled unavailable from the driver");
        fn = (EncodeTiledFn)p;
    }
    if (((uintptr_t)base & 15) || (s1 & 15) || (s2 & 15))
        return fail(err, errlen, "tensor map: base and strides must be 16-byte aligned");
    const cuuint64_t dims[3] = {n0, n1, n2};
    const cuuint64_t strides[2] = {s1, s2};
    const cuuint32_t box[3] = {b0, b1, b2};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims,
                    strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(err, errlen, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return 0;
}

}  // namespace vx27
