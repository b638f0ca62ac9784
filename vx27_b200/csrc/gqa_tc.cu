// K2 main loop on the 5th-generation tensor cores: split-KV flash decoding for one
// (sequence, KV head, split) per CTA, serving the G = nq/nkv query heads of the group.
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
constexpr int TC_THREADS = 192;
constexpr int HDIM = 256;
constexpr uint32_t TMEM_COLS = 128;    // S[2] at 0,16; O[2] (two halves) at 32..95

struct TcSmem {
    uint8_t ring[NSLOT][SLOT_BYTES];
    uint8_t q[4][2048];                // Q^T operand: 4 chunks of [16 rows x 128 bytes]
    uint8_t p[2][2][2048];             // P^T operand per buffer: 2 chunks of 64 positions
    uint64_t full[NSLOT], empty[NSLOT];
    uint64_t s_full[2], s_empty[2], p_full[2], o_full[2], o_empty[2], mma_done;
    uint64_t grp[2], grp_end;          // softmax-group rendezvous (bounded, unlike bar.sync)
    float red_max[2][4][8];
    float red_sum[4][8];
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

// Byte offset of element (row, col) of a K-major operand stored as 128-byte swizzled
// rows: col in [0, 64) within one chunk.
__device__ __forceinline__ uint32_t sw128(int row, int col) {
    return (uint32_t)(row * 128 + ((((col >> 3) ^ (row & 7)) & 7) << 4) + (col & 7) * 2);
}

__device__ __forceinline__ uint16_t bf16_bits(float x) { return f32_to_bf16(x); }

template <int G>
__global__ void __launch_bounds__(TC_THREADS, 1)
gqa_split_tc(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
             const __grid_constant__ CUtensorMap tmk32, const __grid_constant__ CUtensorMap tmv32,
             const float *__restrict__ q, const int *__restrict__ pos, float *__restrict__ parts,
             int cap, int B, int nq, int nkv, int n_splits, int p_begin, int p_end,
             uint32_t *status) {
    extern __shared__ uint8_t smem_raw[];
    TcSmem &sm = *reinterpret_cast<TcSmem *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const int s = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int h0 = kvh * G;  // the G query heads of this KV head (G = nq / nkv)

    // range of this split: [p_begin, p_end) (decode: [0, pos[b]]) cut into n_splits
    // pieces on 128-position boundaries
    int p0, p1;
    {
        const int rb = p_end >= 0 ? p_begin : 0;
        const int re = p_end >= 0 ? p_end : pos[b] + 1;
        const int tiles = (re - rb + TC_TILE - 1) / TC_TILE;
        const int per = (tiles + n_splits - 1) / n_splits;
        p0 = rb + s * per * TC_TILE;
        p1 = min(re, rb + (s + 1) * per * TC_TILE);
        if (p1 < p0) p1 = p0;
    }
    p0 = max(p0, 0);
    p1 = min(p1, cap);
    const size_t rec = (size_t)B * nq * (HDIM + 2);
    float *po = parts + (size_t)s * rec;
    float *pml = po + (size_t)B * nq * HDIM;
    const int n_tiles = p1 > p0 ? (p1 - p0 + TC_TILE - 1) / TC_TILE : 0;
    if (n_tiles == 0) {  // empty range: neutral record
        for (int e = tid; e < G * HDIM; e += TC_THREADS)
            po[((size_t)b * nq + h0 + e / HDIM) * HDIM + e % HDIM] = 0.0f;
        if (tid < G) {
            pml[((size_t)b * nq + h0 + tid) * 2] = -INFINITY;
            pml[((size_t)b * nq + h0 + tid) * 2 + 1] = 0.0f;
        }
        return;
    }
    const int row0 = (b * nkv + kvh) * cap + p0;

    // ---- prologue --------------------------------------------------------------
    if (tid == 0) {
        for (int i = 0; i < NSLOT; i++) { mbar_init(&sm.full[i], 1); mbar_init(&sm.empty[i], 1); }
        for (int i = 0; i < 2; i++) {
            mbar_init(&sm.s_full[i], 1);
            mbar_init(&sm.s_empty[i], 128);
            mbar_init(&sm.p_full[i], 128);
            mbar_init(&sm.o_full[i], 1);
            mbar_init(&sm.o_empty[i], 128);
        }
        mbar_init(&sm.mma_done, 1);
        mbar_init(&sm.grp[0], 128);
        mbar_init(&sm.grp[1], 128);
        mbar_init(&sm.grp_end, 128);
        sm.abort = 0;
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc(&sm.tmem_base, TMEM_COLS);
        tmem_relinquish();
        if (lane == 0) { tma_prefetch_desc(&tmk); tma_prefetch_desc(&tmv); }
    }
    if (warp >= 2) {
        const int t = tid - 64;  // 0..127
        // zero Q and both P operands (rows >= 2G stay zero), then write q hi/lo rows
        uint4 z = make_uint4(0, 0, 0, 0);
        for (int e = t; e < (int)(sizeof(sm.q) + sizeof(sm.p)) / 16; e += 128)
            reinterpret_cast<uint4 *>(&sm.q[0][0])[e] = z;  // q and p are contiguous
        named_bar(1, 128);
        for (int e = t; e < G * (HDIM / 2); e += 128) {
            const int g = e / (HDIM / 2), d = (e % (HDIM / 2)) * 2;
            const float2 v = *reinterpret_cast<const float2 *>(
                q + ((size_t)b * nq + h0 + g) * HDIM + d);
            const uint16_t hx = bf16_bits(v.x), hy = bf16_bits(v.y);
            const uint16_t lx = bf16_bits(v.x - bf16_to_f32(hx)), ly = bf16_bits(v.y - bf16_to_f32(hy));
            const int c = d >> 6, col = d & 63;
            *reinterpret_cast<uint32_t *>(&sm.q[c][sw128(g, col)]) = hx | ((uint32_t)hy << 16);
            *reinterpret_cast<uint32_t *>(&sm.q[c][sw128(g + G, col)]) = lx | ((uint32_t)ly << 16);
        }
        fence_proxy_async();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;

    if (warp == 0) {
        // ---- TMA producer --------------------------------------------------------
        if (lane == 0) {
            const int n_items = n_tiles * 8;
            int j = 0;
            for (; j < n_items; j++) {
                const int slot = j % NSLOT, round = j / NSLOT;
                if (round > 0 && !tc_wait(&sm.empty[slot], (round - 1) & 1, sm, status, VX_DEV_TIMEOUT_TMA))
                    break;
                const int tile = j >> 3, r = j & 7;
                // the last tile fetches only the 32-row boxes that hold positions of the
                // range (the rows past it are masked, and V's are zeroed, by the softmax warps)
                const int rows_left = p1 - (p0 + tile * TC_TILE);
                if (rows_left < TC_TILE) {
                    const int nsub = (rows_left + 31) / 32;
                    mbar_arrive_expect_tx(&sm.full[slot], nsub * (SLOT_BYTES / 4));
                    for (int k = 0; k < nsub; k++)
                        tma_load_2d(sm.ring[slot] + k * (SLOT_BYTES / 4), r < 4 ? &tmk32 : &tmv32,
                                    (r & 3) * 64, row0 + tile * TC_TILE + 32 * k, &sm.full[slot]);
                } else {
                    mbar_arrive_expect_tx(&sm.full[slot], SLOT_BYTES);
                    tma_load_2d(sm.ring[slot], r < 4 ? &tmk : &tmv, (r & 3) * 64,
                                row0 + tile * TC_TILE, &sm.full[slot]);
                }
            }
            if (sm.abort) {  // let the copies already issued land before the CTA exits
                for (int k = max(0, j - NSLOT); k < j; k++) {
                    const uint32_t addr = smem_u32(&sm.full[k % NSLOT]);
                    for (int it = 0; it < (1 << 20); it++) {
                        uint32_t ok;
                        asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                                     : "=r"(ok) : "r"(addr), "r"((uint32_t)((k / NSLOT) & 1)) : "memory");
                        if (ok) break;
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ---- MMA issuer ----------------------------------------------------------
        if (lane == 0) {
            const uint32_t id1 = idesc_bf16(128, 16, false, false);
            const uint32_t id2 = idesc_bf16(128, 16, true, false);
            const uint32_t ring0 = smem_u32(sm.ring[0]), q0 = smem_u32(sm.q[0]);
            bool ok = true;
            for (int i = 0; i <= n_tiles && ok; i++) {
                if (i < n_tiles) {  // S[i&1] = K_i Q^T
                    const int bb = i & 1;
                    if (i >= 2) ok = tc_wait(&sm.s_empty[bb], ((i >> 1) - 1) & 1, sm, status, VX_DEV_TIMEOUT_MMA);
                    for (int c = 0; c < 4 && ok; c++) {
                        const int j = 8 * i + c, slot = j % NSLOT;
                        ok = tc_wait(&sm.full[slot], (j / NSLOT) & 1, sm, status, VX_DEV_TIMEOUT_MMA);
                        if (!ok) break;
                        tc_fence_after();
#pragma unroll
                        for (int kk = 0; kk < 4; kk++)
                            mma_bf16(tmem + bb * 16,
                                     sdesc_sw128(ring0 + slot * SLOT_BYTES + kk * 32, 16, 1024),
                                     sdesc_sw128(q0 + c * 2048 + kk * 32, 16, 1024), id1,
                                     (c | kk) != 0);
                        mma_commit(&sm.empty[slot]);
                    }
                    if (ok) mma_commit(&sm.s_full[bb]);
                }
                if (i >= 1 && ok) {  // O[(i-1)&1] = V_{i-1}^T P_{i-1}^T
                    const int t = i - 1, bb = t & 1;
                    ok = tc_wait(&sm.p_full[bb], (t >> 1) & 1, sm, status, VX_DEV_TIMEOUT_MMA);
                    if (ok && t >= 2)
                        ok = tc_wait(&sm.o_empty[bb], ((t >> 1) - 1) & 1, sm, status, VX_DEV_TIMEOUT_MMA);
                    const uint32_t pb = smem_u32(sm.p[bb][0]);
                    for (int half = 0; half < 2 && ok; half++) {
                        const int j0 = 8 * t + 4 + 2 * half, s0 = j0 % NSLOT, s1 = (j0 + 1) % NSLOT;
                        ok = tc_wait(&sm.full[s0], (j0 / NSLOT) & 1, sm, status, VX_DEV_TIMEOUT_MMA) &&
                             tc_wait(&sm.full[s1], ((j0 + 1) / NSLOT) & 1, sm, status, VX_DEV_TIMEOUT_MMA);
                        if (!ok) break;
                        tc_fence_after();
#pragma unroll
                        for (int kk = 0; kk < 8; kk++)
                            mma_bf16(tmem + 32 + bb * 32 + half * 16,
                                     sdesc_sw128(ring0 + s0 * SLOT_BYTES + kk * 2048, SLOT_BYTES, 1024),
                                     sdesc_sw128(pb + (kk >> 2) * 2048 + (kk & 3) * 32, 16, 1024),
                                     id2, kk != 0);
                        mma_commit(&sm.empty[s0]);
                        mma_commit(&sm.empty[s1]);
                    }
                    if (ok) mma_commit(&sm.o_full[bb]);
                }
            }
            mma_commit(&sm.mma_done);
            tc_wait(&sm.mma_done, 0, sm, status, VX_DEV_TIMEOUT_MMA);
        }
    } else {
        // ---- softmax / correction / epilogue (warps 2..5) -------------------------
        const int q4 = warp & 3;               // TMEM lane quarter of this warp
        const int r = q4 * 32 + lane;          // position within a tile; output dim r, r+128
        const uint32_t lane_addr = tmem + ((uint32_t)(q4 * 32) << 16);
        const float sc2 = 1.4426950408889634f * 0.0625f;  // log2(e) / sqrt(256)
        float m2[8], l[8], acc_a[8], acc_b[8], al[8], al_prev[8];
#pragma unroll
        for (int h = 0; h < 8; h++) {
            m2[h] = -INFINITY; l[h] = 0.f; acc_a[h] = 0.f; acc_b[h] = 0.f; al_prev[h] = 0.f;
        }
        bool ok = true;
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
        for (int i = 0; i < n_tiles && ok; i++) {
            const int bb = i & 1;
            ok = tc_wait(&sm.s_full[bb], (i >> 1) & 1, sm, status, VX_DEV_TIMEOUT_MMA);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            tc_fence_after();
            float v[16];
            tmem_ld16(lane_addr + bb * 16, v);
            tc_fence_before();
            mbar_arrive(&sm.s_empty[bb]);
            const int pabs = p0 + i * TC_TILE + r;
            const bool valid = pabs < p1;
            float x[8];
#pragma unroll
            for (int h = 0; h < 8; h++) {
                x[h] = (h < G && valid) ? (v[h] + v[h + G]) * sc2 : -INFINITY;
                const float t = warp_max(x[h]);
                if (lane == 0) sm.red_max[bb][q4][h] = t;
            }
            // every thread of the group must see all four warps' maxima
            mbar_arrive(&sm.grp[bb]);
            ok = tc_wait(&sm.grp[bb], (i >> 1) & 1, sm, status, VX_DEV_TIMEOUT_MMA);
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
            if (i == n_tiles - 1 && p0 + n_tiles * TC_TILE > p1) {
                // V rows past the range may hold anything: zero them before V^T P^T reads them
                for (int c = 0; c < 4 && ok; c++) {
                    const int j = 8 * i + 4 + c;
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
            if (i >= 1) correction(i - 1);
#pragma unroll
            for (int h = 0; h < 8; h++) al_prev[h] = al[h];
        }
        if (ok) correction(n_tiles - 1);
        // epilogue: total l per head, normalised partial output
#pragma unroll
        for (int h = 0; h < 8; h++) {
            const float t = warp_sum(l[h]);
            if (lane == 0) sm.red_sum[q4][h] = t;
        }
        mbar_arrive(&sm.grp_end);
        const bool all = tc_wait(&sm.grp_end, 0, sm, status, VX_DEV_TIMEOUT_MMA);
        if (ok && all) {
#pragma unroll
            for (int h = 0; h < 8; h++) {
                if (h < G) {
                    const float L = sm.red_sum[0][h] + sm.red_sum[1][h] + sm.red_sum[2][h] +
                                    sm.red_sum[3][h];
                    const size_t hq = (size_t)b * nq + h0 + h;
                    const float inv = L > 0.f ? 1.0f / L : 0.f;
                    po[hq * HDIM + r] = acc_a[h] * inv;
                    po[hq * HDIM + r + 128] = acc_b[h] * inv;
                    if (r == 0) {
                        pml[hq * 2] = L > 0.f ? m2[h] * 0.6931471805599453f : -INFINITY;
                        pml[hq * 2 + 1] = L;
                    }
                }
            }
        }
    }
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

size_t tc_smem_bytes() { return sizeof(TcSmem) + 1024; }

int launch_split_tc(const void *kc, const void *vc, const float *q, const int *pos, float *parts,
                    int cap, int B, int nq, int nkv, int n_splits, int p_begin, int p_end,
                    cudaStream_t st, char *err, size_t errlen) {
    CUtensorMap mk, mv, mk32, mv32;
    const uint64_t rows = (uint64_t)B * nkv * cap;
    if (make_tmap_bf16_2d(&mk, kc, rows, HDIM, HDIM * 2, 64, TC_TILE, err, errlen) ||
        make_tmap_bf16_2d(&mv, vc, rows, HDIM, HDIM * 2, 64, TC_TILE, err, errlen) ||
        make_tmap_bf16_2d(&mk32, kc, rows, HDIM, HDIM * 2, 64, 32, err, errlen) ||
        make_tmap_bf16_2d(&mv32, vc, rows, HDIM, HDIM * 2, 64, 32, err, errlen))
        return -1;
    const size_t smem = tc_smem_bytes();
    const dim3 grid(n_splits, nkv, B);
    uint32_t *stw = dev_status();
#define VX_TCG(GG)                                                                        \
    case GG: {                                                                            \
        static bool attr = false;                                                         \
        if (!attr) {                                                                      \
            VX_CK(cudaFuncSetAttribute(gqa_split_tc<GG>,                                  \
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,       \
                                       (int)smem));                                       \
            attr = true;                                                                  \
        }                                                                                 \
        gqa_split_tc<GG><<<grid, TC_THREADS, smem, st>>>(mk, mv, mk32, mv32, q, pos, parts, cap, \
                                                         B, nq, nkv, n_splits, p_begin,    \
                                                         p_end, stw);                      \
        break;                                                                            \
    }
    switch (nq / nkv) {
        VX_TCG(1) VX_TCG(2) VX_TCG(4) VX_TCG(6) VX_TCG(8)
        default:
            return fail(err, errlen, "vx27_gqa: group size %d (nq/nkv) unsupported", nq / nkv);
    }
#undef VX_TCG
    VX_CK(cudaGetLastError());
    return 0;
}

// Same launch with an explicit device status word (null: timeouts end the waits without
// being recorded). Touches no allocator, for the entry point that allocates nothing.
int launch_split_tc_status(const void *kc, const void *vc, const float *q, const int *pos,
                           float *parts, int cap, int B, int nq, int nkv, int n_splits,
                           uint32_t *status, cudaStream_t st, char *err, size_t errlen) {
    CUtensorMap mk, mv, mk32, mv32;
    const uint64_t rows = (uint64_t)B * nkv * cap;
    if (make_tmap_bf16_2d(&mk, kc, rows, HDIM, HDIM * 2, 64, TC_TILE, err, errlen) ||
        make_tmap_bf16_2d(&mv, vc, rows, HDIM, HDIM * 2, 64, TC_TILE, err, errlen) ||
        make_tmap_bf16_2d(&mk32, kc, rows, HDIM, HDIM * 2, 64, 32, err, errlen) ||
        make_tmap_bf16_2d(&mv32, vc, rows, HDIM, HDIM * 2, 64, 32, err, errlen))
        return -1;
    const size_t smem = tc_smem_bytes();
    const dim3 grid(n_splits, nkv, B);
#define VX_TCS(GG)                                                                        \
    case GG: {                                                                            \
        static bool attr = false;                                                         \
        if (!attr) {                                                                      \
            VX_CK(cudaFuncSetAttribute(gqa_split_tc<GG>,                                  \
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,       \
                                       (int)smem));                                       \
            attr = true;                                                                  \
        }                                                                                 \
        gqa_split_tc<GG><<<grid, TC_THREADS, smem, st>>>(mk, mv, mk32, mv32, q, pos, parts, cap, \
                                                         B, nq, nkv, n_splits, 0, -1,      \
                                                         status);                          \
        break;                                                                            \
    }
    switch (nq / nkv) {
        VX_TCS(1) VX_TCS(2) VX_TCS(4) VX_TCS(6) VX_TCS(8)
        default:
            return fail(err, errlen, "vx27_gqa: group size %d (nq/nkv) unsupported", nq / nkv);
    }
#undef VX_TCS
    VX_CK(cudaGetLastError());
    return 0;
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
