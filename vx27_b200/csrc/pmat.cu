// K5: the packed-weight matvec of the layer projections on the device, batched over
// tokens: yb[b][r] = W[r] . xb[b] (src/vx27_pmat.h:12-20, vx27_pmat / vx27_pmat_batch).
// The weights stay packed in HBM in the reference's in-memory layouts and every output is
// bit-identical to the reference, so the per-format arithmetic order is reproduced:
//   BP3_128 (dtype 4; groups of 128 columns: three bit planes of 4 u32 + an fp16 scale,
//            52 B with padding): eight fp32 lanes over the whole row, lane l taking the
//            columns = l mod 8 in increasing order, q*scale by one multiply, then a fused
//            multiply-add; the lanes summed left to right at the end
//            (src/vx27_pmat.c:28-63, 133-177). Eight threads per row, thread = lane, so a
//            row's lanes run in parallel; x is staged in shared memory transposed by lane
//            so each thread reads its 16 values of a group as four float4. q*scale costs
//            two instructions per weight (bp3_codes).
//   Q8_K    (dtype 2; blocks of 256: float d, int8 qs[256], int16 bsums[16], 292 B): per
//            block eight FMA lanes summed left to right, times d in double, accumulated
//            in double (:10-24, :100-105, :187-195). One thread per row.
//   F32     (dtype 0): double products accumulated in column order (:96-99, :196-204).
//            One thread per row.
// Tokens run in passes of up to 8 (blockIdx.y), each thread keeping its accumulators
// for all of them, so a weight byte is read from HBM once per 8 tokens. One launch serves
// up to VX27_PMAT_MAX_GROUPS projections of the same x (a layer's input projections):
// their row blocks share the grid, so a small projection (48 rows) runs beside the large
// ones instead of as a launch of three CTAs.
#include "common.cuh"
#include "../../include/vx27_pmat.h"

namespace vx27 {
namespace {

constexpr int BP3_THREADS = 128;
constexpr int BP3_ROWS = BP3_THREADS / 8;  // 8 lanes per row; 16 rows (16 * 52 B = 832 B)
constexpr int XS_LANE = 20;                // floats per lane slot: 16 used, 4 pad (banks)
constexpr int ROW_THREADS = 128;           // Q8_K / F32: one thread per row
constexpr unsigned FULL = 0xffffffffu;
constexpr int MAXG = VX27_PMAT_MAX_GROUPS;

// The projections of one launch (same x, dtype and cols): CTAs blk0[i] .. blk0[i+1]-1
// along x serve group i.
struct PmatGroups {
    const uint8_t *W[MAXG];
    float *y[MAXG];
    int rows[MAXG];
    int blk0[MAXG + 1];
    int n;
};

__device__ __forceinline__ int pm_group(const PmatGroups &g, int bx) {
    int i = 0;
#pragma unroll
    for (int j = 1; j < MAXG; j++)
        if (j < g.n && bx >= g.blk0[j]) i = j;
    return i;
}

// The group scale's fp16 -> fp32 exactly as the reference forms it (src/vx27_pmat.c:38-41):
// exponent rebased by 112; an fp16 subnormal keeps exponent field 1 instead of scaling.
__device__ __forceinline__ float bp3_scale(uint16_t h) {
    const uint32_t u = h, sign = (u & 0x8000u) << 16, ex = (u >> 10) & 0x1Fu, man = u & 0x3FFu;
    uint32_t bits;
    if (ex == 0) bits = man ? (sign | ((ex + 1 + 112u) << 23) | (man << 13)) : sign;
    else if (ex == 31) bits = sign | 0x7F800000u | (man << 13);
    else bits = sign | ((ex + 112u) << 23) | (man << 13);
    return __uint_as_float(bits);
}

// Four codes of a lane, bytes c' = q + 4 (0..7) of v4, to q * scale. Placed in the
// mantissa of 2.0 a code gives a = 2 + c'/64 exactly. With EXACT_FMA (a finite positive
// scale, s1 = 64 sc, s2 = -132 sc, both exact) one fused multiply-add gives
// a * 64 sc - 132 sc = q * sc: the exact value has at most 14 significant bits, so its one
// rounding is exact and the result equals the reference's rounded product, signed zeros
// included (+0 for q = 0, as 0.0f * sc is for sc > 0). Otherwise (zero, negative, infinite
// or NaN scale; s1 = sc) q is formed exactly first and multiplied as the reference does.
template <bool EXACT_FMA>
__device__ __forceinline__ void bp3_codes(uint32_t v4, float s1, float s2, float (&qv)[4]) {
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const float a = __uint_as_float(__byte_perm(v4, 0x40000000u, 0x7044u | (j << 8)));
        if (EXACT_FMA) qv[j] = __fmaf_rn(a, s1, s2);
        else qv[j] = __fmul_rn(__fmaf_rn(a, 64.f, -132.f), s1);
    }
}

// Groups of 128 columns of x staged per chunk (two chunk buffers of 5-10 KB).
__host__ __device__ constexpr int bp3_kc(int tb) { return tb == 1 ? 8 : 16 / tb; }

// One 128-column group of R rows for this lane: each row's 16 weights against TB tokens'
// x, every x value read from shared memory once for the R rows.
template <int TB, int KC, int R, bool EXACT_FMA>
__device__ __forceinline__ void bp3_group(const uint32_t *const (&gw)[R], int l,
                                          const float (&s1)[R], const float (&s2)[R],
                                          const float *xk, float (&acc)[R][TB]) {
    uint32_t p[R][12];
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int i = 0; i < 12; i++) p[r][i] = gw[r][i];
#pragma unroll
    for (int w = 0; w < 4; w++) {
        float qv[R][4];
#pragma unroll
        for (int r = 0; r < R; r++) {
            // this lane's columns of word w: 32w + 8j + l, j = 0..3, one code per byte,
            // bit 2 flipped so that code ^ 4 = q + 4 in 0..7
            const uint32_t v4 = (((p[r][w] >> l) & 0x01010101u) |
                                 (((p[r][4 + w] >> l) & 0x01010101u) << 1) |
                                 (((p[r][8 + w] >> l) & 0x01010101u) << 2)) ^ 0x04040404u;
            bp3_codes<EXACT_FMA>(v4, s1[r], s2[r], qv[r]);
        }
#pragma unroll
        for (int b = 0; b < TB; b++) {
            const float4 xv = *reinterpret_cast<const float4 *>(
                xk + (size_t)b * KC * 8 * XS_LANE + 4 * w);
#pragma unroll
            for (int r = 0; r < R; r++) {
                acc[r][b] = fmaf(qv[r][0], xv.x, acc[r][b]);
                acc[r][b] = fmaf(qv[r][1], xv.y, acc[r][b]);
                acc[r][b] = fmaf(qv[r][2], xv.z, acc[r][b]);
                acc[r][b] = fmaf(qv[r][3], xv.w, acc[r][b]);
            }
        }
    }
}

// Rows per thread: two when a pass has 4 or 8 tokens, so that each x value read from shared
// memory feeds two rows' FMAs (the 8 lanes of a row read 8 different x float4s, so a
// warp's x load takes one shared-memory wavefront per row it serves).
__host__ __device__ constexpr int bp3_rows_per_thread(int tb) { return tb >= 4 ? 2 : 1; }

// Shared memory of a BP3 CTA: its block of packed rows (one bulk copy), then two x chunk
// buffers: element e of group kk of token b at xs[((b * KC + kk) * 8 + (e & 7)) * XS_LANE +
// (e >> 3)].
__host__ __device__ constexpr size_t bp3_xs_bytes(int tb) {
    return (size_t)2 * tb * bp3_kc(tb) * 8 * XS_LANE * 4;
}

__device__ __forceinline__ void cp_async_4(float *dst, const float *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Groups k0 .. k0+kn-1 of the nb tokens' x into a chunk buffer, transposed by lane, as
// asynchronous 4-byte copies: thread t copies element t of each group (coalesced reads;
// the 32 stores of a warp hit 32 different banks).
template <int KC>
__device__ __forceinline__ void bp3_stage_x(float *xsb, const float *xb, int b0, int nb,
                                            int cols, int k0, int kn, int tid) {
    float *d = xsb + (tid & 7) * XS_LANE + (tid >> 3);
    for (int b = 0; b < nb; b++)
        for (int kk = 0; kk < kn; kk++)
            cp_async_4(d + (b * KC + kk) * 8 * XS_LANE,
                       xb + (size_t)(b0 + b) * cols + (size_t)(k0 + kk) * 128 + tid);
}
__host__ __device__ inline size_t bp3_w_bytes(int cols, int R) {
    return ((size_t)BP3_ROWS * R * (size_t)(cols >> 7) * 52 + 15) & ~(size_t)15;
}

template <int TB>
__global__ void __launch_bounds__(BP3_THREADS)
pmat_bp3_k(const __grid_constant__ PmatGroups g, const float *__restrict__ xb, int cols, int B,
           uint32_t *status) {
    extern __shared__ __align__(128) uint8_t pm_smem[];
    __shared__ uint64_t wbar;
    constexpr int R = bp3_rows_per_thread(TB), ROWS = BP3_ROWS * R;
    const int tid = threadIdx.x, l = tid & 7, rl = tid >> 3, base = (tid & 31) & ~7;
    const int gi = pm_group(g, blockIdx.x), rows = g.rows[gi];
    const uint8_t *W = g.W[gi];
    float *yb = g.y[gi];
    const int r0 = (blockIdx.x - g.blk0[gi]) * ROWS, nr = min(ROWS, rows - r0);
    const int b0 = blockIdx.y * TB, nb = min(TB, B - b0);
    const int ng = cols >> 7;
    const size_t rb = (size_t)ng * 52;
    constexpr int KC = bp3_kc(TB);
    uint8_t *wsm = pm_smem;
    float *xs0 = reinterpret_cast<float *>(pm_smem + bp3_w_bytes(cols, R));
    float *xs1 = xs0 + TB * KC * 8 * XS_LANE;
    // the CTA's rows (thread row rl serves rows rl, rl + 16, ...) are contiguous in W and
    // start on a 16-byte boundary (16 * 52 is a multiple of 16): one bulk copy of the
    // 16-byte-aligned part, the tail by plain loads
    const size_t blk = (size_t)nr * rb, blk16 = blk & ~(size_t)15;
    const uint8_t *src = W + (size_t)r0 * rb;
    if (tid == 0) {
        mbar_init(&wbar, 1);
        fence_barrier_init();
    }
    __syncthreads();
    grid_dep_wait();  // x may come from the previous kernel
    if (tid == 0) {
        grid_dep_launch();
        mbar_arrive_expect_tx(&wbar, (uint32_t)blk16);
        for (size_t off = 0; off < blk16; off += 65536)
            bulk_g2s(wsm + off, src + off, (uint32_t)min((size_t)65536, blk16 - off), &wbar);
    }
    bp3_stage_x<KC>(xs0, xb, b0, nb, cols, 0, min(KC, ng), tid);
    cp_async_commit();
    for (size_t i = blk16 + tid; i < blk; i += BP3_THREADS) wsm[i] = src[i];
    float acc[R][TB];
    const uint8_t *wr[R];
#pragma unroll
    for (int r = 0; r < R; r++) {
#pragma unroll
        for (int b = 0; b < TB; b++) acc[r][b] = 0.f;
        const int row = rl + BP3_ROWS * r;
        wr[r] = wsm + (size_t)(row < nr ? row : 0) * rb;
    }
    bool ok = true;
    // x chunk c + 1 is copied in while chunk c is used; slots of tokens past nb are left
    // as they are (their sums are never stored)
    for (int k0 = 0, c = 0; k0 < ng; k0 += KC, c++) {
        const int kn = min(KC, ng - k0);
        const float *xc = (c & 1) ? xs1 : xs0;
        if (k0 + KC < ng)
            bp3_stage_x<KC>((c & 1) ? xs0 : xs1, xb, b0, nb, cols, k0 + KC,
                            min(KC, ng - k0 - KC), tid);
        cp_async_commit();
        cp_async_wait<1>();  // this thread's copies of chunk c have landed
        if (k0 > 0) __syncthreads();
        else {  // the weights: every thread waits (bounded), outcome made uniform
            uint32_t done = 0;
            for (uint32_t it = 0; it < (1u << 26) && !done; it++)
                asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0; selp.u32 %0, 1, 0, p; }"
                             : "=r"(done) : "r"(smem_u32(&wbar)) : "memory");
            ok = !__syncthreads_or(!done);  // a timeout leaves this CTA's outputs unwritten
            if (!ok && tid == 0) dev_flag(status, VX_DEV_TIMEOUT_TMA);
        }
        if (!ok) break;
        // the chunk's group scales of each row: lane l converts group k0 + l's, the row's
        // other lanes receive it by shuffle
        float sc_l[R];
#pragma unroll
        for (int r = 0; r < R; r++)
            sc_l[r] = l < kn ? bp3_scale(*reinterpret_cast<const unsigned short *>(
                                   wr[r] + (size_t)(k0 + l) * 52 + 48))
                             : 0.f;
        for (int kk = 0; kk < kn; kk++) {
            float sc[R], s64[R], s132[R];
            const uint32_t *gw[R];
            bool fast = true;  // every row's scale positive and finite
#pragma unroll
            for (int r = 0; r < R; r++) {
                sc[r] = __shfl_sync(FULL, sc_l[r], base + kk);
                s64[r] = sc[r] * 64.f;
                s132[r] = sc[r] * -132.f;
                fast = fast && sc[r] > 0.f && sc[r] <= 3.40282347e38f;
                gw[r] = reinterpret_cast<const uint32_t *>(wr[r] + (size_t)(k0 + kk) * 52);
            }
            const float *xk = xc + ((size_t)kk * 8 + l) * XS_LANE;
            if (fast)
                bp3_group<TB, KC, R, true>(gw, l, s64, s132, xk, acc);
            else
                bp3_group<TB, KC, R, false>(gw, l, sc, sc, xk, acc);
        }
        __syncthreads();  // chunk c's buffer is refilled two chunks on
    }
    cp_async_wait<0>();
    // lanes 0..7 of each row summed left to right
#pragma unroll
    for (int r = 0; r < R; r++) {
        const int row = rl + BP3_ROWS * r;
#pragma unroll
        for (int b = 0; b < TB; b++) {
            float t = __shfl_sync(FULL, acc[r][b], base);
#pragma unroll
            for (int j = 1; j < 8; j++) t = __fadd_rn(t, __shfl_sync(FULL, acc[r][b], base + j));
            if (ok && l == 0 && row < nr && b < nb) yb[(size_t)(b0 + b) * rows + r0 + row] = t;
        }
    }
}

template <int TB>
__global__ void __launch_bounds__(ROW_THREADS)
pmat_q8k_k(const __grid_constant__ PmatGroups g, const float *__restrict__ xb, int cols, int B) {
    const int gi = pm_group(g, blockIdx.x), rows = g.rows[gi];
    const uint8_t *W = g.W[gi];
    float *yb = g.y[gi];
    const int r = (blockIdx.x - g.blk0[gi]) * ROW_THREADS + threadIdx.x;
    if (r >= rows) return;
    const int b0 = blockIdx.y * TB, nb = min(TB, B - b0);
    const int nblk = cols >> 8;
    const uint8_t *row = W + (size_t)r * nblk * 292;
    double s[TB];
#pragma unroll
    for (int b = 0; b < TB; b++) s[b] = 0.0;
    for (int k = 0; k < nblk; k++) {
        const uint8_t *blk = row + (size_t)k * 292;
        const float d = __ldg(reinterpret_cast<const float *>(blk));
        const uint32_t *qw = reinterpret_cast<const uint32_t *>(blk + 4);
        float a[TB][8];
#pragma unroll
        for (int b = 0; b < TB; b++)
#pragma unroll
            for (int j = 0; j < 8; j++) a[b][j] = 0.f;
        for (int i = 0; i < 256; i += 8) {
            const uint32_t w0 = __ldg(qw + i / 4), w1 = __ldg(qw + i / 4 + 1);
            float qv[8];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                qv[j] = (float)(int)(int8_t)(w0 >> (8 * j));
                qv[4 + j] = (float)(int)(int8_t)(w1 >> (8 * j));
            }
#pragma unroll
            for (int b = 0; b < TB; b++) {
                const int bb = b < nb ? b : 0;
                const float4 *xp = reinterpret_cast<const float4 *>(
                    xb + (size_t)(b0 + bb) * cols + (size_t)k * 256 + i);
                const float4 x0 = __ldg(xp), x1 = __ldg(xp + 1);
                a[b][0] = fmaf(qv[0], x0.x, a[b][0]);
                a[b][1] = fmaf(qv[1], x0.y, a[b][1]);
                a[b][2] = fmaf(qv[2], x0.z, a[b][2]);
                a[b][3] = fmaf(qv[3], x0.w, a[b][3]);
                a[b][4] = fmaf(qv[4], x1.x, a[b][4]);
                a[b][5] = fmaf(qv[5], x1.y, a[b][5]);
                a[b][6] = fmaf(qv[6], x1.z, a[b][6]);
                a[b][7] = fmaf(qv[7], x1.w, a[b][7]);
            }
        }
#pragma unroll
        for (int b = 0; b < TB; b++) {
            float t = a[b][0];
#pragma unroll
            for (int j = 1; j < 8; j++) t = __fadd_rn(t, a[b][j]);
            s[b] = __dadd_rn(s[b], __dmul_rn((double)t, (double)d));
        }
    }
#pragma unroll
    for (int b = 0; b < TB; b++)
        if (b < nb) yb[(size_t)(b0 + b) * rows + r] = (float)s[b];
}

template <int TB>
__global__ void __launch_bounds__(ROW_THREADS)
pmat_f32_k(const __grid_constant__ PmatGroups g, const float *__restrict__ xb, int cols, int B) {
    const int gi = pm_group(g, blockIdx.x), rows = g.rows[gi];
    const float *W = reinterpret_cast<const float *>(g.W[gi]);
    float *yb = g.y[gi];
    const int r = (blockIdx.x - g.blk0[gi]) * ROW_THREADS + threadIdx.x;
    if (r >= rows) return;
    const int b0 = blockIdx.y * TB, nb = min(TB, B - b0);
    const float *row = W + (size_t)r * cols;
    double s[TB];
#pragma unroll
    for (int b = 0; b < TB; b++) s[b] = 0.0;
    for (int c = 0; c < cols; c++) {
        const double w = (double)__ldg(row + c);
#pragma unroll
        for (int b = 0; b < TB; b++) {
            const int bb = b < nb ? b : 0;
            s[b] = __dadd_rn(s[b], __dmul_rn(w, (double)__ldg(xb + (size_t)(b0 + bb) * cols + c)));
        }
    }
#pragma unroll
    for (int b = 0; b < TB; b++)
        if (b < nb) yb[(size_t)(b0 + b) * rows + r] = (float)s[b];
}

template <int TB>
int launch_pmat(PmatGroups g, uint32_t dtype, const float *xb, int cols, int B,
                cudaStream_t st, char *err, size_t errlen) {
    const unsigned passes = (unsigned)((B + TB - 1) / TB);
    const int per = dtype == VX27_PMAT_BP3_128 ? BP3_ROWS * bp3_rows_per_thread(TB) : ROW_THREADS;
    int nblk = 0;
    for (int i = 0; i < MAXG; i++) {
        g.blk0[i] = nblk;
        if (i < g.n) nblk += (g.rows[i] + per - 1) / per;
    }
    g.blk0[MAXG] = nblk;
    const dim3 grid((unsigned)nblk, passes);
    if (dtype == VX27_PMAT_BP3_128) {
        const size_t smem = bp3_w_bytes(cols, bp3_rows_per_thread(TB)) + bp3_xs_bytes(TB);
        if (smem > 220 * 1024)
            return fail(err, errlen, "vx27_pmat: cols=%d too wide for one CTA", cols);
        if (ensure_smem_attr((const void *)pmat_bp3_k<TB>, smem, err, errlen)) return -1;
        VX_CK(launch_pdl(pmat_bp3_k<TB>, grid, dim3(BP3_THREADS), smem, st, g, xb, cols, B,
                         dev_status()));
    } else if (dtype == VX27_PMAT_Q8_K) {
        VX_CK(launch_pdl(pmat_q8k_k<TB>, grid, dim3(ROW_THREADS), 0, st, g, xb, cols, B));
    } else {
        VX_CK(launch_pdl(pmat_f32_k<TB>, grid, dim3(ROW_THREADS), 0, st, g, xb, cols, B));
    }
    return 0;
}

}  // namespace
}  // namespace vx27

using namespace vx27;

extern "C" size_t vx27_pmat_row_bytes(uint32_t dtype, int cols) {
    if (cols <= 0) return 0;
    if (dtype == VX27_PMAT_F32) return (size_t)cols * 4;
    if (dtype == VX27_PMAT_Q8_K) return (size_t)(cols / 256) * 292;
    if (dtype == VX27_PMAT_BP3_128) return (size_t)(cols / 128) * 52;
    return 0;
}

extern "C" int vx27_pmat_multi_dev(int n, const void *const *W, uint32_t dtype,
                                   const float *xb, float *const *yb, const int *rows, int cols,
                                   int B, void *stream, char *err, size_t errlen) {
    if (n < 1 || n > MAXG || !W || !yb || !rows)
        return fail(err, errlen, "vx27_pmat: n=%d projections (1..%d) or null arrays", n, MAXG);
    if (!xb) return fail(err, errlen, "vx27_pmat: null x");
    if (cols <= 0 || B <= 0 || (long long)B > 65535ll * 8)
        return fail(err, errlen, "vx27_pmat: bad shape cols=%d B=%d", cols, B);
    if (dtype != VX27_PMAT_F32 && dtype != VX27_PMAT_Q8_K && dtype != VX27_PMAT_BP3_128)
        return fail(err, errlen, "vx27_pmat: dtype %u unsupported (0, 2 or 4)", dtype);
    if ((dtype == VX27_PMAT_Q8_K && cols % 256) || (dtype == VX27_PMAT_BP3_128 && cols % 128))
        return fail(err, errlen, "vx27_pmat: cols=%d not a whole number of blocks", cols);
    if (dtype != VX27_PMAT_F32 && ((uintptr_t)xb & 15))
        return fail(err, errlen, "vx27_pmat: xb must be 16-byte aligned");
    PmatGroups g = {};
    g.n = n;
    long long blocks = 0;
    for (int i = 0; i < n; i++) {
        if (!W[i] || !yb[i] || rows[i] <= 0)
            return fail(err, errlen, "vx27_pmat: projection %d: null pointer or rows=%d", i,
                        rows[i]);
        if ((uintptr_t)W[i] & (dtype == VX27_PMAT_BP3_128 ? 15 : 3))
            return fail(err, errlen,
                        "vx27_pmat: projection %d: W must be 4-byte (BP3_128: 16-byte) aligned",
                        i);
        blocks += rows[i] / 16 + 1;
        g.W[i] = (const uint8_t *)W[i];
        g.y[i] = yb[i];
        g.rows[i] = rows[i];
    }
    if (blocks > 0x7fffffffll) return fail(err, errlen, "vx27_pmat: too many rows");
    cudaStream_t st = (cudaStream_t)stream;
    if (B == 1) return launch_pmat<1>(g, dtype, xb, cols, B, st, err, errlen);
    if (B == 2) return launch_pmat<2>(g, dtype, xb, cols, B, st, err, errlen);
    if (B <= 4) return launch_pmat<4>(g, dtype, xb, cols, B, st, err, errlen);
    return launch_pmat<8>(g, dtype, xb, cols, B, st, err, errlen);
}

extern "C" int vx27_pmat_batch_dev(const void *W, uint32_t dtype, const float *xb, float *yb,
                                   int rows, int cols, int B, void *stream, char *err,
                                   size_t errlen) {
    return vx27_pmat_multi_dev(1, &W, dtype, xb, &yb, &rows, cols, B, stream, err, errlen);
}
