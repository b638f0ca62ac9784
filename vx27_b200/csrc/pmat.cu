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
//            so each thread reads its 16 values of a group as four float4.
//   Q8_K    (dtype 2; blocks of 256: float d, int8 qs[256], int16 bsums[16], 292 B): per
//            block eight FMA lanes summed left to right, times d in double, accumulated
//            in double (:10-24, :100-105, :187-195). One thread per row.
//   F32     (dtype 0): double products accumulated in column order (:96-99, :196-204).
//            One thread per row.
// Tokens run in passes of up to 8 (blockIdx.y), each thread keeping its accumulators
// for all of them, so a weight byte is read from HBM once per 8 tokens.
#include "common.cuh"
#include "../../include/vx27_pmat.h"

namespace vx27 {
namespace {

constexpr int BP3_THREADS = 128;
constexpr int BP3_ROWS = BP3_THREADS / 8;  // 8 lanes per row; 16 rows (16 * 52 B = 832 B)
constexpr int BP3_KC = 8;                  // groups of 128 columns staged per chunk
constexpr int XS_LANE = 20;                // floats per lane slot: 16 used, 4 pad (banks)
constexpr int ROW_THREADS = 128;           // Q8_K / F32: one thread per row
constexpr unsigned FULL = 0xffffffffu;

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

// Shared memory of a BP3 CTA: its block of packed rows (one bulk copy), then the staged
// x chunk: element e of group kk of token b at xs[((b * BP3_KC + kk) * 8 + (e & 7)) *
// XS_LANE + (e >> 3)].
__host__ __device__ constexpr size_t bp3_xs_bytes(int tb) {
    return (size_t)tb * BP3_KC * 8 * XS_LANE * 4;
}
__host__ __device__ inline size_t bp3_w_bytes(int cols) {
    return ((size_t)BP3_ROWS * (size_t)(cols >> 7) * 52 + 15) & ~(size_t)15;
}

template <int TB>
__global__ void __launch_bounds__(BP3_THREADS)
pmat_bp3_k(const uint8_t *__restrict__ W, const float *__restrict__ xb, float *__restrict__ yb,
           int rows, int cols, int B, uint32_t *status) {
    extern __shared__ __align__(128) uint8_t pm_smem[];
    __shared__ uint64_t wbar;
    const int tid = threadIdx.x, l = tid & 7, rl = tid >> 3;
    const int r0 = blockIdx.x * BP3_ROWS, nr = min(BP3_ROWS, rows - r0);
    const int b0 = blockIdx.y * TB, nb = min(TB, B - b0);
    const int ng = cols >> 7;
    const size_t rb = (size_t)ng * 52;
    uint8_t *wsm = pm_smem;
    float *xs = reinterpret_cast<float *>(pm_smem + bp3_w_bytes(cols));
    // the CTA's rows are contiguous in W and start on a 16-byte boundary (BP3_ROWS * 52 is
    // a multiple of 16): one bulk copy of the 16-byte-aligned part, the tail by plain loads
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
    for (size_t i = blk16 + tid; i < blk; i += BP3_THREADS) wsm[i] = src[i];
    float acc[TB];
#pragma unroll
    for (int b = 0; b < TB; b++) acc[b] = 0.f;
    const uint8_t *wr = wsm + (size_t)(rl < nr ? rl : 0) * rb;
    bool ok = true;
    for (int k0 = 0; k0 < ng; k0 += BP3_KC) {
        const int kn = min(BP3_KC, ng - k0);
        __syncthreads();  // the previous chunk has been read
        for (int idx = tid; idx < TB * kn * 32; idx += BP3_THREADS) {
            const int b = idx / (kn * 32), rem = idx - b * kn * 32, kk = rem >> 5;
            const int e4 = (rem & 31) * 4;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (b < nb)
                v = __ldg(reinterpret_cast<const float4 *>(xb + (size_t)(b0 + b) * cols +
                                                           (size_t)(k0 + kk) * 128 + e4));
            float *d = xs + ((size_t)(b * BP3_KC + kk) * 8 + (e4 & 7)) * XS_LANE + (e4 >> 3);
            d[0] = v.x;
            d[XS_LANE] = v.y;
            d[2 * XS_LANE] = v.z;
            d[3 * XS_LANE] = v.w;
        }
        __syncthreads();
        if (k0 == 0) {  // the weights: every thread waits (bounded), outcome made uniform
            uint32_t done = 0;
            for (uint32_t it = 0; it < (1u << 26) && !done; it++)
                asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0; selp.u32 %0, 1, 0, p; }"
                             : "=r"(done) : "r"(smem_u32(&wbar)) : "memory");
            ok = !__syncthreads_or(!done);  // a timeout leaves this CTA's outputs unwritten
            if (!ok && tid == 0) dev_flag(status, VX_DEV_TIMEOUT_TMA);
        }
        if (!ok) break;
        for (int kk = 0; kk < kn; kk++) {
            const uint32_t *gw = reinterpret_cast<const uint32_t *>(wr + (size_t)(k0 + kk) * 52);
            uint32_t p[12];
#pragma unroll
            for (int i = 0; i < 12; i++) p[i] = gw[i];
            const float sc = bp3_scale(*reinterpret_cast<const unsigned short *>(gw + 12));
            const float *xk = xs + ((size_t)kk * 8 + l) * XS_LANE;
#pragma unroll
            for (int w = 0; w < 4; w++) {
                // this lane's columns of word w: 32w + 8j + l, j = 0..3, one code per byte,
                // bit 2 flipped so that code ^ 4 = q + 4 in 0..7
                const uint32_t v4 = (((p[w] >> l) & 0x01010101u) |
                                     (((p[4 + w] >> l) & 0x01010101u) << 1) |
                                     (((p[8 + w] >> l) & 0x01010101u) << 2)) ^ 0x04040404u;
                float qv[4];
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    // 2^23 + (q + 4) minus 2^23 + 4 = q exactly, then q * scale rounded once
                    const float qf = __fsub_rn(__uint_as_float(0x4B000000u | ((v4 >> (8 * j)) & 7u)),
                                               8388612.0f);
                    qv[j] = __fmul_rn(qf, sc);
                }
#pragma unroll
                for (int b = 0; b < TB; b++) {
                    const float4 xv = *reinterpret_cast<const float4 *>(
                        xk + (size_t)b * BP3_KC * 8 * XS_LANE + 4 * w);
                    acc[b] = fmaf(qv[0], xv.x, acc[b]);
                    acc[b] = fmaf(qv[1], xv.y, acc[b]);
                    acc[b] = fmaf(qv[2], xv.z, acc[b]);
                    acc[b] = fmaf(qv[3], xv.w, acc[b]);
                }
            }
        }
    }
    // lanes 0..7 of the row summed left to right
    const int base = (tid & 31) & ~7;
#pragma unroll
    for (int b = 0; b < TB; b++) {
        float t = __shfl_sync(FULL, acc[b], base);
#pragma unroll
        for (int j = 1; j < 8; j++) t = __fadd_rn(t, __shfl_sync(FULL, acc[b], base + j));
        if (ok && l == 0 && rl < nr && b < nb) yb[(size_t)(b0 + b) * rows + r0 + rl] = t;
    }
}

template <int TB>
__global__ void __launch_bounds__(ROW_THREADS)
pmat_q8k_k(const uint8_t *__restrict__ W, const float *__restrict__ xb, float *__restrict__ yb,
           int rows, int cols, int B) {
    const int r = blockIdx.x * ROW_THREADS + threadIdx.x;
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
pmat_f32_k(const float *__restrict__ W, const float *__restrict__ xb, float *__restrict__ yb,
           int rows, int cols, int B) {
    const int r = blockIdx.x * ROW_THREADS + threadIdx.x;
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
int launch_pmat(const void *W, uint32_t dtype, const float *xb, float *yb, int rows, int cols,
                int B, cudaStream_t st, char *err, size_t errlen) {
    const unsigned passes = (unsigned)((B + TB - 1) / TB);
    if (dtype == VX27_PMAT_BP3_128) {
        const dim3 grid((unsigned)((rows + BP3_ROWS - 1) / BP3_ROWS), passes);
        const size_t smem = bp3_w_bytes(cols) + bp3_xs_bytes(TB);
        if (smem > 220 * 1024)
            return fail(err, errlen, "vx27_pmat_batch_dev: cols=%d too wide for one CTA", cols);
        if (ensure_smem_attr((const void *)pmat_bp3_k<TB>, smem, err, errlen)) return -1;
        VX_CK(launch_pdl(pmat_bp3_k<TB>, grid, dim3(BP3_THREADS), smem, st,
                         (const uint8_t *)W, xb, yb, rows, cols, B, dev_status()));
    } else if (dtype == VX27_PMAT_Q8_K) {
        const dim3 grid((unsigned)((rows + ROW_THREADS - 1) / ROW_THREADS), passes);
        VX_CK(launch_pdl(pmat_q8k_k<TB>, grid, dim3(ROW_THREADS), 0, st,
                         (const uint8_t *)W, xb, yb, rows, cols, B));
    } else {
        const dim3 grid((unsigned)((rows + ROW_THREADS - 1) / ROW_THREADS), passes);
        VX_CK(launch_pdl(pmat_f32_k<TB>, grid, dim3(ROW_THREADS), 0, st,
                         (const float *)W, xb, yb, rows, cols, B));
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

extern "C" int vx27_pmat_batch_dev(const void *W, uint32_t dtype, const float *xb, float *yb,
                                   int rows, int cols, int B, void *stream, char *err,
                                   size_t errlen) {
    if (!W || !xb || !yb) return fail(err, errlen, "vx27_pmat_batch_dev: null pointer argument");
    if (rows <= 0 || cols <= 0 || B <= 0 || (long long)B > 65535ll * 8)
        return fail(err, errlen, "vx27_pmat_batch_dev: bad shape rows=%d cols=%d B=%d", rows, cols, B);
    if (dtype != VX27_PMAT_F32 && dtype != VX27_PMAT_Q8_K && dtype != VX27_PMAT_BP3_128)
        return fail(err, errlen, "vx27_pmat_batch_dev: dtype %u unsupported (0, 2 or 4)", dtype);
    if ((dtype == VX27_PMAT_Q8_K && cols % 256) || (dtype == VX27_PMAT_BP3_128 && cols % 128))
        return fail(err, errlen, "vx27_pmat_batch_dev: cols=%d not a whole number of blocks", cols);
    if (((uintptr_t)W & (dtype == VX27_PMAT_BP3_128 ? 15 : 3)) ||
        (dtype != VX27_PMAT_F32 && ((uintptr_t)xb & 15)))
        return fail(err, errlen,
                    "vx27_pmat_batch_dev: W must be 4-byte (BP3_128: 16-byte) aligned, xb "
                    "16-byte aligned");
    cudaStream_t st = (cudaStream_t)stream;
    if (B == 1) return launch_pmat<1>(W, dtype, xb, yb, rows, cols, B, st, err, errlen);
    if (B == 2) return launch_pmat<2>(W, dtype, xb, yb, rows, cols, B, st, err, errlen);
    if (B <= 4) return launch_pmat<4>(W, dtype, xb, yb, rows, cols, B, st, err, errlen);
    return launch_pmat<8>(W, dtype, xb, yb, rows, cols, B, st, err, errlen);
}
