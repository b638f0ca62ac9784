// Shared helpers for the vx27 CUDA library (sm_100a): status/error plumbing,
// BF16 bit conversions, activation loads, and bounded mbarrier waits.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>
#include "../../include/vx27cuda.h"

namespace vx27 {

// ---- status -----------------------------------------------------------------
// Records the message in a thread-local buffer (vx27cuda_last_error) and in the
// caller's err/errlen when given. Returns -1 so call sites can `return fail(...)`.
int fail(char *err, size_t errlen, const char *fmt, ...);
int check_cuda(cudaError_t e, const char *what, char *err, size_t errlen);
// For the void-returning reference entry points: record, print, and abort unless
// VX27CUDA_NO_ABORT=1 is set in the environment (then outputs are left untouched).
void compat_fail(const char *fn, const char *msg);

#define VX_CK(call)                                                              \
    do {                                                                         \
        cudaError_t e_ = (call);                                                 \
        if (e_ != cudaSuccess) return ::vx27::check_cuda(e_, #call, err, errlen); \
    } while (0)

// ---- bf16 bit-level conversions (round to nearest even, as the oracle) -------
__host__ __device__ __forceinline__ float u32_as_f32(uint32_t u) {
#ifdef __CUDA_ARCH__
    return __uint_as_float(u);
#else
    float f;
    memcpy(&f, &u, 4);
    return f;
#endif
}
__host__ __device__ __forceinline__ uint32_t f32_as_u32(float f) {
#ifdef __CUDA_ARCH__
    return __float_as_uint(f);
#else
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
#endif
}
__host__ __device__ __forceinline__ float bf16_to_f32(uint16_t h) {
    return u32_as_f32((uint32_t)h << 16);
}
__host__ __device__ __forceinline__ uint16_t f32_to_bf16(float x) {
    uint32_t u = f32_as_u32(x);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

// Two floats to a packed bf16x2 word (round to nearest even), lo in bits 0-15.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}
// 2^x with the SFU instruction (relative error of a few ulp; 2^-inf = 0).
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// ---- device-side waits ------------------------------------------------------
// Every spin in this library is bounded; on timeout the kernel records a code in
// the per-device status word (dev_status(), read by vx27cuda_device_status) and
// abandons the wait.
#define VX_SPIN_LIMIT (1u << 26)
enum : uint32_t { VX_DEV_OK = 0, VX_DEV_TIMEOUT_TMA = 1, VX_DEV_TIMEOUT_MMA = 2,
                  VX_DEV_BAD_ARG = 3 };
// Device pointer of the status word of the current device: a module global, its address
// looked up on first use (no allocation).
uint32_t *dev_status();

__device__ __forceinline__ void dev_flag(uint32_t *st, uint32_t code) {
    if (st) atomicCAS(st, 0u, code);
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// Programmatic dependent launch: wait until the grid this one depends on (the previous
// kernel on the stream, when launched with the programmatic-serialization attribute) has
// finished and its memory is visible; and let the next such grid be scheduled early.
__device__ __forceinline__ void grid_dep_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_dep_launch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Returns true when the phase with the given parity completed, false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint32_t *st,
                                          uint32_t code) {
    uint32_t addr = smem_u32(bar);
    for (uint32_t it = 0; it < VX_SPIN_LIMIT; ++it) {
        uint32_t ok;
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; "
            "selp.u32 %0, 1, 0, p; }"
            : "=r"(ok) : "r"(addr), "r"(parity) : "memory");
        if (ok) return true;
    }
    dev_flag(st, code);
    return false;
}
// 1-D bulk copy global -> shared (TMA engine, no tensor map), completion on mbarrier.
// Both addresses 16-byte aligned and bytes a multiple of 16.
// Bulk prefetch of [gsrc, gsrc + bytes) into L2 (16-byte aligned, size a multiple of 16):
// more reads in flight without holding shared memory; a later copy of the range hits L2.
__device__ __forceinline__ void bulk_prefetch_l2(const void *gsrc, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(gsrc), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_g2s(void *smem_dst, const void *gsrc, uint32_t bytes,
                                         uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_u32(smem_dst)), "l"(gsrc), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

// Hardware named barrier for a subset of the CTA's warps (ids 1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---- activation element access ----------------------------------------------
template <bool BF16>
__device__ __forceinline__ float act_ld(const void *p, size_t i) {
    if constexpr (BF16) return bf16_to_f32(((const uint16_t *)p)[i]);
    else return ((const float *)p)[i];
}
template <bool BF16>
__device__ __forceinline__ void act_st(void *p, size_t i, float x) {
    if constexpr (BF16) ((uint16_t *)p)[i] = f32_to_bf16(x);
    else ((float *)p)[i] = x;
}

// The gate mapping of src/vx27_deltanet.c:58-69 (three-regime softplus, beta without
// dt_bias) in double with CUDA's device exp/log, which are within 1 ulp of the correctly
// rounded value; the C library's exp/log are not always correctly rounded either, so the
// double results can differ from vx27_deltanet_gate_params's in the last bit. The
// decode and prefill kernels use this, and vx27_deltanet_gate_params_dev exports it.
__device__ __forceinline__ void dn_gates_device(double a, double A_log, double b, double dt,
                                                double *beta, double *g_log) {
    *beta = 1.0 / (1.0 + exp(-b));
    const double x = a + dt;
    const double sp = x > 20.0 ? x : (x < -20.0 ? exp(x) : log(1.0 + exp(x)));
    *g_log = -exp(A_log) * sp;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

int num_sms();
// Sets a kernel's dynamic shared-memory limit on the current device once per (kernel,
// device, size); -1 with the CUDA error in err.
int ensure_smem_attr(const void *kernel, size_t bytes, char *err, size_t errlen);

// Launch with programmatic stream serialization: the grid may be scheduled while the
// previous kernel on the stream drains; the kernel calls grid_dep_wait() before it reads
// anything that kernel may have written (and grid_dep_launch() after that wait).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

}  // namespace vx27
