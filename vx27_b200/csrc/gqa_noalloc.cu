// vx27_gqa_decode_batch_noalloc: the split-KV GQA decode of vx27_gqa_decode_batch for
// callers that have no device workspace to give and must not have this library
// allocate one. Its partial (m, l, o) records live in a fixed array in the module's own
// global memory instead of a caller workspace or a cudaMalloc.
//
// The array below is held on every GPU where this library's module is loaded, until the
// process exits. With CUDA's lazy module loading (the default since CUDA 12) the module,
// and with it the array, may be loaded only by the first call on a device, so that call
// can fail for lack of device memory; callers make it during their set-up, before they
// hand the rest of the memory to a KV cache. In host code the array's name is only a
// host-side stand-in for the device symbol, so the device address is looked up once per
// device with cudaGetSymbolAddress (on the first call made while that device is current)
// and that address is what the kernels receive.
#include <mutex>
#include "common.cuh"
#include "../../include/vx27_gqa.h"

namespace vx27 {
int gqa_plan_splits(int B, int nkv, int cap, int n_splits, int fit, int flags);
int gqa_decode_dispatch(const float *q, const void *gate, const void *k_cache,
                        const void *v_cache, int cap, const int *pos, void *out, float *parts,
                        int B, int nq, int nkv, int n_splits, int flags, cudaStream_t st,
                        char *err, size_t errlen);
}  // namespace vx27

namespace {

// Partial records of every split of every call; shared by all calls on a device.
static __device__ __align__(256) unsigned char g_gqa_scratch[VX27_GQA_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;  // guards addr[] below: several host threads may make first calls

// Device address of g_gqa_scratch on the current device, looked up on first use.
float *scratch_on_current_device(char *err, size_t errlen) {
    static void *addr[kMaxDevices] = {};
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess)
        return (vx27::check_cuda(e, "vx27_gqa_decode_batch_noalloc: cudaGetDevice", err, errlen),
                nullptr);
    if (dev < 0 || dev >= kMaxDevices)
        return (vx27::fail(err, errlen, "vx27_gqa_decode_batch_noalloc: device %d out of range",
                           dev), nullptr);
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!addr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_gqa_scratch);
        if (e != cudaSuccess || !p)
            return (vx27::check_cuda(e, "vx27_gqa_decode_batch_noalloc: cudaGetSymbolAddress",
                                     err, errlen), nullptr);
        addr[dev] = p;
    }
    return (float *)addr[dev];
}

}  // namespace

extern "C" int vx27_gqa_decode_batch_noalloc(const float *q, const void *gate,
                                             const void *k_cache, const void *v_cache, int cap,
                                             const int *pos, void *out, int B, int nq, int nkv,
                                             int hd, int n_splits, int flags, void *stream,
                                             char *err, size_t errlen) {
    using namespace vx27;
    const char *fn = "vx27_gqa_decode_batch_noalloc";
    if (hd != 256) return fail(err, errlen, "%s: hd=%d unsupported (256 only)", fn, hd);
    if (B <= 0 || B > 65535 || nq <= 0 || nkv <= 0 || nkv > 65535 || nq % nkv)
        return fail(err, errlen, "%s: bad shape B=%d nq=%d nkv=%d", fn, B, nq, nkv);
    if (!q || !k_cache || !v_cache || !pos || !out || cap <= 0)
        return fail(err, errlen, "%s: null pointer argument", fn);
    const size_t record = (size_t)B * nq * (hd + 2) * sizeof(float);
    const int fit = (int)((size_t)VX27_GQA_NOALLOC_SCRATCH_BYTES / record);
    if (fit < 1)
        return fail(err, errlen,
                    "%s: one partial record needs %zu bytes, more than the %u-byte static "
                    "scratch (B*nq*(hd+2)*4 must be <= %u)",
                    fn, record, (unsigned)VX27_GQA_NOALLOC_SCRATCH_BYTES,
                    (unsigned)VX27_GQA_NOALLOC_SCRATCH_BYTES);
    if (n_splits <= 0) {  // the workspace entry point's choice, capped by the array
        n_splits = gqa_plan_splits(B, nkv, cap, 0, fit, flags);
    } else if (n_splits > fit || n_splits > 65535) {
        return fail(err, errlen,
                    "%s: %d splits need %zu bytes of partial records, more than the %u-byte "
                    "static scratch (at most %d splits for this batch)",
                    fn, n_splits, record * n_splits, (unsigned)VX27_GQA_NOALLOC_SCRATCH_BYTES,
                    fit);
    }
    float *parts = scratch_on_current_device(err, errlen);
    if (!parts) return -1;
    // The same kernels as vx27_gqa_decode_batch. Every record the combine reads is written
    // by the split kernel first (empty ranges write a neutral record), so nothing left from
    // an earlier call needs clearing. With one split the kernel writes the gated output
    // itself.
    return gqa_decode_dispatch(q, gate, k_cache, v_cache, cap, pos, out, parts, B, nq, nkv,
                               n_splits, flags, (cudaStream_t)stream, err, errlen);
}
