// vx27_gqa_decode_batch_noalloc: the split-KV GQA decode of vx27_gqa_decode_batch for
// callers that have no device workspace to give and must not have this library
// allocate one. Its partial (m, l, o) records live in a fixed array in the module's own
// global memory instead of a caller workspace or a cudaMalloc.
//
// The array below is reserved on every GPU that loads this library and stays reserved
// until the process exits. In host code its name is only a host-side stand-in for the
// device symbol, so the device address is looked up once per device with
// cudaGetSymbolAddress (on the first call made while that device is current) and that
// address is what the kernels receive.
#include "common.cuh"
#include "../../include/vx27_gqa.h"

namespace vx27 {
int launch_split_tc_status(const void *kc, const void *vc, const float *q, const int *pos,
                           float *parts, int cap, int B, int nq, int nkv, int n_splits,
                           uint32_t *status, cudaStream_t st, char *err, size_t errlen);
int launch_gqa_combine(const float *parts, int n_parts, const void *gate, void *out, int B,
                       int nq, int flags, cudaStream_t st, char *err, size_t errlen);
}  // namespace vx27

namespace {

// Partial records of every split of every call; shared by all calls on a device.
static __device__ __align__(256) unsigned char g_gqa_scratch[VX27_GQA_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
constexpr int kTile = 128;  // split boundaries fall on multiples of 128 cache slots

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
    if (n_splits <= 0) {
        const int blocks = B * nkv;
        n_splits = (2 * num_sms() + blocks - 1) / blocks;
        const int by_ctx = (cap + kTile - 1) / kTile;
        if (n_splits > by_ctx) n_splits = by_ctx;
        if (n_splits > 128) n_splits = 128;
        if (n_splits > fit) n_splits = fit;
        if (n_splits < 1) n_splits = 1;
    } else if (n_splits > fit || n_splits > 65535) {
        return fail(err, errlen,
                    "%s: %d splits need %zu bytes of partial records, more than the %u-byte "
                    "static scratch (at most %d splits for this batch)",
                    fn, n_splits, record * n_splits, (unsigned)VX27_GQA_NOALLOC_SCRATCH_BYTES,
                    fit);
    }
    float *parts = scratch_on_current_device(err, errlen);
    if (!parts) return -1;
    // Every record the combine reads is written by the split kernel first (empty ranges
    // write a neutral record), so nothing left from an earlier call needs clearing.
    cudaStream_t st = (cudaStream_t)stream;
    if (launch_split_tc_status(k_cache, v_cache, q, pos, parts, cap, B, nq, nkv, n_splits,
                               nullptr, st, err, errlen))
        return -1;
    return launch_gqa_combine(parts, n_splits, gate, out, B, nq, flags, st, err, errlen);
}
