// Library runtime: status plumbing, device status word, seeded synthetic inputs,
// RoPE table upload, the device KV cache object and DeltaNet conv-history conversion.
#include <stdarg.h>
#include <stdlib.h>
#include <string.h>
#include <mutex>
#include <vector>
#include "common.cuh"
#include "../../include/vx27_deltanet.h"
#include "../../include/vx27_gqa.h"
#include "../../include/vx27_kv.h"
#include "../../include/vx27_rope.h"

namespace vx27 {

static std::mutex g_rt_mu;  // guards the per-device caches below

// The status word lives in the module's own global memory (zero at module load), one per
// device, so reading its address allocates nothing: entry points that must not allocate
// report their timeouts here too.
static __device__ uint32_t g_dev_status;

uint32_t *dev_status() {
    static uint32_t *ptrs[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(g_rt_mu);
    if (!ptrs[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_dev_status) != cudaSuccess || !p) return nullptr;
        ptrs[dev] = (uint32_t *)p;
    }
    return ptrs[dev];
}

static thread_local char t_last_error[512] = "";

int fail(char *err, size_t errlen, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_last_error, sizeof t_last_error, fmt, ap);
    va_end(ap);
    if (err && errlen) snprintf(err, errlen, "%s", t_last_error);
    return -1;
}

int check_cuda(cudaError_t e, const char *what, char *err, size_t errlen) {
    return fail(err, errlen, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

void compat_fail(const char *fn, const char *msg) {
    snprintf(t_last_error, sizeof t_last_error, "%s: %s", fn, msg);
    fprintf(stderr, "libvx27cuda: %s\n", t_last_error);
    const char *na = getenv("VX27CUDA_NO_ABORT");
    if (!(na && na[0] == '1')) abort();
}

// The dynamic shared-memory limit of a kernel is a per-device attribute: set it once per
// (kernel, device, size) and remember that, so a process driving several GPUs (or
// several host threads) launches correctly on each.
int ensure_smem_attr(const void *kernel, size_t bytes, char *err, size_t errlen) {
    struct Done { const void *k; int dev; size_t bytes; };
    static std::vector<Done> done;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return check_cuda(e, "cudaGetDevice", err, errlen);
    std::lock_guard<std::mutex> lock(g_rt_mu);
    for (const Done &d : done)
        if (d.k == kernel && d.dev == dev && d.bytes >= bytes) return 0;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e != cudaSuccess) return check_cuda(e, "cudaFuncSetAttribute", err, errlen);
    done.push_back({kernel, dev, bytes});
    return 0;
}

int num_sms() {
    static int cached[64] = {};
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    std::lock_guard<std::mutex> lock(g_rt_mu);
    if (!cached[dev]) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            return 148;
        cached[dev] = n;
    }
    return cached[dev];
}

// ---- synthetic inputs: same formula as oracle/vx27_oracle.c (splitmix64 + Box-Muller)
__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}
static uint64_t stream_key(uint64_t seed, uint64_t stream) {
    return splitmix64(splitmix64(seed) ^ (stream * 0xD1B54A32D192ED03ull));
}
__global__ void fill_normal_k(void *dst, size_t n, int bf16, uint64_t key, float mean,
                              float stddev, uint64_t offset) {
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < n;
         e += (size_t)gridDim.x * blockDim.x) {
        const uint64_t i = e + offset;  // element index within the stream
        const uint64_t j = i >> 1;
        const uint64_t r1 = splitmix64(key + 2 * j), r2 = splitmix64(key + 2 * j + 1);
        const double u1 = (double)((r1 >> 11) + 1) * 0x1.0p-53;
        const double u2 = (double)(r2 >> 11) * 0x1.0p-53;
        const double rad = sqrt(-2.0 * log(u1));
        const double th = 6.283185307179586 * u2;
        const double z = (i & 1) ? rad * sin(th) : rad * cos(th);
        const float x = (float)((double)mean + (double)stddev * z);
        if (bf16) ((uint16_t *)dst)[e] = f32_to_bf16(x);
        else ((float *)dst)[e] = x;
    }
}
__global__ void fill_uniform_k(float *dst, size_t n, uint64_t key, float lo, float hi) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        const double u = (double)(splitmix64(key + i) >> 11) * 0x1.0p-53;
        dst[i] = (float)((double)lo + ((double)hi - (double)lo) * u);
    }
}
__global__ void fill_int_k(int *dst, size_t n, int value, int add) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        dst[i] = add ? dst[i] + value : value;
}
static int grid_for(size_t n) {
    size_t g = (n + 255) / 256;
    size_t cap = (size_t)num_sms() * 8;
    return (int)(g < 1 ? 1 : (g > cap ? cap : g));
}

// ---- conv history ring <-> reference state
__global__ void conv_import_k(float *ring, const float *state, const int *pos, int B, int C) {
    const int b = blockIdx.y;
    const int t = pos[b];
    for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < C; c += gridDim.x * blockDim.x) {
        const float *s = state + ((size_t)b * C + c) * 3;
        float *r = ring + (size_t)b * 4 * C;
        r[(size_t)((t - 3) & 3) * C + c] = s[0];
        r[(size_t)((t - 2) & 3) * C + c] = s[1];
        r[(size_t)((t - 1) & 3) * C + c] = s[2];
        r[(size_t)(t & 3) * C + c] = 0.0f;
    }
}
__global__ void conv_export_k(const float *ring, float *state, const int *pos, int B, int C) {
    const int b = blockIdx.y;
    const int t = pos[b];
    for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < C; c += gridDim.x * blockDim.x) {
        float *s = state + ((size_t)b * C + c) * 3;
        const float *r = ring + (size_t)b * 4 * C;
        s[0] = r[(size_t)((t - 3) & 3) * C + c];
        s[1] = r[(size_t)((t - 2) & 3) * C + c];
        s[2] = r[(size_t)((t - 1) & 3) * C + c];
    }
}

__global__ void kv_store_k(uint16_t *k, uint16_t *v, const float *kh, const float *vh, int n,
                           int nkv, int hd, int cap) {
    // kh/vh [n][nkv][hd] -> planes [nkv][cap][hd] (already offset to sequence and p0)
    const size_t total = (size_t)n * nkv * hd;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        const int d = (int)(i % hd);
        const int h = (int)((i / hd) % nkv);
        const int p = (int)(i / ((size_t)hd * nkv));
        const size_t o = ((size_t)h * cap + p) * hd + d;
        k[o] = f32_to_bf16(kh[i]);
        v[o] = f32_to_bf16(vh[i]);
    }
}
__global__ void kv_load_k(const uint16_t *k, const uint16_t *v, float *kh, float *vh, int n,
                          int nkv, int hd, int cap) {
    const size_t total = (size_t)n * nkv * hd;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        const int d = (int)(i % hd);
        const int h = (int)((i / hd) % nkv);
        const int p = (int)(i / ((size_t)hd * nkv));
        const size_t o = ((size_t)h * cap + p) * hd + d;
        kh[i] = bf16_to_f32(k[o]);
        vh[i] = bf16_to_f32(v[o]);
    }
}

}  // namespace vx27

using namespace vx27;

struct vx27_kv_cache {
    int n_layers, batch, n_kv, hd, cap;
    uint16_t *base;  // [layer][2][batch][n_kv][cap][hd]
};

extern "C" {

int vx27cuda_version(void) { return 100; }

const char *vx27cuda_last_error(void) { return t_last_error; }

int vx27cuda_num_sms(void) { return num_sms(); }

int vx27cuda_device_status(void *stream, uint32_t *status, int clear, char *err,
                           size_t errlen) {
    cudaStream_t s = (cudaStream_t)stream;
    uint32_t v = 0, *d = dev_status();
    if (!d) return fail(err, errlen, "vx27cuda_device_status: no device status word");
    VX_CK(cudaMemcpyAsync(&v, d, sizeof v, cudaMemcpyDeviceToHost, s));
    VX_CK(cudaStreamSynchronize(s));
    if (clear) {
        VX_CK(cudaMemsetAsync(d, 0, sizeof v, s));
        VX_CK(cudaStreamSynchronize(s));
    }
    if (status) *status = v;
    return 0;
}

int vx27cuda_fill_normal(void *dst, size_t n, int bf16, uint64_t seed, uint64_t stream_id,
                         uint64_t offset, float mean, float stddev, void *stream, char *err,
                         size_t errlen) {
    if (n == 0) return 0;
    if (!dst) return fail(err, errlen, "vx27cuda_fill_normal: null destination");
    fill_normal_k<<<grid_for(n), 256, 0, (cudaStream_t)stream>>>(
        dst, n, bf16, stream_key(seed, stream_id), mean, stddev, offset);
    VX_CK(cudaGetLastError());
    return 0;
}

int vx27cuda_fill_uniform(float *dst, size_t n, uint64_t seed, uint64_t stream_id, float lo,
                          float hi, void *stream, char *err, size_t errlen) {
    if (n == 0) return 0;
    if (!dst) return fail(err, errlen, "vx27cuda_fill_uniform: null destination");
    fill_uniform_k<<<grid_for(n), 256, 0, (cudaStream_t)stream>>>(
        dst, n, stream_key(seed, stream_id), lo, hi);
    VX_CK(cudaGetLastError());
    return 0;
}

int vx27cuda_fill_int(int *dst, size_t n, int value, void *stream, char *err, size_t errlen) {
    if (n == 0) return 0;
    fill_int_k<<<grid_for(n), 256, 0, (cudaStream_t)stream>>>(dst, n, value, 0);
    VX_CK(cudaGetLastError());
    return 0;
}

int vx27cuda_add_int(int *dst, size_t n, int delta, void *stream, char *err, size_t errlen) {
    if (n == 0) return 0;
    fill_int_k<<<grid_for(n), 256, 0, (cudaStream_t)stream>>>(dst, n, delta, 1);
    VX_CK(cudaGetLastError());
    return 0;
}

int vx27_rope_table_build(float *table_dev, int n_pos, int rope_dim, float theta,
                          float yarn_factor, char *err, size_t errlen) {
    if (n_pos <= 0 || rope_dim <= 0 || (rope_dim & 1) || rope_dim > 256 || !table_dev)
        return fail(err, errlen, "vx27_rope_table_build: bad arguments (n_pos=%d rope_dim=%d)",
                    n_pos, rope_dim);
    const int half = rope_dim / 2;
    std::vector<float> tab((size_t)n_pos * rope_dim);
    for (int p = 0; p < n_pos; p++) {
        float *row = tab.data() + (size_t)p * rope_dim;
        vx27_rope_cos_sin(p, row, row + half, rope_dim, theta, yarn_factor);
    }
    VX_CK(cudaMemcpy(table_dev, tab.data(), tab.size() * sizeof(float), cudaMemcpyHostToDevice));
    return 0;
}

int vx27_deltanet_conv_import(float *conv_ring, const float *state, const int *pos, int B,
                              int C, void *stream, char *err, size_t errlen) {
    if (B <= 0 || C <= 0) return fail(err, errlen, "vx27_deltanet_conv_import: B=%d C=%d", B, C);
    cudaStream_t s = (cudaStream_t)stream;
    float *d_state = nullptr;
    int *d_pos = nullptr;
    VX_CK(cudaMallocAsync((void **)&d_state, (size_t)B * C * 3 * sizeof(float), s));
    VX_CK(cudaMallocAsync((void **)&d_pos, (size_t)B * sizeof(int), s));
    VX_CK(cudaMemcpyAsync(d_state, state, (size_t)B * C * 3 * sizeof(float),
                          cudaMemcpyHostToDevice, s));
    VX_CK(cudaMemcpyAsync(d_pos, pos, (size_t)B * sizeof(int), cudaMemcpyHostToDevice, s));
    conv_import_k<<<dim3((C + 255) / 256, B), 256, 0, s>>>(conv_ring, d_state, d_pos, B, C);
    VX_CK(cudaGetLastError());
    VX_CK(cudaFreeAsync(d_state, s));
    VX_CK(cudaFreeAsync(d_pos, s));
    VX_CK(cudaStreamSynchronize(s));
    return 0;
}

int vx27_deltanet_conv_export(const float *conv_ring, float *state, const int *pos, int B,
                              int C, void *stream, char *err, size_t errlen) {
    if (B <= 0 || C <= 0) return fail(err, errlen, "vx27_deltanet_conv_export: B=%d C=%d", B, C);
    cudaStream_t s = (cudaStream_t)stream;
    float *d_state = nullptr;
    int *d_pos = nullptr;
    VX_CK(cudaMallocAsync((void **)&d_state, (size_t)B * C * 3 * sizeof(float), s));
    VX_CK(cudaMallocAsync((void **)&d_pos, (size_t)B * sizeof(int), s));
    VX_CK(cudaMemcpyAsync(d_pos, pos, (size_t)B * sizeof(int), cudaMemcpyHostToDevice, s));
    conv_export_k<<<dim3((C + 255) / 256, B), 256, 0, s>>>(conv_ring, d_state, d_pos, B, C);
    VX_CK(cudaGetLastError());
    VX_CK(cudaMemcpyAsync(state, d_state, (size_t)B * C * 3 * sizeof(float),
                          cudaMemcpyDeviceToHost, s));
    VX_CK(cudaFreeAsync(d_state, s));
    VX_CK(cudaFreeAsync(d_pos, s));
    VX_CK(cudaStreamSynchronize(s));
    return 0;
}

size_t vx27_kv_bytes(int n_layers, int batch, int n_kv, int hd, int capacity) {
    return (size_t)n_layers * 2 * batch * n_kv * (size_t)capacity * hd * sizeof(uint16_t);
}

int vx27_kv_create(vx27_kv_cache **kv, int n_layers, int batch, int n_kv, int hd,
                   int capacity, char *err, size_t errlen) {
    if (!kv || n_layers <= 0 || batch <= 0 || n_kv <= 0 || hd <= 0 || capacity <= 0 ||
        (hd % 8))
        return fail(err, errlen, "vx27_kv_create: bad arguments");
    vx27_kv_cache *c = (vx27_kv_cache *)calloc(1, sizeof *c);
    if (!c) return fail(err, errlen, "vx27_kv_create: out of host memory");
    c->n_layers = n_layers; c->batch = batch; c->n_kv = n_kv; c->hd = hd; c->cap = capacity;
    const size_t bytes = vx27_kv_bytes(n_layers, batch, n_kv, hd, capacity);
    cudaError_t e = cudaMalloc((void **)&c->base, bytes);
    if (e != cudaSuccess) {
        free(c);
        return check_cuda(e, "vx27_kv_create: cudaMalloc", err, errlen);
    }
    e = cudaMemset(c->base, 0, bytes);
    if (e != cudaSuccess) {
        cudaFree(c->base);
        free(c);
        return check_cuda(e, "vx27_kv_create: cudaMemset", err, errlen);
    }
    *kv = c;
    return 0;
}

void vx27_kv_destroy(vx27_kv_cache *kv) {
    if (!kv) return;
    cudaFree(kv->base);
    free(kv);
}

int vx27_kv_capacity(const vx27_kv_cache *kv) { return kv ? kv->cap : 0; }

int vx27_kv_layer(const vx27_kv_cache *kv, int layer, void **k, void **v) {
    if (!kv || layer < 0 || layer >= kv->n_layers)
        return fail(nullptr, 0, "vx27_kv_layer: bad layer %d", layer);
    const size_t plane = (size_t)kv->batch * kv->n_kv * kv->cap * kv->hd;
    if (k) *k = kv->base + (size_t)layer * 2 * plane;
    if (v) *v = kv->base + (size_t)layer * 2 * plane + plane;
    return 0;
}

static int kv_xfer(const vx27_kv_cache *kv, int layer, int seq, int p0, int n, const float *kin,
                   const float *vin, float *kout, float *vout, char *err, size_t errlen) {
    if (!kv || layer < 0 || layer >= kv->n_layers || seq < 0 || seq >= kv->batch || p0 < 0 ||
        n < 0 || p0 + n > kv->cap)
        return fail(err, errlen, "vx27_kv: bad range (layer %d seq %d p0 %d n %d)", layer, seq,
                    p0, n);
    if (n == 0) return 0;
    void *kp, *vp;
    vx27_kv_layer(kv, layer, &kp, &vp);
    const size_t off = ((size_t)seq * kv->n_kv * kv->cap + p0) * kv->hd;
    uint16_t *K = (uint16_t *)kp + off, *V = (uint16_t *)vp + off;
    const size_t cnt = (size_t)n * kv->n_kv * kv->hd;
    float *dk = nullptr, *dv = nullptr;
    VX_CK(cudaMalloc((void **)&dk, cnt * sizeof(float)));
    cudaError_t e = cudaMalloc((void **)&dv, cnt * sizeof(float));
    if (e != cudaSuccess) { cudaFree(dk); return check_cuda(e, "cudaMalloc", err, errlen); }
    int rc = 0;
    if (kin) {
        e = cudaMemcpy(dk, kin, cnt * 4, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(dv, vin, cnt * 4, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) {
            kv_store_k<<<grid_for(cnt), 256>>>(K, V, dk, dv, n, kv->n_kv, kv->hd, kv->cap);
            e = cudaGetLastError();
        }
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
    } else {
        kv_load_k<<<grid_for(cnt), 256>>>(K, V, dk, dv, n, kv->n_kv, kv->hd, kv->cap);
        e = cudaGetLastError();
        if (e == cudaSuccess) e = cudaMemcpy(kout, dk, cnt * 4, cudaMemcpyDeviceToHost);
        if (e == cudaSuccess) e = cudaMemcpy(vout, dv, cnt * 4, cudaMemcpyDeviceToHost);
    }
    if (e != cudaSuccess) rc = check_cuda(e, "vx27_kv transfer", err, errlen);
    cudaFree(dk);
    cudaFree(dv);
    return rc;
}

int vx27_kv_store_f32(vx27_kv_cache *kv, int layer, int seq, int p0, int n,
                      const float *k_host, const float *v_host, char *err, size_t errlen) {
    if (!k_host || !v_host) return fail(err, errlen, "vx27_kv_store_f32: null input");
    return kv_xfer(kv, layer, seq, p0, n, k_host, v_host, nullptr, nullptr, err, errlen);
}

int vx27_kv_load_f32(const vx27_kv_cache *kv, int layer, int seq, int p0, int n,
                     float *k_host, float *v_host, char *err, size_t errlen) {
    if (!k_host || !v_host) return fail(err, errlen, "vx27_kv_load_f32: null output");
    return kv_xfer(kv, layer, seq, p0, n, nullptr, nullptr, k_host, v_host, err, errlen);
}

}  // extern "C"
