/*
 * libvx27cuda -- B200 (sm_100a) implementation of the vx27 attention hot path.
 *
 * Library-wide definitions shared by vx27_deltanet.h, vx27_gqa.h, vx27_kv.h and
 * vx27_rope.h. The reference (DavidPandleton/vx27) has no counterpart for this header:
 * its hot-path functions return void and report nothing (src/vx27_deltanet.h:10-59).
 *
 * Two tiers share this library:
 *  - the reference entry points, same names and signatures, host pointers, synchronous
 *    (copy in, run on the GPU, copy out). They cannot return a status; on a CUDA error
 *    they print the error and abort the process, unless VX27CUDA_NO_ABORT=1 is set, in
 *    which case the outputs are left untouched and vx27cuda_last_error() tells why;
 *  - the batched, device-resident entry points (vx27_*_batch, vx27_gqa_*, vx27_kv_*):
 *    device pointers, a CUDA stream passed as void*, and an int status (0 = ok,
 *    -1 = error, message copied into err[errlen] when err is not NULL). They enqueue
 *    work on the stream and return without synchronising.
 */
#ifndef VX27CUDA_H
#define VX27CUDA_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Flags of the batched entry points. */
#define VX27_F_ACT_BF16  0x1 /* activations (qkv, a, b, q, k, v, gate) are bf16, else fp32 */
#define VX27_F_OUT_BF16  0x2 /* outputs are bf16, else fp32 */
#define VX27_F_NORM_1P   0x4 /* zero-centred RMSNorm weights: y = x*s*(1+w) */
#define VX27_F_GATES_F64 0x8 /* DeltaNet: a/b hold host-computed beta/g_log as double */
/* DeltaNet decode: the kernel may start reading this layer's state S while the kernel
 * before it on the stream is still running (programmatic dependent launch). Set it only
 * when that kernel does not write S, e.g. when it belongs to another layer; everything
 * else the kernel reads still waits for the previous kernel to finish. */
#define VX27_F_PREFETCH_STATE 0x10
/* DeltaNet decode, gated entry point: the production layer's q/k pre-normalisation
 * (src/vx27_qfwd.c:118-130): zero-centred RMSNorm with norm_w, y = x*s*(1+w), then l2norm
 * and q*1/sqrt(hd), before the l2norm and scaling the delta rule itself applies. */
#define VX27_F_QK_PRENORM 0x20
/* GQA decode (vx27_gqa_decode_batch, vx27_gqa_decode_fused): the kernel may request cache
 * rows below the token's slot, and read pos, while the kernel before it on the stream is
 * still running (programmatic dependent launch). Set it only when that kernel writes
 * neither pos nor any cache row other than row pos[b] (e.g. vx27_gqa_append for the same
 * layer, or another layer's kernel); honoured by the CUDA-core decode. */
#define VX27_F_PREFETCH_KV 0x40
/* GQA decode: which kernel runs the attention. Default (and VX27_F_DECODE_TC): the
 * tensor-core (tcgen05) split-KV kernel. VX27_F_DECODE_CC: a split-KV kernel on the CUDA
 * cores (fp32 FMA), slower on a B200 at every batch shape measured; it is kept as the
 * reference point for that comparison. vx27_gqa_decode_plan reports the choice. */
#define VX27_F_DECODE_CC 0x80
#define VX27_F_DECODE_TC 0x100
/* GQA prefill: one CTA per (query tile, query head) on one SM. By default, when the query
 * heads per KV head are even, two neighbouring heads run as a 2-CTA cluster whose
 * tcgen05 MMAs span both SMs, each SM loading half of every K/V tile. */
#define VX27_F_PREFILL_CTA1 0x200

/* Library version, major*10000 + minor*100 + patch. */
int vx27cuda_version(void);
/* Last error message recorded on the calling thread ("" if none). */
const char *vx27cuda_last_error(void);
/* Reads (and optionally clears) the device status word that bounded device-side waits
 * set when they time out: 0 ok, 1 TMA wait timeout, 2 MMA wait timeout, 3 bad argument
 * seen on the device. Synchronises the stream. */
int vx27cuda_device_status(void *stream, uint32_t *status, int clear, char *err,
                           size_t errlen);
/* Number of streaming multiprocessors of the current device. */
int vx27cuda_num_sms(void);

/* Seeded synthetic inputs on the device: element i of (seed, stream_id) is the same
 * splitmix64 + Box-Muller value on every device and every call; dst[e] receives element
 * offset + e; bf16 != 0 writes bf16 (round to nearest even), else fp32. */
int vx27cuda_fill_normal(void *dst, size_t n, int bf16, uint64_t seed, uint64_t stream_id,
                         uint64_t offset, float mean, float stddev, void *stream, char *err,
                         size_t errlen);
int vx27cuda_fill_uniform(float *dst, size_t n, uint64_t seed, uint64_t stream_id, float lo,
                          float hi, void *stream, char *err, size_t errlen);
/* Sets n ints to value (positions arrays); adds delta to n ints. */
int vx27cuda_fill_int(int *dst, size_t n, int value, void *stream, char *err, size_t errlen);
int vx27cuda_add_int(int *dst, size_t n, int delta, void *stream, char *err, size_t errlen);

#ifdef __cplusplus
}
#endif
#endif
