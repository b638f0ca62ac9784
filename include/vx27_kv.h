/*
 * BF16 KV cache for the 16 full-attention layers (libvx27cuda). Drop-in for
 * src/vx27_kv.h of DavidPandleton/vx27 (sizing, first block) plus the cache storage the
 * reference lacks (second block): its decode path keeps an fp32 cache inline in
 * src/vx27_qfwd.c:183-185 with no storage API.
 */
#ifndef VX27_KV_H
#define VX27_KV_H
#include <stddef.h>
#include <stdint.h>
#include "vx27cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------- reference entry points (src/vx27_kv.h) ------------------------ */
/* 16 layers * 2 * 4 * 256 = 32768 elements per token. Replaces src/vx27_kv.h:7-9. */
uint64_t vx27_kv_elems(int ctx);
double vx27_kv_gb(int ctx, double bytes_per_elem);
int vx27_kv_fits(int ctx, double bytes_per_elem, double budget_gb);

/* ---------------- device cache (no reference counterpart) ------------------------ */
/* Device layout per layer: K and V planes, each bf16 [batch][n_kv][capacity][hd], so
 * one (sequence, KV head) is a contiguous run of positions (1-D bulk-copy friendly). */
typedef struct vx27_kv_cache vx27_kv_cache;

size_t vx27_kv_bytes(int n_layers, int batch, int n_kv, int hd, int capacity);
int vx27_kv_create(vx27_kv_cache **kv, int n_layers, int batch, int n_kv, int hd,
                   int capacity, char *err, size_t errlen);
void vx27_kv_destroy(vx27_kv_cache *kv);
/* Device pointers of one layer's K and V planes. */
int vx27_kv_layer(const vx27_kv_cache *kv, int layer, void **k, void **v);
int vx27_kv_capacity(const vx27_kv_cache *kv);
/* Host fp32 rows in the reference's cache order [n][n_kv][hd] (src/vx27_qfwd.c:183)
 * to/from positions [p0, p0+n) of one sequence; stores round to bf16 (nearest even).
 * Synchronous. These are the checkpoint import/export of the cache. */
int vx27_kv_store_f32(vx27_kv_cache *kv, int layer, int seq, int p0, int n,
                      const float *k_host, const float *v_host, char *err, size_t errlen);
int vx27_kv_load_f32(const vx27_kv_cache *kv, int layer, int seq, int p0, int n,
                     float *k_host, float *v_host, char *err, size_t errlen);

#ifdef __cplusplus
}
#endif
#endif
