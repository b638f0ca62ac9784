/*
 * Partial RoPE (NeoX half-split) for the full-attention layers (libvx27cuda).
 * Drop-in for src/vx27_rope.h of DavidPandleton/vx27, plus a device table builder.
 */
#ifndef VX27_ROPE_H
#define VX27_ROPE_H
#include <stddef.h>
#include "vx27cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------- reference entry points (src/vx27_rope.h) ---------------------- */
/* cos/sin of (pos/yarn) * theta^(-2i/rope_dim), i < rope_dim/2, float libm on the host:
 * bit-identical to the reference. Replaces src/vx27_rope.h:11-12. */
void vx27_rope_cos_sin(int pos, float *cosv, float *sinv, int rope_dim, float theta,
                       float yarn_factor);
/* Rotation of the first rope_dim dims of each head, rest passthrough; on the GPU, with
 * the reference's rounding (no fused multiply-add). Replaces src/vx27_rope.h:14-15. */
void vx27_rope_apply(float *v, int n_heads, int head_dim, int rope_dim, const float *cosv,
                     const float *sinv);
/* Text-only M-RoPE = standard RoPE at (pos, 64, 1e7). Replaces src/vx27_rope.h:17. */
void vx27_mrope_cos_sin_text(int pos, float *cosv, float *sinv);

/* ---------------- device table (no reference counterpart) ------------------------ */
/* table_dev [n_pos][rope_dim] fp32: row p = cos[0..rope_dim/2) then sin[0..rope_dim/2)
 * of vx27_rope_cos_sin(p, ..., theta, yarn_factor), computed on the host and copied, so
 * device positions see the reference's exact values. Synchronous. */
int vx27_rope_table_build(float *table_dev, int n_pos, int rope_dim, float theta,
                          float yarn_factor, char *err, size_t errlen);

#ifdef __cplusplus
}
#endif
#endif
