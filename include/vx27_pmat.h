/*
 * vx27_pmat.h -- the packed-weight matvec of the layer projections, device-resident.
 *
 * Replaces, for device-resident callers, src/vx27_pmat.h:12-20 of the reference
 * (vx27_pmat: one vector; vx27_pmat_batch: B <= 8 vectors in one pass over the
 * weights). The projections around the two attention layers use it: in_proj_qkv / z /
 * a / b and out_proj of a DeltaNet layer, q_proj (query and gate interleaved per head),
 * k_proj, v_proj and o_proj of a GQA layer (src/vx27_qfwd.c:102-213).
 *
 * Weights stay packed in the reference's in-memory layouts, row-major [rows][row_bytes]:
 *   VX27_PMAT_F32      float[cols]
 *   VX27_PMAT_Q8_K     cols/256 blocks of {float d; int8 qs[256]; int16 bsums[16]} (292 B)
 *   VX27_PMAT_BP3_128  cols/128 groups of {uint32 planes[12]; uint16 fp16 scale} (52 B,
 *                      including 2 B of padding; code bit b of column i of the group is
 *                      bit i%32 of planes[4b + i/32]; the 3-bit code is two's complement)
 * Results are bit-identical to the reference's vx27_pmat / vx27_pmat_batch, for any B.
 */
#ifndef VX27_PMAT_DEV_H
#define VX27_PMAT_DEV_H
#include <stddef.h>
#include <stdint.h>
#include "vx27cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

#define VX27_PMAT_F32     0u
#define VX27_PMAT_Q8_K    2u
#define VX27_PMAT_BP3_128 4u

/* Bytes of one packed row of cols columns (0 for an unknown dtype). */
size_t vx27_pmat_row_bytes(uint32_t dtype, int cols);

/*
 * yb[b*rows + r] = sum_c W[r][c] * xb[b*cols + c] for r < rows, b < B (device pointers).
 * cols: a multiple of 256 for Q8_K, of 128 for BP3_128. W 4-byte aligned (BP3_128:
 * 16-byte); xb 16-byte aligned for Q8_K and BP3_128. Asynchronous on stream.
 */
int vx27_pmat_batch_dev(const void *W, uint32_t dtype, const float *xb, float *yb, int rows,
                        int cols, int B, void *stream, char *err, size_t errlen);

#define VX27_PMAT_MAX_GROUPS 4

/*
 * n (1..VX27_PMAT_MAX_GROUPS) projections of the same inputs in one launch, e.g. a
 * DeltaNet layer's in_proj_qkv / z / a / b: for each i < n, yb[i][b*rows[i] + r] =
 * W[i][r] . xb[b] with the same dtype and cols (host arrays of device pointers; each
 * output as vx27_pmat_batch_dev writes it, bit-identical to the reference's vx27_pmat).
 */
int vx27_pmat_multi_dev(int n, const void *const *W, uint32_t dtype, const float *xb,
                        float *const *yb, const int *rows, int cols, int B, void *stream,
                        char *err, size_t errlen);

#ifdef __cplusplus
}
#endif
#endif
