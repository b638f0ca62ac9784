/*
 * Host-side entry points of libvx27cuda whose work is O(1) scalar arithmetic that the
 * reference contract requires to be bit-identical: sizing, the gate mapping, the GQA
 * head map, KV sizing and the RoPE cos/sin tables. They use the same C library
 * functions in the same order as the reference, compiled as ISO C11 without
 * floating-point contraction, so they return the reference's exact bits.
 * Everything that touches tensors runs on the GPU (compat.cu and the batched tier).
 */
#include <math.h>
#include <stdint.h>
#include "../../include/vx27_deltanet.h"
#include "../../include/vx27_gqa.h"
#include "../../include/vx27_kv.h"
#include "../../include/vx27_rope.h"

/* Model constants of the locked target (src/vx27_config.h:14-25, :51). */
enum { QK_HEADS = 16, LIN_HD = 128, N_LINEAR = 48, ATT_Q = 24, ATT_KV = 4 };

/* src/vx27_deltanet.c:5-13 */
int vx27_deltanet_state_per_layer(void) { return QK_HEADS * LIN_HD * LIN_HD; }
int vx27_deltanet_state_total(void) { return vx27_deltanet_state_per_layer() * N_LINEAR; }
double vx27_deltanet_state_mb(int bytes_per_elem) {
    return (double)vx27_deltanet_state_total() * bytes_per_elem / 1e6;
}

/* src/vx27_deltanet.c:58-69: softplus with linear / exponential tails at |x| > 20 */
static double softplus_ref(double x) {
    if (x > 20.0) return x;
    if (x < -20.0) return exp(x);
    return log(1.0 + exp(x));
}
void vx27_deltanet_gate_params(double a, double A_log, double b, double dt_bias,
                               double *beta, double *g_log) {
    if (beta) *beta = 1.0 / (1.0 + exp(-b));
    if (g_log) *g_log = -exp(A_log) * softplus_ref(a + dt_bias);
}

/* src/vx27_gqa.c:6-8 */
int vx27_gqa_kv_for_q(int q_head) { return q_head * ATT_KV / ATT_Q; }

/* src/vx27_kv.c:4-12 */
uint64_t vx27_kv_elems(int ctx) { return (uint64_t)32768 * (uint64_t)ctx; }
double vx27_kv_gb(int ctx, double bytes_per_elem) {
    return (double)vx27_kv_elems(ctx) * bytes_per_elem / 1e9;
}
int vx27_kv_fits(int ctx, double bytes_per_elem, double budget_gb) {
    return vx27_kv_gb(ctx, bytes_per_elem) <= budget_gb;
}

/* src/vx27_rope.c:5-16 */
void vx27_rope_cos_sin(int pos, float *cosv, float *sinv, int rope_dim, float theta,
                       float yarn_factor) {
    if (yarn_factor < 1.0f) yarn_factor = 1.0f;
    const float p = (float)pos / yarn_factor;
    for (int i = 0; i < rope_dim / 2; i++) {
        const float f = powf(theta, -2.0f * (float)i / (float)rope_dim);
        const float ang = p * f;
        cosv[i] = cosf(ang);
        sinv[i] = sinf(ang);
    }
}
/* src/vx27_rope.c:31-33: text-only M-RoPE uses one position for all sections */
void vx27_mrope_cos_sin_text(int pos, float *cosv, float *sinv) {
    vx27_rope_cos_sin(pos, cosv, sinv, 64, 10000000.0f, 1.0f);
}
