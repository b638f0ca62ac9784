// K1: fused Gated DeltaNet decode step for B sequences.
//
// Per token the reference runs, per V head, conv1d_step -> gate_params -> step_exact
// (src/vx27_qfwd.c:276-297, src/vx27_deltanet.c:51-122). Here one persistent kernel
// does it for all (sequence, V head) items, each 128x128 fp32 state read once and
// written once. One CTA per SM, three warp roles:
//   TMA warp      streams each item's 64 KB state into a 3-slot shared-memory ring
//                 (one 1-D bulk copy per item), two items ahead of the compute warps;
//   prep warps    (4) each prepares whole items on its own, up to 8 items ahead:
//                 width-4 causal conv + SiLU on the item's 384 channels (q, k of its QK
//                 head, v of its V head) with the conv-history update, the l2 norms
//                 (double sums as src/vx27_deltanet.c:51), q/sqrt(128), and the gates
//                 (double precision) -> a parameter slot in shared memory;
//   compute warps (8) state from shared memory into registers (thread = 16 rows x 4
//                 columns), S' = S*decay, column sums kv = S'^T k, d = (v - kv)*beta,
//                 S'' = S' + k d^T, o = S''^T q, state stored straight from registers;
//                 optionally the layer's gated RMSNorm output o = rmsnorm(o) * w * silu(z)
//                 (src/vx27_qfwd.c:42-48, 146-151) in the same epilogue.
// Waits on the mbarriers are bounded (2 s, %globaltimer); in the compute group a single
// thread waits and publishes the outcome before the group's bar.sync, and a prep warp
// broadcasts its lane 0's outcome, so a timeout makes a whole group leave together and no
// barrier is left half-arrived.
#include "common.cuh"
#include "../../include/vx27_deltanet.h"

namespace vx27 {
namespace {

constexpr int HD = 128;
constexpr int NCOMP = 256;                 // compute threads (warps 0-7)
constexpr int NPREP = 128;                 // prep threads (warps 8-11)
constexpr int NTHREADS = NCOMP + NPREP + 32;  // + TMA warp (warp 12)
constexpr int NSTATE = 3;                  // state ring slots
constexpr int PF_AHEAD = 1;                // L2 prefetch distance in items
constexpr int NPARAM = 8;                  // parameter ring slots
constexpr int STATE_BYTES = HD * HD * 4;   // 64 KB
constexpr int BAR_COMP = 1;                // named barrier id of the compute warps

struct Params {        // one item's prepared inputs
    float qn[HD], kn[HD], v[HD];
    float beta, decay;
};

struct DnSmem {
    float state[NSTATE][HD * HD];
    Params prm[NPARAM];
    float red[8][HD];
    float d[HD];
    double gss[HD / 32];
    uint64_t sfull[NSTATE], sempty[NSTATE], pfull[NPARAM], pempty[NPARAM];
    int flag_comp, abort;
};

__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait; false when the CTA aborted or ~2 s passed (then it aborts).
__device__ bool dn_wait(uint64_t *bar, uint32_t parity, DnSmem &sm, uint32_t *status,
                        uint32_t code) {
    const uint32_t addr = smem_u32(bar);
    uint64_t t0 = 0;
    for (uint32_t it = 0;; ++it) {
        uint32_t ok;
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; "
            "selp.u32 %0, 1, 0, p; }"
            : "=r"(ok) : "r"(addr), "r"(parity) : "memory");
        if (ok) return true;
        if ((it & 255) == 0) {
            if (*(volatile int *)&sm.abort) return false;
            const uint64_t now = gtimer();
            if (it == 0) t0 = now;
            else if (now - t0 > 2000000000ull) {
                *(volatile int *)&sm.abort = 1;
                dev_flag(status, code);
                return false;
            }
        }
    }
}

template <bool ACT_BF16, bool OUT_BF16, bool GATES_F64, bool GATED, bool PRENORM>
__global__ void __launch_bounds__(NTHREADS, 1)
dn_decode_k(float *__restrict__ S, float *__restrict__ ring, const void *__restrict__ qkv,
            const void *__restrict__ ga, const void *__restrict__ gb,
            const float *__restrict__ A_log, const float *__restrict__ dt_bias,
            const float *__restrict__ conv_w, const int *__restrict__ pos,
            const void *__restrict__ z, const float *__restrict__ norm_w, void *__restrict__ o,
            int B, int nqk, int nv, int prefetch_state, uint32_t *status) {
    extern __shared__ uint8_t dn_smem_raw[];
    DnSmem &sm = *reinterpret_cast<DnSmem *>(((uintptr_t)dn_smem_raw + 127) & ~(uintptr_t)127);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n_items_total = B * nv;
    // items of this CTA: blockIdx.x, blockIdx.x + gridDim.x, ...
    const int n_items = blockIdx.x < n_items_total
                            ? (n_items_total - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const int C = (2 * nqk + nv) * HD;

    if (tid == 0) {
        for (int i = 0; i < NSTATE; i++) { mbar_init(&sm.sfull[i], 1); mbar_init(&sm.sempty[i], 1); }
        for (int i = 0; i < NPARAM; i++) { mbar_init(&sm.pfull[i], 1); mbar_init(&sm.pempty[i], 1); }
        sm.abort = 0;
        fence_barrier_init();
    }
    __syncthreads();
    // Everything below reads the previous kernel's outputs (activations, positions) except,
    // with prefetch_state, the first state copies, which the TMA warp issues before waiting.
    // The next kernel may be scheduled once every CTA is past its wait (not earlier: a chain
    // of early triggers would let a later kernel overtake one that is still running).
    if (warp != 12) grid_dep_wait();
    if (tid == 0) grid_dep_launch();

    if (warp == 12) {
        // ---- TMA: state of item i -> ring slot i % NSTATE --------------------------
        if (lane == 0) {
            int i = 0;
            if (prefetch_state)
                for (; i < n_items && i < NSTATE; i++) {
                    const int item = blockIdx.x + i * gridDim.x;
                    mbar_arrive_expect_tx(&sm.sfull[i], STATE_BYTES);
                    bulk_g2s(sm.state[i], S + (size_t)item * HD * HD, STATE_BYTES, &sm.sfull[i]);
                }
            grid_dep_wait();
            for (; i < n_items; i++) {
                const int slot = i % NSTATE;
                if (i >= NSTATE &&
                    !dn_wait(&sm.sempty[slot], ((i / NSTATE) - 1) & 1, sm, status, VX_DEV_TIMEOUT_TMA))
                    break;
                const int item = blockIdx.x + i * gridDim.x;
                mbar_arrive_expect_tx(&sm.sfull[slot], STATE_BYTES);
                bulk_g2s(sm.state[slot], S + (size_t)item * HD * HD, STATE_BYTES, &sm.sfull[slot]);
                // and the next item's state into L2: one more 64 KB read in flight per SM
                // without shared memory (96.3 us per launch against 101.4 us without; two
                // items ahead 97.7 us, three or more slower still)
                if (i + PF_AHEAD < n_items)
                    bulk_prefetch_l2(S + (size_t)(blockIdx.x + (i + PF_AHEAD) * gridDim.x) * HD * HD,
                                     STATE_BYTES);
            }
            if (sm.abort) {  // let issued copies land before the CTA exits
                for (int k = max(0, i - NSTATE); k < i; k++) {
                    const uint32_t addr = smem_u32(&sm.sfull[k % NSTATE]);
                    for (int it = 0; it < (1 << 20); it++) {
                        uint32_t ok;
                        asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                                     : "=r"(ok) : "r"(addr), "r"((uint32_t)((k / NSTATE) & 1)) : "memory");
                        if (ok) break;
                    }
                }
            }
        }
    } else if (warp >= 8) {
        // ---- prep: warp pw prepares items pw, pw+4, ... into parameter slot i % NPARAM.
        // One warp per item (lane = 4 channels of each of q, k, v), warp-level reductions
        // only, so four items are prepared concurrently.
        const int pw = warp - 8;
        for (int i = pw; i < n_items; i += NPREP / 32) {
            const int slot = i % NPARAM;
            const int item = blockIdx.x + i * gridDim.x;
            const int bi = item / nv, vh = item % nv;
            const int tp = pos[bi];
            // issue the gate inputs early (lane 0)
            double ga_v = 0.0, gb_v = 0.0;
            float al = 0.f, dtb = 0.f;
            const size_t gi = (size_t)bi * nv + vh;
            if (lane == 0) {
                if constexpr (GATES_F64) {
                    ga_v = ((const double *)ga)[gi];
                    gb_v = ((const double *)gb)[gi];
                } else {
                    ga_v = (double)act_ld<ACT_BF16>(ga, gi);
                    gb_v = (double)act_ld<ACT_BF16>(gb, gi);
                    al = A_log[vh];
                    dtb = dt_bias[vh];
                }
            }
            int ok = 1;
            if (lane == 0 && i >= NPARAM)
                ok = dn_wait(&sm.pempty[slot], ((i / NPARAM) - 1) & 1, sm, status, VX_DEV_TIMEOUT_TMA);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            const int qk = vh * nqk / nv;
            const bool qk_owner = (vh == 0) || ((vh - 1) * nqk / nv != qk);
            const int sl0 = (tp - 3) & 3, sl1 = (tp - 2) & 3, sl2 = (tp - 1) & 3, slw = tp & 3;
            float *rb = ring + (size_t)bi * 4 * C;
            float y[3][4];
#pragma unroll
            for (int part = 0; part < 3; part++) {
                const int c0 = part == 0 ? qk * HD : part == 1 ? (nqk + qk) * HD
                                                               : 2 * nqk * HD + vh * HD;
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int c = c0 + lane + 32 * j;
                    const float x = act_ld<ACT_BF16>(qkv, (size_t)bi * C + c);
                    const float4 w = *reinterpret_cast<const float4 *>(conv_w + (size_t)c * 4);
                    float acc = __fmul_rn(w.x, rb[(size_t)sl0 * C + c]);
                    acc = __fadd_rn(acc, __fmul_rn(w.y, rb[(size_t)sl1 * C + c]));
                    acc = __fadd_rn(acc, __fmul_rn(w.z, rb[(size_t)sl2 * C + c]));
                    acc = __fadd_rn(acc, __fmul_rn(w.w, x));
                    y[part][j] = __fdiv_rn(acc, __fadd_rn(1.0f, expf(-acc)));
                    if (part == 2 || qk_owner) rb[(size_t)slw * C + c] = x;
                }
            }
            if constexpr (PRENORM) {
                // production q/k pre-normalisation (src/vx27_qfwd.c:31-39, 118-130):
                // RMSNorm y*s*(1+w) with the fp64 sum of squares, then l2norm, q/sqrt(hd)
#pragma unroll
                for (int part = 0; part < 2; part++) {
                    double ss = 0.0;
#pragma unroll
                    for (int j = 0; j < 4; j++) ss += (double)y[part][j] * (double)y[part][j];
                    ss = warp_sum_d(ss);
                    const float s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)(ss / HD), 1e-6f)));
#pragma unroll
                    for (int j = 0; j < 4; j++)
                        y[part][j] = __fmul_rn(__fmul_rn(y[part][j], s),
                                               __fadd_rn(norm_w[lane + 32 * j], 1.0f));
                    double sl = 0.0;
#pragma unroll
                    for (int j = 0; j < 4; j++) sl += (double)y[part][j] * (double)y[part][j];
                    sl = warp_sum_d(sl);
                    const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)sl, 1e-6f)));
#pragma unroll
                    for (int j = 0; j < 4; j++) y[part][j] = __fmul_rn(y[part][j], rs);
                }
                const float qs0 = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
#pragma unroll
                for (int j = 0; j < 4; j++) y[0][j] = __fmul_rn(y[0][j], qs0);
            }
            double sq = 0.0, sk = 0.0;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                sq += (double)y[0][j] * (double)y[0][j];
                sk += (double)y[1][j] * (double)y[1][j];
            }
            sq = warp_sum_d(sq);
            sk = warp_sum_d(sk);
            const float rq = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)sq, 1e-6f)));
            const float rk = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)sk, 1e-6f)));
            const float qs = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
            Params &P = sm.prm[slot];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int d = lane + 32 * j;
                P.qn[d] = __fmul_rn(__fmul_rn(y[0][j], rq), qs);
                P.kn[d] = __fmul_rn(y[1][j], rk);
                P.v[d] = y[2][j];
            }
            if (lane == 0) {
                double beta, g;
                if constexpr (GATES_F64) {
                    beta = ga_v;
                    g = gb_v;
                } else {
                    dn_gates_device(ga_v, (double)al, gb_v, (double)dtb, &beta, &g);
                }
                P.beta = (float)beta;
                P.decay = (float)exp(g);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.pfull[slot]);
        }
    } else {
        // ---- compute: delta rule on item i ------------------------------------------
        for (int i = 0; i < n_items; i++) {
            const int sslot = i % NSTATE, pslot = i % NPARAM;
            if (tid == 0) {
                const bool ok =
                    dn_wait(&sm.sfull[sslot], (i / NSTATE) & 1, sm, status, VX_DEV_TIMEOUT_TMA) &&
                    dn_wait(&sm.pfull[pslot], (i / NPARAM) & 1, sm, status, VX_DEV_TIMEOUT_TMA);
                sm.flag_comp = ok ? 0 : 1;
            }
            named_bar_sync(BAR_COMP, NCOMP);
            if (sm.flag_comp) break;
            const int item = blockIdx.x + i * gridDim.x;
            const Params &P = sm.prm[pslot];
            const float4 *st = reinterpret_cast<const float4 *>(sm.state[sslot]);
            float4 s[16];
#pragma unroll
            for (int r = 0; r < 16; r++) s[r] = st[(warp * 16 + r) * (HD / 4) + lane];
            const float decay = P.decay;
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int r = 0; r < 16; r++) {
                const float k = P.kn[warp * 16 + r];
                s[r].x = __fmul_rn(s[r].x, decay);
                s[r].y = __fmul_rn(s[r].y, decay);
                s[r].z = __fmul_rn(s[r].z, decay);
                s[r].w = __fmul_rn(s[r].w, decay);
                kv.x = fmaf(s[r].x, k, kv.x);
                kv.y = fmaf(s[r].y, k, kv.y);
                kv.z = fmaf(s[r].z, k, kv.z);
                kv.w = fmaf(s[r].w, k, kv.w);
            }
            *reinterpret_cast<float4 *>(&sm.red[warp][lane * 4]) = kv;
            named_bar_sync(BAR_COMP, NCOMP);  // partials ready; state slot fully read
            if (tid == 0) mbar_arrive(&sm.sempty[sslot]);
            if (tid < HD) {
                float acc = 0.0f;
#pragma unroll
                for (int w = 0; w < 8; w++) acc += sm.red[w][tid];
                sm.d[tid] = (P.v[tid] - acc) * P.beta;
            }
            named_bar_sync(BAR_COMP, NCOMP);
            const float4 dj = *reinterpret_cast<const float4 *>(&sm.d[lane * 4]);
            float4 op = make_float4(0.f, 0.f, 0.f, 0.f);
            float4 *Sg = reinterpret_cast<float4 *>(S + (size_t)item * HD * HD);
#pragma unroll
            for (int r = 0; r < 16; r++) {
                const float k = P.kn[warp * 16 + r], q = P.qn[warp * 16 + r];
                s[r].x = fmaf(k, dj.x, s[r].x);
                s[r].y = fmaf(k, dj.y, s[r].y);
                s[r].z = fmaf(k, dj.z, s[r].z);
                s[r].w = fmaf(k, dj.w, s[r].w);
                op.x = fmaf(s[r].x, q, op.x);
                op.y = fmaf(s[r].y, q, op.y);
                op.z = fmaf(s[r].z, q, op.z);
                op.w = fmaf(s[r].w, q, op.w);
                __stcs(Sg + (warp * 16 + r) * (HD / 4) + lane, s[r]);
            }
            *reinterpret_cast<float4 *>(&sm.red[warp][lane * 4]) = op;
            named_bar_sync(BAR_COMP, NCOMP);
            if constexpr (!GATED) {
                if (tid < HD) {
                    float acc = 0.0f;
#pragma unroll
                    for (int w = 0; w < 8; w++) acc += sm.red[w][tid];
                    act_st<OUT_BF16>(o, (size_t)item * HD + tid, acc);
                }
            } else {
                // gated RMSNorm: sum of squares in double over the head, then
                // y = (o * s) * w, times silu(z) = z / (1 + e^-z)
                float acc = 0.0f, zv = 0.0f;
                if (tid < HD) {
                    zv = act_ld<ACT_BF16>(z, (size_t)item * HD + tid);
#pragma unroll
                    for (int w = 0; w < 8; w++) acc += sm.red[w][tid];
                    const double ss = warp_sum_d((double)acc * (double)acc);
                    if (lane == 0) sm.gss[warp] = ss;
                }
                named_bar_sync(BAR_COMP, NCOMP);
                if (tid < HD) {
                    const double ss = (sm.gss[0] + sm.gss[1]) + (sm.gss[2] + sm.gss[3]);
                    const float sc = 1.0f / sqrtf((float)(ss / HD) + 1e-6f);
                    const float y = acc * sc * norm_w[tid];
                    act_st<OUT_BF16>(o, (size_t)item * HD + tid, y * (zv / (1.0f + expf(-zv))));
                }
            }
            named_bar_sync(BAR_COMP, NCOMP);  // parameter slot and red[] free again
            if (tid == 0) mbar_arrive(&sm.pempty[pslot]);
        }
    }
    // lanes that skipped a lane-0 role wait for it here, so whole warps reach the CTA
    // barrier together (it requires converged warps)
    __syncwarp();
    __syncthreads();
}

template <bool A, bool O, bool G, bool Z, bool PN>
int launch(int grid, cudaStream_t st, float *S, float *ring, const void *qkv, const void *a,
           const void *b, const float *A_log, const float *dt_bias, const float *conv_w,
           const int *pos, const void *z, const float *norm_w, void *o, int B, int nqk, int nv,
           int prefetch_state, char *err, size_t errlen) {
    const size_t smem = sizeof(DnSmem) + 128;
    if (ensure_smem_attr((const void *)dn_decode_k<A, O, G, Z, PN>, smem, err, errlen)) return -1;
    // programmatic dependent launch: the CTAs may start (and, with prefetch_state, begin
    // streaming state) while the previous kernel on the stream drains
    VX_CK(launch_pdl(dn_decode_k<A, O, G, Z, PN>, dim3(grid), dim3(NTHREADS), smem, st, S, ring, qkv,
                     a, b, A_log, dt_bias, conv_w, pos, z, norm_w, o, B, nqk, nv, prefetch_state,
                     dev_status()));
    return 0;
}

// The gates exactly as the decode kernel's prep warps form them: double beta and g_log
// from dn_gates_device, and the fp32 beta and decay = exp(g_log) that the update uses.
template <bool ACT_BF16>
__global__ void gate_params_k(const void *__restrict__ a, const void *__restrict__ b,
                              const float *__restrict__ A_log, const float *__restrict__ dt_bias,
                              double *beta, double *g_log, float *beta_f32, float *decay_f32,
                              int n, int nv) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int vh = i % nv;
        double be, g;
        dn_gates_device((double)act_ld<ACT_BF16>(a, i), (double)A_log[vh],
                        (double)act_ld<ACT_BF16>(b, i), (double)dt_bias[vh], &be, &g);
        if (beta) beta[i] = be;
        if (g_log) g_log[i] = g;
        if (beta_f32) beta_f32[i] = (float)be;
        if (decay_f32) decay_f32[i] = (float)exp(g);
    }
}

// ---- T tokens of one sequence with the state resident (vx27_deltanet_decode_tokens) -----
// CTA (cs, vh) keeps columns [16 cs, 16 cs + 16) of V head vh's 128 x 128 state in
// registers for all T tokens (the delta rule's columns are independent): warps 0-7 hold it,
// one 8-row block of one column per thread, and run each token's decay, S^T k, delta,
// update and S^T q with two column reductions and one barrier. Warps 8-15 prepare the tokens ahead into a
// ring of parameter slots, four groups of two warps taking every fourth token: the width-4
// conv + SiLU of the head's q and k channels (two of each per thread, computed by each of
// the head's 8 CTAs) from the group's copy of their conv history (read from the ring at the
// start, so any position sequence reproduces T single-token calls), then the l2 norms from
// double sums of squares. Warp 16 forms the
// gates (double precision) and the conv of this CTA's 16 v channels 32 tokens at a time.
// Nothing crosses CTAs: the state goes back to global memory at the end, and the ring is
// left untouched here (the CTAs of a QK head may run in different waves, so each must find
// the initial history there) and brought up to date by dn_tokens_ring_k afterwards. Per
// token this replaces one launch and a 1 MB state round trip.
constexpr int TK_SPLIT = 8;
constexpr int TK_COLS = HD / TK_SPLIT;
constexpr int TK_NPARAM = 8;
constexpr int TK_NG = 4;   // prep groups (token t goes to group t % TK_NG)
constexpr int TK_GW = 2;   // warps per prep group; a thread owns 2 q and 2 k channels
constexpr int TK_NCH = 2 * HD + TK_COLS;  // q, k and this CTA's v channels

struct TkParams {
    float qn[HD], kn[HD], v[TK_COLS];
    float beta, decay, pad[2];  // a multiple of 16 bytes: rows are read as float4
};
static_assert(sizeof(TkParams) % 16 == 0, "parameter slots stay 16-byte aligned");
struct TkSmem {
    TkParams prm[TK_NPARAM];
    float gbeta[2][32], gdecay[2][32];  // gates of 32-token batches (gate warp -> prep)
    float gv[2][32][TK_COLS];           // and the conv outputs of this CTA's v channels
    float hq[TK_NG][2 * HD][4];  // conv history of the q/k channels by position & 3, a copy
                                 // per prep group
    float hv[TK_COLS][4];        // and of this CTA's v channels (the gate warp's)
    double nps[TK_NG][2][TK_GW][2];  // [group][token parity][warp][q, k] sums of squares
    float red[2][2][8][TK_COLS];  // [S^T k, S^T q][token parity][warp] column partial sums
    uint64_t pfull[TK_NPARAM], pempty[TK_NPARAM], gfull[2], gempty[2];
    int abort;
};

__device__ bool tk_wait(uint64_t *bar, uint32_t parity, TkSmem &sm, uint32_t *status,
                        uint32_t code) {
    const uint32_t addr = smem_u32(bar);
    uint64_t t0 = 0;
    for (uint32_t it = 0;; ++it) {
        uint32_t ok;
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; "
            "selp.u32 %0, 1, 0, p; }"
            : "=r"(ok) : "r"(addr), "r"(parity) : "memory");
        if (ok) return true;
        if ((it & 255) == 0) {
            if (*(volatile int *)&sm.abort) return false;
            const uint64_t now = gtimer();
            if (it == 0) t0 = now;
            else if (now - t0 > 2000000000ull) {
                *(volatile int *)&sm.abort = 1;
                dev_flag(status, code);
                return false;
            }
        }
    }
}

// The ring after the tokens: slot sl holds the input of the last token whose position is
// sl mod 4 (as T single-token calls leave it), or what it held before when no token wrote
// it.
__global__ void dn_tokens_ring_k(float *__restrict__ ring, const void *__restrict__ qkv,
                                 const int *__restrict__ pos, int T, int C, int act_bf16) {
    __shared__ int last[4];
    if (threadIdx.x < 4) last[threadIdx.x] = -1;
    __syncthreads();
    for (int t = threadIdx.x; t < T; t += blockDim.x) atomicMax(&last[pos[t] & 3], t);
    __syncthreads();
    for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < C; c += gridDim.x * blockDim.x)
#pragma unroll
        for (int sl = 0; sl < 4; sl++) {
            const int t = last[sl];
            if (t >= 0)
                ring[(size_t)sl * C + c] = act_bf16 ? act_ld<true>(qkv, (size_t)t * C + c)
                                                    : act_ld<false>(qkv, (size_t)t * C + c);
        }
}

// bar.sync over a named barrier that also ANDs a predicate over the participating threads
__device__ __forceinline__ bool named_bar_and(int id, int nthreads, bool pred) {
    uint32_t r;
    asm volatile(
        "{ .reg .pred p, q; setp.ne.u32 p, %1, 0; bar.red.and.pred q, %2, %3, p; "
        "selp.u32 %0, 1, 0, q; }"
        : "=r"(r) : "r"((uint32_t)pred), "r"(id), "r"(nthreads) : "memory");
    return r != 0;
}

template <bool ACT_BF16, bool OUT_BF16, bool GATES_F64>
__global__ void __launch_bounds__(544, 1)
dn_tokens_k(float *__restrict__ S, float *__restrict__ ring, const void *__restrict__ qkv,
            const void *__restrict__ ga, const void *__restrict__ gb,
            const float *__restrict__ A_log, const float *__restrict__ dt_bias,
            const float *__restrict__ conv_w, const int *__restrict__ pos, void *__restrict__ o,
            float *__restrict__ S_ckpt, float *__restrict__ conv_ckpt, int T, int nqk, int nv,
            uint32_t *status) {
    __shared__ __align__(16) TkSmem sm;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int cs = blockIdx.x, vh = blockIdx.y;
    const int col0 = cs * TK_COLS;
    const int qk = vh * nqk / nv;
    const int C = (2 * nqk + nv) * HD;
    // the q/k channels' ring entries and snapshots are written by one CTA per QK head
    const bool qk_owner = cs == 0 && ((vh == 0) || ((vh - 1) * nqk / nv != qk));
    auto chan = [&](int ch) {
        return ch < HD ? qk * HD + ch
                       : ch < 2 * HD ? (nqk + qk) * HD + ch - HD : 2 * nqk * HD + vh * HD + col0 + ch - 2 * HD;
    };
    if (tid == 0) {
        for (int i = 0; i < TK_NPARAM; i++) {
            mbar_init(&sm.pfull[i], TK_GW);  // one arrival per warp of the token's prep group
            mbar_init(&sm.pempty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&sm.gfull[i], 1);
            mbar_init(&sm.gempty[i], TK_NG);  // every prep group has read the batch
        }
        sm.abort = 0;
        fence_barrier_init();
    }
    for (int ch = tid; ch < TK_NCH; ch += blockDim.x)
#pragma unroll
        for (int sl = 0; sl < 4; sl++) {
            const float v = ring[(size_t)sl * C + chan(ch)];
            if (ch < 2 * HD) {
#pragma unroll
                for (int g = 0; g < TK_NG; g++) sm.hq[g][ch][sl] = v;
            } else {
                sm.hv[ch - 2 * HD][sl] = v;
            }
        }
    __syncthreads();

    if (warp == 16) {
        // ---- gates and v channels, 32 tokens at a time into a two-batch ring: lane l
        // forms token 32k + l's gates (double precision, as the per-token kernel forms
        // them), then lanes 0-15 run their v channel's conv over the batch's tokens in order
        const int jv = lane & (TK_COLS - 1);
        const int cv = chan(2 * HD + jv);
        const float4 wv = *reinterpret_cast<const float4 *>(conv_w + (size_t)cv * 4);
        for (int k = 0; k * 32 < T; k++) {
            const int gb_ = k & 1;
            if (k >= 2 && !tk_wait(&sm.gempty[gb_], ((k >> 1) - 1) & 1, sm, status, VX_DEV_TIMEOUT_TMA))
                break;
            const int t = k * 32 + lane;
            const int nt = min(32, T - k * 32);
            int pl = 0;
            if (t < T) {
                const size_t gi = (size_t)t * nv + vh;
                double beta, g;
                if constexpr (GATES_F64) {
                    beta = ((const double *)ga)[gi];
                    g = ((const double *)gb)[gi];
                } else {
                    dn_gates_device((double)act_ld<ACT_BF16>(ga, gi), (double)A_log[vh],
                                    (double)act_ld<ACT_BF16>(gb, gi), (double)dt_bias[vh], &beta, &g);
                }
                sm.gbeta[gb_][lane] = (float)beta;
                sm.gdecay[gb_][lane] = (float)exp(g);
                pl = pos[t];
            }
            // the batch's v inputs, all requested before the first is used
            float xv[32];
#pragma unroll
            for (int tt = 0; tt < 32; tt++)
                xv[tt] = (lane < TK_COLS && tt < nt)
                             ? act_ld<ACT_BF16>(qkv, (size_t)(k * 32 + tt) * C + cv) : 0.f;
#pragma unroll
            for (int tt = 0; tt < 32; tt++) {
                const int p = __shfl_sync(0xffffffffu, pl, tt);
                if (lane < TK_COLS && tt < nt) {
                    float *h = sm.hv[jv];
                    float acc = __fmul_rn(wv.x, h[(p - 3) & 3]);
                    acc = __fadd_rn(acc, __fmul_rn(wv.y, h[(p - 2) & 3]));
                    acc = __fadd_rn(acc, __fmul_rn(wv.z, h[(p - 1) & 3]));
                    acc = __fadd_rn(acc, __fmul_rn(wv.w, xv[tt]));
                    h[p & 3] = xv[tt];
                    sm.gv[gb_][tt][jv] = __fdiv_rn(acc, __fadd_rn(1.0f, expf(-acc)));
                    if (conv_ckpt) {  // the history after the token, oldest first
#pragma unroll
                        for (int k2 = 0; k2 < 3; k2++)
                            conv_ckpt[((size_t)(k * 32 + tt) * C + cv) * 3 + k2] = h[(p - 2 + k2) & 3];
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.gfull[gb_]);
        }
    } else if (warp >= 8) {
        // ---- prep: TK_NG groups of TK_GW warps; group g takes the tokens t = g mod TK_NG,
        // so TK_NG tokens are prepared at once. Thread jj of a group owns q channels jj and
        // jj + 64 and the same k channels, with the group's own copy of their conv history,
        // into which it first writes the other groups' tokens' inputs in token order (the
        // ring's semantics), all read from global memory a token window ahead.
        constexpr int NJ = 2, TW = TK_NG;  // channels of q (and of k) per thread; window
        const int g = (warp - 8) / TK_GW, wg = (warp - 8) % TK_GW;
        const int jj = tid - 256 - 32 * TK_GW * g;
        float(*hh)[4] = sm.hq[g];
        int cq[NJ], ck[NJ];
        float4 wq[NJ], wk[NJ];
#pragma unroll
        for (int j = 0; j < NJ; j++) {
            cq[j] = chan(jj + 64 * j);
            ck[j] = chan(HD + jj + 64 * j);
            wq[j] = *reinterpret_cast<const float4 *>(conv_w + (size_t)cq[j] * 4);
            wk[j] = *reinterpret_cast<const float4 *>(conv_w + (size_t)ck[j] * 4);
        }
        const float qs = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
        const bool own = qk_owner;  // this CTA writes the q/k channels' snapshots
        auto conv = [&](float *h, float4 wt, float x, int p) {
            float acc = __fmul_rn(wt.x, h[(p - 3) & 3]);
            acc = __fadd_rn(acc, __fmul_rn(wt.y, h[(p - 2) & 3]));
            acc = __fadd_rn(acc, __fmul_rn(wt.z, h[(p - 1) & 3]));
            acc = __fadd_rn(acc, __fmul_rn(wt.w, x));
            h[p & 3] = x;
            return __fdiv_rn(acc, __fadd_rn(1.0f, expf(-acc)));
        };
        // the inputs of tokens t - TW + 1 .. t (the other groups' and this one's)
        float xq[TW][NJ], xk[TW][NJ], nq[TW][NJ], nk[TW][NJ];
        int xp[TW], np[TW];
        auto ld = [&](int t, float(&q)[NJ], float(&k)[NJ], int &p) {
            if (t >= 0 && t < T) {
#pragma unroll
                for (int j = 0; j < NJ; j++) {
                    q[j] = act_ld<ACT_BF16>(qkv, (size_t)t * C + cq[j]);
                    k[j] = act_ld<ACT_BF16>(qkv, (size_t)t * C + ck[j]);
                }
                p = pos[t];
            } else {
#pragma unroll
                for (int j = 0; j < NJ; j++) q[j] = k[j] = 0.f;
                p = 0;
            }
        };
#pragma unroll
        for (int i = 0; i < TW; i++) ld(g - TW + 1 + i, nq[i], nk[i], np[i]);
        for (int t = g; t < T; t += TK_NG) {
            const int slot = t % TK_NPARAM, par = (t / TK_NG) & 1;
#pragma unroll
            for (int i = 0; i < TW; i++) {
                xp[i] = np[i];
#pragma unroll
                for (int j = 0; j < NJ; j++) {
                    xq[i][j] = nq[i][j];
                    xk[i][j] = nk[i][j];
                }
            }
#pragma unroll
            for (int i = 0; i < TW; i++) ld(t + 1 + i, nq[i], nk[i], np[i]);  // next window
            if (jj == 0 && (t & 31) == g &&
                !tk_wait(&sm.gfull[(t >> 5) & 1], (t >> 6) & 1, sm, status, VX_DEV_TIMEOUT_TMA))
                *(volatile int *)&sm.abort = 1;
            if (t >= TK_NPARAM &&
                !tk_wait(&sm.pempty[slot], ((t / TK_NPARAM) - 1) & 1, sm, status, VX_DEV_TIMEOUT_TMA))
                *(volatile int *)&sm.abort = 1;
            const bool ok = !*(volatile int *)&sm.abort;
            // the other groups' tokens t - TW + 1 .. t - 1 enter this group's history first
#pragma unroll
            for (int i = 0; i < TW - 1; i++) {
                if (t - TW + 1 + i >= 0) {
#pragma unroll
                    for (int j = 0; j < NJ; j++) {
                        hh[jj + 64 * j][xp[i] & 3] = xq[i][j];
                        hh[HD + jj + 64 * j][xp[i] & 3] = xk[i][j];
                    }
                }
            }
            const int p = xp[TW - 1];
            float yq[NJ], yk[NJ];
            double sq = 0.0, sk = 0.0;
#pragma unroll
            for (int j = 0; j < NJ; j++) {
                yq[j] = conv(hh[jj + 64 * j], wq[j], xq[TW - 1][j], p);
                yk[j] = conv(hh[HD + jj + 64 * j], wk[j], xk[TW - 1][j], p);
                sq += (double)yq[j] * (double)yq[j];
                sk += (double)yk[j] * (double)yk[j];
            }
            if (conv_ckpt && own) {  // the history after token t, oldest first
#pragma unroll
                for (int j = 0; j < NJ; j++)
#pragma unroll
                    for (int k2 = 0; k2 < 3; k2++) {
                        conv_ckpt[((size_t)t * C + cq[j]) * 3 + k2] = hh[jj + 64 * j][(p - 2 + k2) & 3];
                        conv_ckpt[((size_t)t * C + ck[j]) * 3 + k2] = hh[HD + jj + 64 * j][(p - 2 + k2) & 3];
                    }
            }
            // l2 norms from double sums of squares: warp sums, then every thread adds the
            // group's warps' (one barrier per token)
            sq = warp_sum_d(sq);
            sk = warp_sum_d(sk);
            if (lane == 0) {
                sm.nps[g][par][wg][0] = sq;
                sm.nps[g][par][wg][1] = sk;
            }
            named_bar_sync(2 + g, 32 * TK_GW);
            double ssq = 0.0, ssk = 0.0;
#pragma unroll
            for (int w2 = 0; w2 < TK_GW; w2++) {
                ssq += sm.nps[g][par][w2][0];
                ssk += sm.nps[g][par][w2][1];
            }
            const float rq = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)ssq, 1e-6f)));
            const float rk = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)ssk, 1e-6f)));
            if (ok) {
                TkParams &P = sm.prm[slot];
#pragma unroll
                for (int j = 0; j < NJ; j++) {
                    P.qn[jj + 64 * j] = __fmul_rn(__fmul_rn(yq[j], rq), qs);
                    P.kn[jj + 64 * j] = __fmul_rn(yk[j], rk);
                }
                if (jj < TK_COLS) P.v[jj] = sm.gv[(t >> 5) & 1][t & 31][jj];
                if (jj == 0) {
                    P.beta = sm.gbeta[(t >> 5) & 1][t & 31];
                    P.decay = sm.gdecay[(t >> 5) & 1][t & 31];
                    // this group's last token of a full batch: one of the batch's TK_NG
                    // releases (a partial batch is the last one and is not refilled)
                    if ((t & 31) == 32 - TK_NG + g) mbar_arrive(&sm.gempty[(t >> 5) & 1]);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.pfull[slot]);
        }
    } else {
        // ---- state: thread (row block rb, column col) holds rows 8 rb .. 8 rb + 7 of
        // column col. One CTA barrier per token: the partial sums of both reductions are
        // kept by token parity, and token t's output (and its parameter slot's release)
        // waits for token t + 1's barrier.
        const int rb = tid >> 4, col = tid & (TK_COLS - 1);
        float *Sh = S + (size_t)vh * HD * HD;
        float s[8];
#pragma unroll
        for (int i = 0; i < 8; i++) s[i] = Sh[(size_t)(8 * rb + i) * HD + col0 + col];
        auto rows8 = [&](const float *v, float (&r)[8]) {
            const float4 a = reinterpret_cast<const float4 *>(v + 8 * rb)[0];
            const float4 b = reinterpret_cast<const float4 *>(v + 8 * rb)[1];
            r[0] = a.x; r[1] = a.y; r[2] = a.z; r[3] = a.w;
            r[4] = b.x; r[5] = b.y; r[6] = b.z; r[7] = b.w;
        };
        // token tt's output from the per-warp partials (all threads are past writing them)
        auto out_of = [&](int tt) {
            if (tid < TK_COLS) {
                float ot = 0.f;
#pragma unroll
                for (int w2 = 0; w2 < 8; w2++) ot += sm.red[1][tt & 1][w2][tid];
                act_st<OUT_BF16>(o, ((size_t)tt * nv + vh) * HD + col0 + tid, ot);
            }
            if (tid == 0) mbar_arrive(&sm.pempty[tt % TK_NPARAM]);
        };
        bool ok = true;
        for (int t = 0; t < T && ok; t++) {
            const int slot = t % TK_NPARAM, par = t & 1;
            ok = tk_wait(&sm.pfull[slot], (t / TK_NPARAM) & 1, sm, status, VX_DEV_TIMEOUT_TMA);
            const TkParams &P = sm.prm[slot];  // (after a failed wait: read, then discarded)
            const float decay = P.decay;
            float kr[8];
            rows8(P.kn, kr);
            float kv = 0.f;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                s[i] = __fmul_rn(s[i], decay);
                kv = fmaf(s[i], kr[i], kv);
            }
            kv += __shfl_xor_sync(0xffffffffu, kv, 16);
            if (lane < TK_COLS) sm.red[0][par][warp][col] = kv;
            ok = named_bar_and(1, 256, ok);  // the partials, and one outcome for all threads
            if (!ok) break;
            if (t >= 1) out_of(t - 1);
            float kvt = 0.f;
#pragma unroll
            for (int w2 = 0; w2 < 8; w2++) kvt += sm.red[0][par][w2][col];
            const float delta = (P.v[col] - kvt) * P.beta;
            float qr[8];
            rows8(P.qn, qr);
            float op = 0.f;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                s[i] = fmaf(kr[i], delta, s[i]);
                op = fmaf(s[i], qr[i], op);
            }
            op += __shfl_xor_sync(0xffffffffu, op, 16);
            if (lane < TK_COLS) sm.red[1][par][warp][col] = op;
            if (S_ckpt) {
                float *Sc = S_ckpt + ((size_t)t * nv + vh) * HD * HD;
#pragma unroll
                for (int i = 0; i < 8; i++) Sc[(size_t)(8 * rb + i) * HD + col0 + col] = s[i];
            }
        }
        named_bar_sync(1, 256);  // the last token's partials (every thread leaves alike)
        if (ok) out_of(T - 1);
#pragma unroll
        for (int i = 0; i < 8; i++) Sh[(size_t)(8 * rb + i) * HD + col0 + col] = s[i];
    }
    __syncwarp();
    __syncthreads();
}

}  // namespace
}  // namespace vx27

using namespace vx27;

extern "C" int vx27_deltanet_gate_params_dev(const void *a, const void *b, const float *A_log,
                                             const float *dt_bias, double *beta, double *g_log,
                                             float *beta_f32, float *decay_f32, int n, int nv,
                                             int flags, void *stream, char *err,
                                             size_t errlen) {
    if (n < 0 || nv <= 0) return fail(err, errlen, "vx27_deltanet_gate_params_dev: n=%d nv=%d", n, nv);
    if (n == 0) return 0;
    if (!a || !b || !A_log || !dt_bias)
        return fail(err, errlen, "vx27_deltanet_gate_params_dev: null pointer argument");
    const int threads = 256;
    long long blocks = ((long long)n + threads - 1) / threads;
    if (blocks > 8LL * num_sms()) blocks = 8LL * num_sms();
    cudaStream_t st = (cudaStream_t)stream;
    if (flags & VX27_F_ACT_BF16)
        gate_params_k<true><<<(int)blocks, threads, 0, st>>>(a, b, A_log, dt_bias, beta, g_log,
                                                           beta_f32, decay_f32, n, nv);
    else
        gate_params_k<false><<<(int)blocks, threads, 0, st>>>(a, b, A_log, dt_bias, beta, g_log,
                                                            beta_f32, decay_f32, n, nv);
    VX_CK(cudaGetLastError());
    return 0;
}

static int decode_batch_impl(const char *fn, float *S, float *conv_ring, const void *qkv,
                             const void *a, const void *b, const float *A_log,
                             const float *dt_bias, const float *conv_w, const int *pos,
                             const void *z, const float *norm_w, void *o, int B, int nqk, int nv,
                             int hd, int flags, void *stream, char *err, size_t errlen) {
    if (hd != HD) return fail(err, errlen, "%s: hd=%d unsupported (128 only)", fn, hd);
    if (B <= 0 || nqk <= 0 || nv <= 0 || nv < nqk || (long long)B * nv > (1ll << 30))
        return fail(err, errlen, "%s: bad shape B=%d nqk=%d nv=%d", fn, B, nqk, nv);
    if (!S || !conv_ring || !qkv || !a || !b || !conv_w || !pos || !o)
        return fail(err, errlen, "%s: null pointer argument", fn);
    const bool g64 = flags & VX27_F_GATES_F64;
    if (!g64 && (!A_log || !dt_bias)) return fail(err, errlen, "%s: A_log/dt_bias required", fn);
    if (((uintptr_t)S & 15) || ((uintptr_t)conv_w & 15))
        return fail(err, errlen, "%s: S and conv_w must be 16-byte aligned", fn);
    const bool gated = z != nullptr;
    if (gated && !norm_w) return fail(err, errlen, "%s: norm_w required with z", fn);
    const int items = B * nv;
    const int grid = items < num_sms() ? items : num_sms();
    cudaStream_t st = (cudaStream_t)stream;
    const int pf = (flags & VX27_F_PREFETCH_STATE) ? 1 : 0;
    const int pn = (flags & VX27_F_QK_PRENORM) ? 1 : 0;
    if (pn && !gated)
        return fail(err, errlen, "%s: VX27_F_QK_PRENORM needs the gated entry point (norm_w)", fn);
    const int key = (flags & VX27_F_ACT_BF16 ? 1 : 0) | (flags & VX27_F_OUT_BF16 ? 2 : 0) |
                    (g64 ? 4 : 0) | (gated ? 8 : 0);
#define VX_L(K, A_, O_, G_, Z_, P_)                                                          \
    case K:                                                                                  \
        return launch<A_, O_, G_, Z_, P_>(grid, st, S, conv_ring, qkv, a, b, A_log, dt_bias, \
                                          conv_w, pos, z, norm_w, o, B, nqk, nv, pf, err, errlen);
    switch (key | (pn ? 16 : 0)) {
        VX_L(0, false, false, false, false, false)
        VX_L(1, true, false, false, false, false)
        VX_L(2, false, true, false, false, false)
        VX_L(3, true, true, false, false, false)
        VX_L(4, false, false, true, false, false)
        VX_L(5, true, false, true, false, false)
        VX_L(6, false, true, true, false, false)
        VX_L(7, true, true, true, false, false)
        VX_L(8, false, false, false, true, false)
        VX_L(9, true, false, false, true, false)
        VX_L(10, false, true, false, true, false)
        VX_L(11, true, true, false, true, false)
        VX_L(12, false, false, true, true, false)
        VX_L(13, true, false, true, true, false)
        VX_L(14, false, true, true, true, false)
        VX_L(15, true, true, true, true, false)
        VX_L(24, false, false, false, true, true)
        VX_L(25, true, false, false, true, true)
        VX_L(26, false, true, false, true, true)
        VX_L(27, true, true, false, true, true)
        VX_L(28, false, false, true, true, true)
        VX_L(29, true, false, true, true, true)
        VX_L(30, false, true, true, true, true)
        VX_L(31, true, true, true, true, true)
    }
#undef VX_L
    return fail(err, errlen, "%s: bad flags", fn);
}

extern "C" int vx27_deltanet_decode_batch(float *S, float *conv_ring, const void *qkv,
                                          const void *a, const void *b, const float *A_log,
                                          const float *dt_bias, const float *conv_w,
                                          const int *pos, void *o, int B, int nqk, int nv,
                                          int hd, int flags, void *stream, char *err,
                                          size_t errlen) {
    return decode_batch_impl("vx27_deltanet_decode_batch", S, conv_ring, qkv, a, b, A_log,
                             dt_bias, conv_w, pos, nullptr, nullptr, o, B, nqk, nv, hd, flags,
                             stream, err, errlen);
}

extern "C" int vx27_deltanet_decode_batch_gated(float *S, float *conv_ring, const void *qkv,
                                                const void *a, const void *b,
                                                const float *A_log, const float *dt_bias,
                                                const float *conv_w, const int *pos,
                                                const void *z, const float *norm_w, void *o,
                                                int B, int nqk, int nv, int hd, int flags,
                                                void *stream, char *err, size_t errlen) {
    if (!z) return fail(err, errlen, "vx27_deltanet_decode_batch_gated: z required");
    return decode_batch_impl("vx27_deltanet_decode_batch_gated", S, conv_ring, qkv, a, b,
                             A_log, dt_bias, conv_w, pos, z, norm_w, o, B, nqk, nv, hd, flags,
                             stream, err, errlen);
}

extern "C" int vx27_deltanet_decode_tokens(float *S, float *conv_ring, const void *qkv,
                                           const void *a, const void *b, const float *A_log,
                                           const float *dt_bias, const float *conv_w,
                                           const int *pos, void *o, float *S_ckpt,
                                           float *conv_ckpt, int T, int nqk, int nv, int hd,
                                           int flags, void *stream, char *err,
                                           size_t errlen) {
    const char *fn = "vx27_deltanet_decode_tokens";
    if (T <= 0) return fail(err, errlen, "%s: T=%d", fn, T);
    if (hd != HD) return fail(err, errlen, "%s: hd=%d unsupported (128 only)", fn, hd);
    if (nqk <= 0 || nv < nqk) return fail(err, errlen, "%s: bad shape nqk=%d nv=%d", fn, nqk, nv);
    if (!qkv || !a || !b || !pos || !o) return fail(err, errlen, "%s: null pointer argument", fn);
    if (!S || !conv_ring || !conv_w) return fail(err, errlen, "%s: null pointer argument", fn);
    const bool g64 = flags & VX27_F_GATES_F64;
    if (!g64 && (!A_log || !dt_bias)) return fail(err, errlen, "%s: A_log/dt_bias required", fn);
    if (((uintptr_t)S & 15) || ((uintptr_t)conv_w & 15))
        return fail(err, errlen, "%s: S and conv_w must be 16-byte aligned", fn);
    if (flags & VX27_F_QK_PRENORM)
        return fail(err, errlen, "%s: VX27_F_QK_PRENORM needs the gated entry point (norm_w)", fn);
    if (nv > 65535) return fail(err, errlen, "%s: nv=%d", fn, nv);
    cudaStream_t st = (cudaStream_t)stream;
    uint32_t *status = dev_status();
    const dim3 grid(TK_SPLIT, nv);
    constexpr int TK_THREADS = 544;  // 8 state warps, 8 prep warps, the gate warp
    const int key = (flags & VX27_F_ACT_BF16 ? 1 : 0) | (flags & VX27_F_OUT_BF16 ? 2 : 0) |
                    (g64 ? 4 : 0);
#define VX_T(K, A_, O_, G_)                                                                    \
    case K:                                                                                    \
        dn_tokens_k<A_, O_, G_><<<grid, TK_THREADS, 0, st>>>(S, conv_ring, qkv, a, b, A_log, dt_bias, \
                                                      conv_w, pos, o, S_ckpt, conv_ckpt, T,    \
                                                      nqk, nv, status);                        \
        break;
    switch (key) {
        VX_T(0, false, false, false)
        VX_T(1, true, false, false)
        VX_T(2, false, true, false)
        VX_T(3, true, true, false)
        VX_T(4, false, false, true)
        VX_T(5, true, false, true)
        VX_T(6, false, true, true)
        VX_T(7, true, true, true)
    }
#undef VX_T
    VX_CK(cudaGetLastError());
    const int C = (2 * nqk + nv) * HD;
    dn_tokens_ring_k<<<(C + 255) / 256, 256, 0, st>>>(conv_ring, qkv, pos, T, C,
                                                      (flags & VX27_F_ACT_BF16) ? 1 : 0);
    VX_CK(cudaGetLastError());
    return 0;
}
