/*
 * moe_oracle.h -- CPU restatement of momij's 2-bit MoE expert path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * path in libmomij_moe.so and the timed CPU baseline in bench.py; nothing in
 * the product links, imports or calls it.
 *
 * Parity status: UNPINNED against MLX gather_qmm itself.  The reference's
 * canonical path calls MLX.gatherQuantizedMM (mlx-swift 0.31.6, rev
 * 0bb916c67f4b9e5c682cbe02a42c701c93ab5021, swift/Package.resolved:32-37),
 * whose source is not vendored, and neither Swift, Metal nor MLX can run in
 * this container; the reference's kernel tests compare Metal variants to each
 * other and hold no recorded outputs.  The restatement is instead pinned by
 * (1) an independent float64 numpy restatement written from the dense
 * dequantised matrices (oracle/oracle.py), (2) closed-form known answers on
 * the reference test fixtures (MomijCoreTests.swift:264-274, 491-500), and
 * (3) the committed golden vectors under tests/golden/.
 *
 * Semantics restated (file:line are within penta2himajin/momij):
 *   route     swift/Sources/MomijCore/SeedlessMetal.swift:2720-2791
 *             (maple_route_top8: fp32 softmax, K rounds of argmax on the
 *             logits, strict '>' so the lower expert index wins ties,
 *             renormalise the selected gates by their sum) and
 *             MapleMoE.swift:49-55 (same selection for T>1).
 *   gqmm2     SeedlessMetal.swift:2145-2221 (ld16_b2/qd2 + gqmm2_rows):
 *             y[mk,n] = sum_g s[e,n,g]*sum_{k in g} q*x + b[e,n,g]*sum_{k in g} x
 *             with e = inds[mk], x row = mk if lhs_per_expert else mk/Ktop,
 *             code k of a uint32 word at bits [2(k%16), 2(k%16)+1] (LSB
 *             first), group index k/gs.  Accumulated here in float64 and
 *             rounded once to the activation dtype (MLX casts gather_qmm
 *             outputs to the activation dtype, MapleMoE.swift:65-75).
 *   swiglu    SeedlessMetal.swift:2435-2450 (maple_clamped_swiglu) and
 *             MapleMoE.swift:35-39: act = silu(min(g,7)) * clip(u,-7,7) on the
 *             rounded up||gate outputs, rounded once to the activation dtype.
 *             ug row layout [2I] = up || gate (MapleMoE.swift:69-70).
 *   combine   MapleMoE.swift:76-78 and maple_score_reduce
 *             (SeedlessMetal.swift:2452-2470): y = sum_k float(d_k)*score_k,
 *             then cast.  score_resid (SeedlessMetal.swift:2474-2493):
 *             h = cast(float(h) + float(cast(acc))).
 */
#ifndef MOMIJ_MOE_ORACLE_H
#define MOMIJ_MOE_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* dtype of activations, scales, biases and outputs: 0 = bf16, 1 = fp16. */
enum { ORACLE_BF16 = 0, ORACLE_F16 = 1 };

double oracle_half_to_double(uint16_t h, int dtype);
uint16_t oracle_double_to_half(double d, int dtype);

/* logits f32[M,E] -> inds i32[M,K] (descending logit, lower index on ties),
 * scores f32[M,K] (renormalised gates).  Returns 0, or -1 on bad shape. */
int oracle_route(const float* logits, int M, int E, int K, int32_t* inds, float* scores);

/* Per-expert token lists: offsets i32[E+1], pair i32[M*K] (mk = m*K+k, sorted
 * by expert then mk), weight f32[M*K] (the pair's score). */
int oracle_permute(const int32_t* inds, const float* scores, int M, int K, int E,
                   int32_t* offsets, int32_t* pair, float* weight);

/* gather-qmv; see header comment. x rows: M (shared) or M*Ktop (per expert).
 * out [M*Ktop, N].  Returns 0, -1 bad shape, -2 expert index out of range. */
int oracle_gqmm2(const uint16_t* x, const uint32_t* w, const uint16_t* s, const uint16_t* b,
                 const int32_t* inds, uint16_t* out, int M, int Ktop, int Kdim, int N, int E,
                 int gs, int lhs_per_expert, int dtype);

/* ug [rows, 2I] (up || gate) -> act [rows, I]. */
void oracle_clamped_swiglu(const uint16_t* ug, uint16_t* act, int rows, int I, float clamp, int dtype);

/* down [M*Ktop, H] x scores [M*Ktop] -> y [M, H]. */
void oracle_score_reduce(const uint16_t* down, const float* scores, uint16_t* y, int M, int Ktop,
                         int H, int dtype);
/* h [M, H] += cast(sum_k score*down) with the two-kernel rounding. */
void oracle_score_resid(const uint16_t* down, const float* scores, uint16_t* h, int M, int Ktop,
                        int H, int dtype);

/* Whole expert FFN for given routing: up||gate gather, SwiGLU, down gather,
 * combine.  ug/act/down are caller scratch ([M*Ktop,2I], [M*Ktop,I],
 * [M*Ktop,H]) so tests can inspect the staged intermediates.  resid_h may be
 * NULL (y written) or point to h (h += y with two-kernel rounding, y unused). */
int oracle_expert_ffn(const uint16_t* x, const uint32_t* w_ug, const uint16_t* s_ug,
                      const uint16_t* b_ug, const uint32_t* w_dn, const uint16_t* s_dn,
                      const uint16_t* b_dn, const int32_t* inds, const float* scores, uint16_t* y,
                      uint16_t* resid_h, int M, int H, int I, int E, int Ktop, int gs, float clamp,
                      int dtype, uint16_t* ug, uint16_t* act, uint16_t* down);

/* Number of OpenMP threads the oracle uses (for the CPU-baseline record). */
int oracle_num_threads(void);
void oracle_set_num_threads(int n);

#ifdef __cplusplus
}
#endif
#endif
