// route_core.cuh -- router top-k of one token by one warp, shared by the
// router kernels (route.cu) and the fused layer kernel (layer.cu).
//
// Semantics follow maple_route_top8 (momij SeedlessMetal.swift:2720-2791):
// K rounds of argmax on the logits where a strictly larger value replaces
// the running best (so the lower expert index keeps a tie); scores are the
// selected softmax gates renormalised by their sum.  The softmax denominator
// cancels in that renormalisation, so the scores are computed directly as
// exp(l_k - l_max) / sum_selected exp(l_j - l_max) (fp32).
//
// The selection is split from the scores so that a caller on a critical
// path (the fused layer kernel) can start streaming the selected experts'
// weights before the exponentials are evaluated.
#pragma once

#include "common.cuh"

namespace momij {

// Order-preserving 64-bit key of (logit, expert): larger logit first, and on
// equal logits the lower expert index first.
__device__ __forceinline__ unsigned long long route_key(float v, int e) {
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (unsigned long long)(0xffffffffu - (uint32_t)e);
}
__device__ __forceinline__ int route_key_expert(unsigned long long k) {
    return (int)(0xffffffffu - (uint32_t)(k & 0xffffffffull));
}

// Top-K indices of one token (one warp; E <= 1024, K <= 32), in descending
// logit order: inds[k] for k < K (written by lanes 0..K-1).  Each lane keeps
// its best remaining key; a round is one warp max-reduction, and only the
// winning lane rescans its (<= 32) logits.
__device__ __forceinline__ void route_topk_warp(const float* __restrict__ lg, int E, int K,
                                                int* __restrict__ inds) {
    const int lane = threadIdx.x & 31;
    const int nv = (E + 31) >> 5;
    uint32_t taken = 0;
    auto lane_best = [&]() -> unsigned long long {
        unsigned long long best = 0ull;
        for (int i = 0; i < nv; ++i) {
            const int e = lane + 32 * i;
            if (e < E && !((taken >> i) & 1u)) {
                const unsigned long long k = route_key(lg[e], e);
                best = k > best ? k : best;
            }
        }
        return best;
    };
    unsigned long long mine = lane_best();
    int my_ind = 0;
    for (int k = 0; k < K; ++k) {
        unsigned long long best = mine;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
            best = other > best ? other : best;
        }
        const int e = route_key_expert(best);
        if (lane == k) my_ind = e;
        if ((e & 31) == lane) {
            taken |= 1u << (e >> 5);
            mine = lane_best();
        }
    }
    if (lane < K) inds[lane] = my_ind;
}

// Renormalised scores of the K selected experts (inds[0] holds the largest
// logit).  One warp; lanes 0..K-1 write scores[k].
__device__ __forceinline__ void route_scores_warp(const float* __restrict__ lg, int K,
                                                  const int* __restrict__ inds,
                                                  float* __restrict__ scores) {
    const int lane = threadIdx.x & 31;
    const float mx = lg[inds[0]];
    const float ex = (lane < K) ? expf(lg[inds[lane]] - mx) : 0.f;
    // sum in k order (lane 0 first), as the reference's sequential renorm
    float s = 0.f;
    for (int k = 0; k < K; ++k) s += __shfl_sync(0xffffffffu, ex, k);
    if (lane < K) scores[lane] = ex / s;
}

// Both steps for one token.
__device__ __forceinline__ void route_token_warp(const float* __restrict__ lg, int E, int K,
                                                 int32_t* __restrict__ inds,
                                                 float* __restrict__ scores) {
    route_topk_warp(lg, E, K, inds);
    __syncwarp();
    route_scores_warp(lg, K, inds, scores);
}

}  // namespace momij
