// route_core.cuh -- router top-k shared by the router kernels (route.cu) and
// the fused layer kernels (layer.cu, decode.cu): one token by one warp, or a
// small batch block-wide by ranks (route_tokens).
//
// Selection follows maple_route_top8 (momij SeedlessMetal.swift:2720-2791)
// exactly: K rounds, each a reduction tree over a threadgroup of W = 256
// positions (expert e at position e; positions >= E hold -inf; a selected
// expert becomes -inf) in which, at stage s = W/2, ..., 1, position t < s takes
// the candidate of position t + s only if its value is strictly greater
// (:2764-2775).  Among equal values the tree therefore keeps the expert whose
// index bits, read from the lowest bit up, are smallest (the minimum of the
// bit-reversed index) -- not the lowest index: with ties at experts 2 and 4
// the stage s = 4 gives position 0 expert 4 (if expert 0 is smaller) and the
// stages s = 2 and 1 keep it.  Signed zeros compare equal and a NaN never
// replaces nor is replaced, as with the reference's '>'.  The tree is
// emulated stage by stage here (W/32 positions per lane, then the lane
// stages by shuffles); for E > 256 (beyond the reference's kernel) the width
// is the next power of two.
//
// Scores follow the reference's staging: softmax gates e_i / Z over all
// experts (e_i = exp(l_i - max)), the selected gates divided by their sum
// taken in k order (:2755-2790).
#pragma once

#include "common.cuh"

namespace momij {

__host__ __device__ inline int route_tree_width(int E) {
    int W = 256;
    while (W < E) W <<= 1;
    return W;
}

// Top-K indices of one token (one warp; E <= 32 * J, K <= 32), in the
// reference's selection order: inds[k] for k < K (written by lane 0).
// Positions >= E and experts already selected take no further part (the
// reference marks them -inf, which differs only when fewer than K finite
// logits remain).
template <int J>
__device__ __forceinline__ void route_topk_tree(const float* __restrict__ lg, int E, int K,
                                                int* __restrict__ inds) {
    const int lane = threadIdx.x & 31;
    const int W = route_tree_width(E), Jw = W >> 5;  // positions per lane (<= J)
    float val[J];
    uint32_t present = 0;
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const int e = lane + 32 * j;
        const bool in = j < Jw && e < E;
        val[j] = in ? lg[e] : -INFINITY;
        present |= (in ? 1u : 0u) << j;
    }
    for (int k = 0; k < K; ++k) {
        float v[J];
        int jx[J];
        bool pr[J];
#pragma unroll
        for (int j = 0; j < J; ++j) {
            v[j] = val[j];
            jx[j] = j;
            pr[j] = (present >> j) & 1u;
        }
        // stages s >= 32: positions lane + 32 j and lane + 32 (j + sj), in the lane
#pragma unroll
        for (int sj = J / 2; sj >= 1; sj >>= 1) {
            if (sj < Jw) {
#pragma unroll
                for (int j = 0; j < sj; ++j) {
                    if (pr[j + sj] && (!pr[j] || v[j + sj] > v[j])) {
                        v[j] = v[j + sj];
                        jx[j] = jx[j + sj];
                        pr[j] = true;
                    }
                }
            }
        }
        // stages s = 16 .. 1: position lane takes lane + s
        float bv = v[0];
        int bi = lane + 32 * jx[0];
        bool bp = pr[0];
#pragma unroll
        for (int s = 16; s >= 1; s >>= 1) {
            const float ov = __shfl_down_sync(0xffffffffu, bv, s);
            const int oi = __shfl_down_sync(0xffffffffu, bi, s);
            const bool op = __shfl_down_sync(0xffffffffu, bp ? 1 : 0, s) != 0;
            if (lane < s && op && (!bp || ov > bv)) {
                bv = ov;
                bi = oi;
                bp = true;
            }
        }
        bi = __shfl_sync(0xffffffffu, bi, 0);
        if (lane == 0) inds[k] = bi;
        if ((bi & 31) == lane) present &= ~(1u << (bi >> 5));
    }
}

// Renormalised scores of the K selected experts.  One warp; lanes 0..K-1
// write scores[k].
__device__ __forceinline__ void route_scores_warp(const float* __restrict__ lg, int E, int K,
                                                  const int* __restrict__ inds,
                                                  float* __restrict__ scores) {
    const int lane = threadIdx.x & 31;
    float mx = -INFINITY;
    for (int e = lane; e < E; e += 32) mx = fmaxf(mx, lg[e]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float z = 0.f;
    for (int e = lane; e < E; e += 32) z += expf(lg[e] - mx);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
    const float gate = (lane < K) ? expf(lg[inds[lane]] - mx) / z : 0.f;
    float s = 0.f;  // sum in k order (lane 0 first), as the reference's sequential renorm
    for (int k = 0; k < K; ++k) s += __shfl_sync(0xffffffffu, gate, k);
    if (lane < K) scores[lane] = gate / s;
}


// Router of the M tokens by the `nthr` threads from thread `t0` (a named
// barrier `bar` over them): candidate (m, e) lands at position
// #{e' : l(e') > l(e), or l(e') == l(e) and rev(e') < rev(e)} when that is
// below K -- value order, then the reference's tree order on ties (the
// smaller bit-reversed index); the float compare makes signed zeros equal.  Tokens with a NaN logit take the reference's tree step by step
// (route_topk_tree).  Scores (route_scores_warp) unless `with_scores` is
// false: the caller then computes them, e.g. beside other work.
__device__ inline void route_tokens(const float* s_logits, const int* s_nan, int M,
                                    int E, int K, int t0, int nthr, int bar, int* s_inds, float* s_scores,
                                    long long* stamp_ranks = nullptr, bool with_scores = true) {
    const int t = threadIdx.x - t0;
    // threads per candidate: a power of two (<= 32) so that one pass covers
    // every candidate when the threads suffice (at least 1)
    int kParts = 1;
    while (kParts < 32 && M * E * kParts * 2 <= nthr) kParts <<= 1;
    for (int base = 0; base < M * E * kParts; base += nthr) {
        const int it = base + t;
        const int c = it / kParts, sub = it % kParts;
        int r = 0;
        const bool valid = c < M * E;
        const int m = valid ? c / E : 0;
        if (valid && !s_nan[m]) {
            const float* lr = s_logits + m * E;
            const int e = c - m * E;
            const float lc = lr[e];
            const unsigned rc = __brev((unsigned)e);  // bit-reversed order of any power-of-two width
#pragma unroll 8
            for (int j = sub; j < E; j += kParts) {
                const float lj = lr[j];
                r += (lj > lc) | ((lj == lc) & (__brev((unsigned)j) < rc));
            }
        }
        for (int o = 1; o < kParts; o <<= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
        if (valid && sub == 0 && !s_nan[m] && r < K) s_inds[m * K + r] = c - m * E;
    }
    const int w = t >> 5, nw = nthr >> 5;
    for (int m = w; m < M; m += nw)
        if (s_nan[m]) {
            if (E <= 256) route_topk_tree<8>(s_logits + m * E, E, K, s_inds + m * K);
            else route_topk_tree<32>(s_logits + m * E, E, K, s_inds + m * K);
        }
    bar_sync(bar, nthr);
    if (stamp_ranks && t == 0) {
        unsigned long long tt;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(tt));
        *stamp_ranks = (long long)tt;
    }
    if (with_scores)
        for (int m = w; m < M; m += nw) route_scores_warp(s_logits + m * E, E, K, s_inds + m * K, s_scores + m * K);
}

// Both steps for one token.
__device__ __forceinline__ void route_token_warp(const float* __restrict__ lg, int E, int K,
                                                 int32_t* __restrict__ inds,
                                                 float* __restrict__ scores) {
    if (E <= 256) route_topk_tree<8>(lg, E, K, inds);
    else route_topk_tree<32>(lg, E, K, inds);
    __syncwarp();
    route_scores_warp(lg, E, K, inds, scores);
}

}  // namespace momij
