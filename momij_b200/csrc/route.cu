// route.cu -- router top-k, per-expert token lists and the GEMV work plan.
//
// Router semantics follow maple_route_top8 (momij SeedlessMetal.swift:
// 2720-2791): softmax in fp32, K rounds of argmax on the logits where a
// strictly larger value replaces the running best (so the lower expert index
// keeps a tie), scores are the selected gates divided by their sum.
#include "kernels.cuh"
#include "route_core.cuh"

namespace momij {

__global__ void route_kernel(const float* __restrict__ logits, int M, int E, int K,
                             int32_t* __restrict__ inds, float* __restrict__ scores) {
    pdl_wait();
    const int warps = blockDim.x >> 5;
    for (int m = blockIdx.x * warps + (threadIdx.x >> 5); m < M; m += gridDim.x * warps)
        route_token_warp(logits + (size_t)m * E, E, K, inds + (size_t)m * K, scores + (size_t)m * K);
    pdl_launch_dependents();
}

// ---- work plan for the gather-GEMV kernels ------------------------------
// Sorts the P = M*Ktop pairs by (expert, pair index) and cuts each expert's
// run into units of at most `tmax` pairs.  plan layout (int32):
//   [0] units U, [1] plan status, [2] error word of the consuming kernels
//   (reset here), [3] reserved,
//   [4 + 4u .. 4 + 4u + 3] unit u = (expert, first sorted position, count, 0),
//   [4 + 4P + q] pair index at sorted position q.
// Runs as one block of 1024 threads; P <= MOMIJ_MAX_PAIRS.  allow_pad: an
// index of -1 marks an empty slot (expert-parallel receive buffers): it joins
// no unit, so its output row is left untouched.
constexpr int kPlanCountE = 1024;  // experts up to which the plan is a counting sort

// The plan by counting (E <= kPlanCountE): per-expert counts, their scans
// (sorted offsets, empty slots first; unit offsets), then warp w places the
// pairs of experts w, w + 32, ... in pair order with ballots and writes their
// units.  Same plan as the rank version below, in O(E * P / 32) per warp
// instead of O(P) per pair.
__device__ void plan_by_counts(const int* s_e, int P, int E, int tmax, int32_t* __restrict__ plan,
                               int* s_cnt, int* s_off, int* s_uoff, int* s_total) {
    const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, warp = tid >> 5, nw = nt >> 5;
    int32_t* units = plan + kPlanHeader;
    int32_t* sorted = plan + kPlanHeader + 4 * P;
    for (int e = tid; e <= E; e += nt) s_cnt[e] = 0;  // [E]: empty slots
    __syncthreads();
    for (int i = tid; i < P; i += nt) {
        const int e = s_e[i];
        atomicAdd(&s_cnt[e < 0 ? E : e], 1);
    }
    __syncthreads();
    if (warp == 0) {
        int cpos = s_cnt[E], cu = 0;  // empty slots sort first
        for (int base = 0; base < E; base += 32) {
            const int e = base + lane;
            const int c = e < E ? s_cnt[e] : 0, nu = (c + tmax - 1) / tmax;
            int ic = c, iu = nu;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int yc = __shfl_up_sync(0xffffffffu, ic, o), yu = __shfl_up_sync(0xffffffffu, iu, o);
                if (lane >= o) {
                    ic += yc;
                    iu += yu;
                }
            }
            if (e < E) {
                s_off[e] = cpos + ic - c;
                s_uoff[e] = cu + iu - nu;
            }
            cpos += __shfl_sync(0xffffffffu, ic, 31);
            cu += __shfl_sync(0xffffffffu, iu, 31);
        }
        if (lane == 0) *s_total = cu;
    }
    __syncthreads();
    const unsigned below = (1u << lane) - 1u;
    for (int e = warp; e <= E; e += nw) {  // e == E: the empty slots (index -1), at the front
        const int c = s_cnt[e];
        if (c == 0) continue;
        const int key = e == E ? -1 : e, start = e == E ? 0 : s_off[e];
        int pos = start;
        for (int base = 0; base < P && pos - start < c; base += 32) {
            const int i = base + lane;
            const bool hit = i < P && s_e[i] == key;
            const unsigned m = __ballot_sync(0xffffffffu, hit);
            if (hit) sorted[pos + __popc(m & below)] = i;
            pos += __popc(m);
        }
        if (e < E)
            for (int k = lane; k * tmax < c; k += 32)
                reinterpret_cast<int4*>(units)[s_uoff[e] + k] =
                    make_int4(e, start + k * tmax, min(tmax, c - k * tmax), 0);
    }
    __syncthreads();
    if (tid == 0) {
        plan[0] = *s_total;
        plan[1] = MOMIJ_OK;
        plan[2] = 0;
    }
}

__device__ void build_plan_block(const int32_t* __restrict__ inds, int P, int E, int tmax,
                                 int32_t* __restrict__ plan, int allow_pad) {
    __shared__ int s_e[MOMIJ_MAX_PAIRS];
    __shared__ int s_flag[MOMIJ_MAX_PAIRS];
    __shared__ int s_warp[32];
    __shared__ int s_bad;
    __shared__ int s_cnt[kPlanCountE + 1], s_off[kPlanCountE], s_uoff[kPlanCountE], s_total;
    const int tid = threadIdx.x, nt = blockDim.x;
    if (tid == 0) s_bad = 0;
    __syncthreads();
    for (int i = tid; i < P; i += nt) {
        int e = inds[i];
        if (e < (allow_pad ? -1 : 0) || e >= E) s_bad = 1;
        s_e[i] = e;
    }
    __syncthreads();
    if (s_bad) {
        if (tid == 0) { plan[0] = 0; plan[1] = MOMIJ_ERR_EXPERT_INDEX; plan[2] = 0; }
        return;
    }
    if (E <= kPlanCountE) {
        plan_by_counts(s_e, P, E, tmax, plan, s_cnt, s_off, s_uoff, &s_total);
        return;
    }
    int32_t* units = plan + kPlanHeader;
    int32_t* sorted = plan + kPlanHeader + 4 * P;
    // stable rank of pair i among all pairs ordered by expert
    int my_pos = -1, my_less = 0, my_before = 0, my_cnt = 0, my_e = 0;
    if (tid < P) {
        my_e = s_e[tid];
        for (int j = 0; j < P; ++j) {
            int ej = s_e[j];
            my_less += ej < my_e;
            my_cnt += ej == my_e;
            my_before += (ej == my_e) & (j < tid);
        }
        my_pos = my_less + my_before;
        s_flag[my_pos] = my_e >= 0 && (my_before % tmax) == 0;  // empty slots sort first, no unit
        sorted[my_pos] = tid;
    }
    __syncthreads();
    // exclusive scan of the unit-start flags over sorted positions (one per thread)
    int f = (tid < P) ? s_flag[tid] : 0;
    int incl = f;
    const int lane = tid & 31, warp = tid >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) s_warp[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int t = (lane < (nt >> 5)) ? s_warp[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int y = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= o) t += y;
        }
        s_warp[lane] = t;  // inclusive prefix of warp totals
    }
    __syncthreads();
    int excl = incl - f + (warp > 0 ? s_warp[warp - 1] : 0);
    __syncthreads();
    // publish uid per sorted position back through s_flag
    if (tid < P) s_flag[tid] = f ? excl : -1;
    __syncthreads();
    if (tid < P && my_e >= 0 && (my_before % tmax) == 0) {
        int u = s_flag[my_pos];
        int cnt = my_cnt - my_before;
        units[4 * u + 0] = my_e;
        units[4 * u + 1] = my_pos;
        units[4 * u + 2] = cnt < tmax ? cnt : tmax;
        units[4 * u + 3] = 0;
    }
    if (tid == nt - 1) {
        plan[0] = s_warp[(nt >> 5) - 1];
        plan[1] = MOMIJ_OK;
        plan[2] = 0;
    }
}

__global__ void __launch_bounds__(1024) plan_kernel(const int32_t* __restrict__ inds, int P,
                                                    int E, int tmax, int32_t* __restrict__ plan,
                                                    int allow_pad) {
    pdl_wait();
    build_plan_block(inds, P, E, tmax, plan, allow_pad);
    pdl_launch_dependents();
}

// Router for all M tokens followed by the plan, in one block (decode sizes).
__global__ void __launch_bounds__(1024) route_plan_kernel(const float* __restrict__ logits, int M,
                                                          int E, int K, int tmax,
                                                          int32_t* __restrict__ inds,
                                                          float* __restrict__ scores,
                                                          int32_t* __restrict__ plan) {
    pdl_wait();
    const int warps = blockDim.x >> 5;
    for (int m = threadIdx.x >> 5; m < M; m += warps)
        route_token_warp(logits + (size_t)m * E, E, K, inds + (size_t)m * K, scores + (size_t)m * K);
    __syncthreads();
    build_plan_block(inds, M * K, E, tmax, plan, 0);
    pdl_launch_dependents();
}

// ---- per-expert token lists (counting sort, stable in the pair index) ----
// Every block histograms all P indices in shared memory and scans the counts
// (so each knows every expert's offset), then collects the pairs of experts
// blockIdx.x, blockIdx.x + gridDim.x, ... in pair order with block-wide
// ballots: positions are deterministic whatever the grid size.  Block 0
// writes the offsets [E + 1].
__global__ void __launch_bounds__(kPermuteThreads) permute_kernel(const int32_t* __restrict__ inds,
                                                                  const float* __restrict__ scores, int P,
                                                                  int E, int32_t* __restrict__ offsets,
                                                                  int32_t* __restrict__ pair,
                                                                  float* __restrict__ weight,
                                                                  int32_t* __restrict__ status) {
    extern __shared__ int s_cnt[];  // E + 1
    constexpr int kWarps = kPermuteThreads / 32;
    __shared__ int s_bad;
    __shared__ int s_wsum[kWarps];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    pdl_wait();  // the indices may come from the previous kernel on the stream
    if (tid == 0) s_bad = 0;
    for (int e = tid; e <= E; e += kPermuteThreads) s_cnt[e] = 0;
    __syncthreads();
    for (int i = tid; i < P; i += kPermuteThreads) {
        const int e = inds[i];
        if (e < 0 || e >= E) s_bad = 1;
        else atomicAdd(&s_cnt[e], 1);
    }
    __syncthreads();
    if (s_bad) {
        if (blockIdx.x == 0 && tid == 0 && status) *status = MOMIJ_ERR_EXPERT_INDEX;
        return;
    }
    if (warp == 0) {  // exclusive scan of the counts, in place; s_cnt[E] = P
        int carry = 0;
        for (int base = 0; base < E; base += 32) {
            const int e = base + lane;
            const int v = e < E ? s_cnt[e] : 0;
            int incl = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            if (e < E) s_cnt[e] = carry + incl - v;
            carry += __shfl_sync(0xffffffffu, incl, 31);
        }
        if (lane == 0) s_cnt[E] = carry;
    }
    __syncthreads();
    if (blockIdx.x == 0)
        for (int e = tid; e <= E; e += kPermuteThreads) offsets[e] = s_cnt[e];
    const unsigned below = (1u << lane) - 1u;
    for (int e = blockIdx.x; e < E; e += gridDim.x) {
        int pos = s_cnt[e];
        const int end = s_cnt[e + 1];
        for (int base = 0; base < P && pos < end; base += kPermuteThreads) {
            const int i = base + tid;
            const bool hit = i < P && inds[i] == e;
            const unsigned m = __ballot_sync(0xffffffffu, hit);
            if (lane == 0) s_wsum[warp] = __popc(m);
            __syncthreads();
            int before = 0, total = 0;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) {
                const int c = s_wsum[w];
                before += w < warp ? c : 0;
                total += c;
            }
            if (hit) {
                const int q = pos + before + __popc(m & below);
                pair[q] = i;
                weight[q] = scores[i];
            }
            pos += total;
            __syncthreads();
        }
    }
    pdl_launch_dependents();
}

}  // namespace momij
