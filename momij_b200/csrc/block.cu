// block.cu -- the dense pieces around the expert path: the router's gate GEMV
// (logits = x W_gate^T, fp32 accumulation), the fused decode router (gate
// GEMV + softmax + top-k + renormalisation in one launch, the last-arriving
// CTA doing the selection) and the RMSNorm that precedes an MoE block.
//
// Reference semantics:
//   * gate GEMV: maple_batched_gemv / maple_gate_gemv (momij
//     SeedlessMetal.swift:2542-2595): y[m, e] = sum_k float(W[e, k]) *
//     float(x[m, k]) in fp32;
//   * fused router: MapleFused.fusedRouter (MapleFused.swift:79-255): the
//     logits as above, softmax p_e = exp(l_e - max) / (sum + 1e-20) with the
//     sum taken per thread over e = t, t + 256, ..., then down a 32-lane
//     shuffle tree, then over the eight simdgroups in order; top-k over p
//     (strict '>' everywhere: within a thread the lower e, in the shuffle
//     tree the lane with the smaller bit-reversed index, across simdgroups
//     the lower one keeps a tie); scores p_k / (sum_k p_k + 1e-20) with the
//     sum in selection order.  The reference defines it for one token and
//     top-8; here every token of the batch is routed alike and K <= 32;
//   * RMSNorm: maple_rms_norm (SeedlessMetal.swift:2496-2527): ss = sum x^2
//     in fp32, inv = 1 / sqrt(ss / H + eps), out = round((x * inv) * w).
#include "common.cuh"
#include "kernels.cuh"

namespace momij {

namespace {

constexpr int kGateTokens = 8;  // tokens per pass over a weight row

template <int WT>
__device__ __forceinline__ void load8(const uint16_t* p, float (&f)[8]) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        f[2 * i] = Half<WT>::to_f((uint16_t)(w[i] & 0xffffu));
        f[2 * i + 1] = Half<WT>::to_f((uint16_t)(w[i] >> 16));
    }
}

// Logits of tokens [m0, m0 + mt) (mt <= kGateTokens) for expert row e, by one
// warp: 16-byte loads of the row and of the tokens' x, fp32 sums per lane,
// then a shuffle tree.  H % 256 == 0.
template <int XT, int WT>
__device__ __forceinline__ void gate_row_warp(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w,
                                              int e, int m0, int mt, int H, float (&acc)[kGateTokens]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int m = 0; m < kGateTokens; ++m) acc[m] = 0.f;
    const uint16_t* wr = w + (size_t)e * H;
    for (int k = lane * 8; k < H; k += 256) {
        float wf[8];
        load8<WT>(wr + k, wf);
#pragma unroll
        for (int m = 0; m < kGateTokens; ++m) {
            if (m < mt) {
                float xf[8];
                load8<XT>(x + (size_t)(m0 + m) * H + k, xf);
#pragma unroll
                for (int i = 0; i < 8; ++i) acc[m] = fmaf(wf[i], xf[i], acc[m]);
            }
        }
    }
#pragma unroll
    for (int m = 0; m < kGateTokens; ++m)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], o);
}

}  // namespace

// grid (ceil(E / warps), ceil(M / kGateTokens)); one warp per expert row.
template <int XT, int WT>
__global__ void __launch_bounds__(256) gate_gemv_kernel(const uint16_t* __restrict__ x,
                                                        const uint16_t* __restrict__ w, float* __restrict__ logits,
                                                        int M, int H, int E) {
    pdl_wait();
    pdl_launch_dependents();
    const int e = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int m0 = blockIdx.y * kGateTokens, mt = min(kGateTokens, M - m0);
    if (e >= E) return;
    float acc[kGateTokens];
    gate_row_warp<XT, WT>(x, w, e, m0, mt, H, acc);
    if ((threadIdx.x & 31) == 0)
        for (int m = 0; m < mt; ++m) logits[(size_t)(m0 + m) * E + e] = acc[m];
}

// Fused router: CTA b computes the logits of experts [8b, 8b + 8) for all M
// tokens (one warp each) into `logits`, then counts itself in; the last CTA
// routes every token.  `ctr` (one word, zero between calls) is reset by the
// last CTA.  M <= kGateTokens * gridDim.y is covered by looping the tokens.
template <int XT, int WT>
__global__ void __launch_bounds__(256) fused_router_kernel(const uint16_t* __restrict__ x,
                                                           const uint16_t* __restrict__ w, unsigned* ctr,
                                                           float* logits, int32_t* inds, float* scores, int M,
                                                           int H, int E, int K) {
    pdl_wait();
    pdl_launch_dependents();
    const int tid = threadIdx.x, lane = tid & 31, sg = tid >> 5;
    const int e = blockIdx.x * 8 + sg;
    if (e < E) {
        for (int m0 = 0; m0 < M; m0 += kGateTokens) {
            const int mt = min(kGateTokens, M - m0);
            float acc[kGateTokens];
            gate_row_warp<XT, WT>(x, w, e, m0, mt, H, acc);
            if (lane == 0)
                for (int m = 0; m < mt; ++m) logits[(size_t)(m0 + m) * E + e] = acc[m];
        }
    }
    __threadfence();
    __syncthreads();
    __shared__ int s_last;
    if (tid == 0) {
        const unsigned prev = atomicAdd(ctr, 1u);
        s_last = prev == gridDim.x - 1;
        if (s_last) *reinterpret_cast<volatile unsigned*>(ctr) = 0u;  // ready for the next call
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();

    // ---- the last CTA: per token, softmax, top-K, renormalisation ----------
    extern __shared__ float s_p[];  // [E] probabilities of the current token
    __shared__ float s_red[8];
    __shared__ int s_idx[32];
    __shared__ float s_val[32];
    for (int m = 0; m < M; ++m) {
        const float* lg = logits + (size_t)m * E;
        float mx = -1e30f;
        for (int j = tid; j < E; j += 256) {
            const float v = __ldcg(lg + j);
            if (v > mx) mx = v;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float t = __shfl_down_sync(0xffffffffu, mx, o);
            if (t > mx) mx = t;
        }
        if (lane == 0) s_red[sg] = mx;
        __syncthreads();
        if (tid == 0) {
            float v = s_red[0];
            for (int s = 1; s < 8; ++s) if (s_red[s] > v) v = s_red[s];
            s_red[0] = v;
        }
        __syncthreads();
        const float lmax = s_red[0];
        __syncthreads();
        float sum = 0.f;
        for (int j = tid; j < E; j += 256) {
            const float v = expf(__ldcg(lg + j) - lmax);
            s_p[j] = v;
            sum += v;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_down_sync(0xffffffffu, sum, o);
        if (lane == 0) s_red[sg] = sum;
        __syncthreads();
        if (tid == 0) {
            float v = s_red[0];
            for (int s = 1; s < 8; ++s) v += s_red[s];
            s_red[0] = v;
        }
        __syncthreads();
        const float inv = 1.0f / (s_red[0] + 1e-20f);
        for (int j = tid; j < E; j += 256) s_p[j] = s_p[j] * inv;
        __syncthreads();
        // rank of candidate j: experts that the reference's scan prefers --
        // a larger p, or an equal p at a lower simdgroup, at a lane with a
        // smaller bit-reversed index, or (same thread) at a lower e
        for (int j = tid; j < E; j += 256) {
            const float pj = s_p[j];
            const int tj = j & 255;
            const unsigned oj = ((unsigned)(tj >> 5) << 5) | (__brev((unsigned)(tj & 31)) >> 27);
            int r = 0;
            for (int i = 0; i < E; ++i) {
                const float pi = s_p[i];
                const int ti = i & 255;
                const unsigned oi = ((unsigned)(ti >> 5) << 5) | (__brev((unsigned)(ti & 31)) >> 27);
                r += (pi > pj) | ((pi == pj) & ((oi < oj) | ((oi == oj) & (i < j))));
            }
            if (r < K) {
                s_idx[r] = j;
                s_val[r] = pj;
            }
        }
        __syncthreads();
        if (tid < K) {
            float ssum = 0.f;
            for (int k = 0; k < K; ++k) ssum += s_val[k];
            inds[(size_t)m * K + tid] = s_idx[tid];
            scores[(size_t)m * K + tid] = s_val[tid] / (ssum + 1e-20f);
        }
        __syncthreads();
    }
}

// One CTA (256 threads) per token.
template <int DT>
__global__ void __launch_bounds__(256) rms_norm_kernel(const uint16_t* __restrict__ x,
                                                       const uint16_t* __restrict__ w, uint16_t* __restrict__ out,
                                                       int H, float eps) {
    pdl_wait();
    pdl_launch_dependents();
    const int m = blockIdx.x, tid = threadIdx.x;
    const uint16_t* xm = x + (size_t)m * H;
    __shared__ float red[256];
    float acc = 0.f;
    for (int i = tid; i < H; i += 256) {
        const float xi = Half<DT>::to_f(xm[i]);
        acc = fmaf(xi, xi, acc);
    }
    red[tid] = acc;
    __syncthreads();
    for (int s = 128; s > 0; s >>= 1) {
        if (tid < s) red[tid] += red[tid + s];
        __syncthreads();
    }
    const float inv = 1.0f / sqrtf(red[0] / (float)H + eps);
    for (int i = tid; i < H; i += 256)
        out[(size_t)m * H + i] = Half<DT>::from_f(__fmul_rn(__fmul_rn(Half<DT>::to_f(xm[i]), inv), Half<DT>::to_f(w[i])));
}

#define MOMIJ_BLOCK_INST(XT, WT)                                                                         \
    template __global__ void gate_gemv_kernel<XT, WT>(const uint16_t*, const uint16_t*, float*, int, int, int); \
    template __global__ void fused_router_kernel<XT, WT>(const uint16_t*, const uint16_t*, unsigned*, float*,   \
                                                         int32_t*, float*, int, int, int, int);
MOMIJ_BLOCK_INST(MOMIJ_DTYPE_BF16, MOMIJ_DTYPE_BF16)
MOMIJ_BLOCK_INST(MOMIJ_DTYPE_BF16, MOMIJ_DTYPE_F16)
MOMIJ_BLOCK_INST(MOMIJ_DTYPE_F16, MOMIJ_DTYPE_BF16)
MOMIJ_BLOCK_INST(MOMIJ_DTYPE_F16, MOMIJ_DTYPE_F16)
template __global__ void rms_norm_kernel<MOMIJ_DTYPE_BF16>(const uint16_t*, const uint16_t*, uint16_t*, int, float);
template __global__ void rms_norm_kernel<MOMIJ_DTYPE_F16>(const uint16_t*, const uint16_t*, uint16_t*, int, float);

}  // namespace momij
