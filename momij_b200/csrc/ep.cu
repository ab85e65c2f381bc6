// ep.cu -- the compute around the two all-to-all exchanges of expert-parallel
// decode (experts sharded contiguously over `world` ranks, E / world each):
//
//   dispatch: every (token, slot) pair of this rank goes to the rank owning its
//             expert: slot_map[p] = dest * capacity + (rank of p among this
//             rank's pairs bound for dest, in pair order), send_meta holds the
//             expert's local index there (-1: empty slot), send_x the token's
//             hidden row;
//   (all-to-all of send_x / send_meta, expert FFN on the received rows -- the
//    gather-GEMV surfaces skip empty slots -- and the reverse all-to-all)
//   combine:  y[m] = sum_k score[m,k] * back[slot_map[m*K + k]] in fp32 in k
//             order, rounded once (or added into the residual stream like
//             maple_score_resid), exactly as the single-GPU combine.
//
// The slot assignment is deterministic, so every rank computes the same bits
// whatever the world size.
#include "common.cuh"
#include "kernels.cuh"

namespace momij {

__global__ void __launch_bounds__(1024) ep_slots_kernel(const int32_t* __restrict__ inds, int P, int E,
                                                        int world, int capacity, int32_t* __restrict__ send_meta,
                                                        int32_t* __restrict__ slot_map, int32_t* status) {
    __shared__ int s_dest[MOMIJ_MAX_PAIRS];
    __shared__ int s_bad;
    pdl_wait();
    const int tid = threadIdx.x, eloc = E / world;
    if (tid == 0) s_bad = 0;
    for (int i = tid; i < world * capacity; i += blockDim.x) send_meta[i] = -1;
    __syncthreads();
    for (int p = tid; p < P; p += blockDim.x) {
        const int e = inds[p];
        if (e < 0 || e >= E) s_bad = 1;
        s_dest[p] = (e >= 0 && e < E) ? e / eloc : 0;
    }
    __syncthreads();
    if (s_bad) {
        if (tid == 0 && status) *status = MOMIJ_ERR_EXPERT_INDEX;
        for (int p = tid; p < P; p += blockDim.x) slot_map[p] = -1;
        return;
    }
    for (int p = tid; p < P; p += blockDim.x) {
        const int d = s_dest[p];
        int before = 0;
        for (int q = 0; q < p; ++q) before += s_dest[q] == d;
        if (before < capacity) {
            slot_map[p] = d * capacity + before;
            send_meta[d * capacity + before] = inds[p] - d * eloc;
        } else {  // cannot happen with capacity >= P; reported, never written out of bounds
            slot_map[p] = -1;
            if (status) atomicExch(status, MOMIJ_ERR_WORKSPACE);
        }
    }
    pdl_launch_dependents();
}

// send_x[slot_map[p]] = x[p / K], 16 bytes per thread.
__global__ void ep_gather_kernel(const uint4* __restrict__ x, const int32_t* __restrict__ slot_map, int P,
                                 int K, int row16, uint4* __restrict__ send_x) {
    pdl_wait();
    const long long n = (long long)P * row16;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const int p = (int)(i / row16), c = (int)(i - (long long)p * row16);
        const int s = slot_map[p];
        if (s >= 0) send_x[(size_t)s * row16 + c] = x[(size_t)(p / K) * row16 + c];
    }
    pdl_launch_dependents();
}

template <int DT, int RESID>
__global__ void ep_combine_kernel(const uint16_t* __restrict__ back, const float* __restrict__ scores,
                                  const int32_t* __restrict__ slot_map, uint16_t* __restrict__ y, int M,
                                  int K, int H, const int32_t* status) {
    pdl_wait();
    if (status && *status != MOMIJ_OK) return;
    const long long n = (long long)M * H;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const long long m = i / H, h = i - m * H;
        float acc = 0.f;
        for (int k = 0; k < K; ++k) {
            const long long mk = m * K + k;
            acc = fmaf(Half<DT>::to_f(back[(size_t)slot_map[mk] * H + h]), scores[mk], acc);
        }
        if (RESID) {
            const float delta = Half<DT>::to_f(Half<DT>::from_f(acc));
            y[i] = Half<DT>::from_f(Half<DT>::to_f(y[i]) + delta);
        } else {
            y[i] = Half<DT>::from_f(acc);
        }
    }
    pdl_launch_dependents();
}

template __global__ void ep_combine_kernel<MOMIJ_DTYPE_BF16, 0>(const uint16_t*, const float*, const int32_t*,
                                                                uint16_t*, int, int, int, const int32_t*);
template __global__ void ep_combine_kernel<MOMIJ_DTYPE_BF16, 1>(const uint16_t*, const float*, const int32_t*,
                                                                uint16_t*, int, int, int, const int32_t*);
template __global__ void ep_combine_kernel<MOMIJ_DTYPE_F16, 0>(const uint16_t*, const float*, const int32_t*,
                                                               uint16_t*, int, int, int, const int32_t*);
template __global__ void ep_combine_kernel<MOMIJ_DTYPE_F16, 1>(const uint16_t*, const float*, const int32_t*,
                                                               uint16_t*, int, int, int, const int32_t*);

}  // namespace momij
