// misc.cu -- elementwise SwiGLU, score-weighted combine, synthetic fill.
#include "kernels.cuh"

namespace momij {

// act[r, j] = cast(silu(min(g, clamp)) * clip(u, -clamp, clamp)), ug[r] = up || gate.
// Follows maple_clamped_swiglu (momij SeedlessMetal.swift:2435-2450).
template <int DT>
__global__ void swiglu_kernel(const uint16_t* __restrict__ ug, uint16_t* __restrict__ act,
                              int rows, int I, float clamp) {
    pdl_wait();
    const long long n = (long long)rows * I;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / I, j = i - r * I;
        float u = Half<DT>::to_f(ug[r * 2 * I + j]);
        float g = Half<DT>::to_f(ug[r * 2 * I + I + j]);
        g = fminf(g, clamp);
        u = fminf(fmaxf(u, -clamp), clamp);
        act[i] = Half<DT>::from_f(g / (1.f + expf(-g)) * u);
    }
    pdl_launch_dependents();
}

// y[m,h] = cast(sum_k float(down[m*Ktop+k, h]) * scores[m*Ktop+k])   (RESID=0)
// h[m,h] = cast(float(h) + float(cast(acc)))                          (RESID=1)
// Follows maple_score_reduce / maple_score_resid (momij SeedlessMetal.swift:
// 2452-2493).  A non-null plan with a non-OK status skips the write.
template <int DT, int RESID>
__global__ void combine_kernel(const uint16_t* __restrict__ down, const float* __restrict__ scores,
                               uint16_t* __restrict__ y, int M, int Ktop, int H,
                               const int32_t* __restrict__ plan) {
    pdl_wait();
    if (plan && (plan[1] != MOMIJ_OK || plan[2] != MOMIJ_OK)) return;
    const long long n = (long long)M * H;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const long long m = i / H, h = i - m * H;
        float acc = 0.f;
        for (int k = 0; k < Ktop; ++k) {
            const long long mk = m * Ktop + k;
            acc = fmaf(Half<DT>::to_f(down[mk * H + h]), scores[mk], acc);
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

template __global__ void swiglu_kernel<MOMIJ_DTYPE_BF16>(const uint16_t*, uint16_t*, int, int, float);
template __global__ void swiglu_kernel<MOMIJ_DTYPE_F16>(const uint16_t*, uint16_t*, int, int, float);
template __global__ void combine_kernel<MOMIJ_DTYPE_BF16, 0>(const uint16_t*, const float*, uint16_t*,
                                                             int, int, int, const int32_t*);
template __global__ void combine_kernel<MOMIJ_DTYPE_BF16, 1>(const uint16_t*, const float*, uint16_t*,
                                                             int, int, int, const int32_t*);
template __global__ void combine_kernel<MOMIJ_DTYPE_F16, 0>(const uint16_t*, const float*, uint16_t*,
                                                            int, int, int, const int32_t*);
template __global__ void combine_kernel<MOMIJ_DTYPE_F16, 1>(const uint16_t*, const float*, uint16_t*,
                                                            int, int, int, const int32_t*);

// ---- synthetic inputs (bit-identical to momij_b200/synth.py) -------------
__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
__device__ __forceinline__ uint64_t hash64(uint64_t seed, uint64_t stream, uint64_t i) {
    return splitmix64(seed * 0xD1B54A32D192ED03ull + stream * 0x8CB92BA72F3D8DD7ull + i);
}
__device__ __forceinline__ uint16_t f32_to_half_bits(float f, int dtype) {
    return dtype == MOMIJ_DTYPE_F16 ? Half<MOMIJ_DTYPE_F16>::from_f(f)
                                    : Half<MOMIJ_DTYPE_BF16>::from_f(f);
}

__global__ void synth_fill_kernel(void* dst, int64_t n, int kind, float a, float c, uint64_t seed,
                                  uint64_t stream_id, int64_t start, int dtype) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const uint64_t idx = (uint64_t)(start + i);
        if (kind == 0) {
            static_cast<uint32_t*>(dst)[i] = (uint32_t)(hash64(seed, stream_id, idx) >> 32);
        } else if (kind == 1) {
            const float u = (float)(hash64(seed, stream_id, idx) >> 40) * 5.9604644775390625e-08f;
            const float v = __fadd_rn(__fmul_rn(a, u), c);
            static_cast<uint16_t*>(dst)[i] = f32_to_half_bits(v, dtype);
        } else {
            long long s = 0;
#pragma unroll
            for (int j = 0; j < 3; ++j) {
                const uint64_t h = hash64(seed, stream_id, 3 * idx + j);
#pragma unroll
                for (int q = 0; q < 4; ++q) s += (long long)((h >> (16 * q)) & 0xffffull);
            }
            const float v = (float)((double)(s - 393210) / 65536.0);
            if (kind == 2) static_cast<uint16_t*>(dst)[i] = f32_to_half_bits(v, dtype);
            else static_cast<float*>(dst)[i] = v;
        }
    }
}

}  // namespace momij
