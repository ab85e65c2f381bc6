// kernels.cuh -- kernel declarations and launch-argument structs.
#pragma once

#include "common.cuh"

namespace momij {

// Gather-GEMV modes.
enum GemvMode { kModeRows = 0, kModeUpSwiglu = 1 };

struct GemvArgs {
    const uint16_t* x;   // activation vectors, 16-bit, row length Kd
    int x_per_pair;      // 1: vector of pair mk is x[mk]; 0: x[mk / Ktop]
    int digit_all_tokens;  // 1: digitise all M token vectors once (shared x, M <= 8)
    const uint32_t* w;   // [E, N, Kd/16]
    const uint16_t* s;   // [E, N, Kd/gs]
    const uint16_t* b;
    int32_t* plan;       // see build_plan_block; plan[2] is the kernels' error word
    uint16_t* out;       // [P, out_cols]
    int Kd, N, E, M, Ktop, P;
    int rows_per_unit;   // N (rows mode) or N/2 (up||gate row pairs)
    int out_cols;
    float clamp;
    int nK;              // 256-code chunks per row
    int max_units, max_tiles, max_vec;
    int slice_rows;      // cap on the (unit, row) slice a CTA handles at once (it loops over slices)
    int batch_tiles;     // tiles per epilogue batch (a multiple of item_tiles): red and scale buffers
    // dynamic shared-memory carve-up (byte offsets)
    int off_tiles, off_units, off_upair, off_uslot, off_vecs, off_fs, off_dig, off_red, off_sb, off_stage;
};

__global__ void route_kernel(const float* logits, int M, int E, int K, int32_t* inds,
                             float* scores);
__global__ void plan_kernel(const int32_t* inds, int P, int E, int tmax, int32_t* plan, int allow_pad);
__global__ void route_plan_kernel(const float* logits, int M, int E, int K, int tmax,
                                  int32_t* inds, float* scores, int32_t* plan);
constexpr int kPermuteThreads = 256;
__global__ void permute_kernel(const int32_t* inds, const float* scores, int P, int E,
                               int32_t* offsets, int32_t* pair, float* weight, int32_t* status);

template <int DT, int GS, int MODE, int TMAX, int STAGES>
__global__ void gemv_kernel(const GemvArgs a);

template <int DT>
__global__ void swiglu_kernel(const uint16_t* ug, uint16_t* act, int rows, int I, float clamp);
template <int DT, int RESID>
__global__ void combine_kernel(const uint16_t* down, const float* scores, uint16_t* y, int M,
                               int Ktop, int H, const int32_t* plan);
// expert-parallel dispatch / combine (ep.cu)
__global__ void ep_slots_kernel(const int32_t* inds, int P, int E, int world, int capacity,
                                int32_t* send_meta, int32_t* slot_map, int32_t* status);
__global__ void ep_gather_kernel(const uint4* x, const int32_t* slot_map, int P, int K, int row16,
                                 uint4* send_x);
template <int DT, int RESID>
__global__ void ep_combine_kernel(const uint16_t* back, const float* scores, const int32_t* slot_map,
                                  uint16_t* y, int M, int K, int H, const int32_t* status);
__global__ void synth_fill_kernel(void* dst, int64_t n, int kind, float a, float c, uint64_t seed,
                                  uint64_t stream_id, int64_t start, int dtype);

// block.cu: router gate GEMV, fused router, RMSNorm
template <int XT, int WT>
__global__ void gate_gemv_kernel(const uint16_t* x, const uint16_t* w, float* logits, int M, int H, int E);
template <int XT, int WT>
__global__ void fused_router_kernel(const uint16_t* x, const uint16_t* w, unsigned* ctr, float* logits,
                                    int32_t* inds, float* scores, int M, int H, int E, int K);
template <int DT>
__global__ void rms_norm_kernel(const uint16_t* x, const uint16_t* w, uint16_t* out, int H, float eps);

}  // namespace momij
