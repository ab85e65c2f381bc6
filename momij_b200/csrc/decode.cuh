// decode.cuh -- arguments and shared-memory plan of the fused decode-layer
// kernel (decode.cu): one MoE FFN layer for M <= 8 tokens in one launch, the
// 2-bit weights streamed by TMA and multiplied on the tcgen05 tensor cores.
#pragma once

#include <cuda.h>

#include "kernels.cuh"

namespace momij {

// Control words at the start of the workspace (the work-plan header of the
// multi-kernel path): [1] routing status, [2] sticky error word (a bounded
// wait that gave up), [3] grid-barrier arrivals, [4] grid-barrier generation.
constexpr int kCtrlStatus = 1, kCtrlError = 2, kCtrlArrive = 3, kCtrlGen = 4;

constexpr int kDecWarps = 16;             // dequantise + epilogue: 4 warpgroups of 4 warps
constexpr int kDecThreads = 32 * kDecWarps;
constexpr int kDecProducers = 2;          // TMA-issuing warps (lane 0 each), alternate stages
constexpr int kDecThreadsAll = kDecThreads + 32 * (kDecProducers + 1);  // + the MMA-issuing warp
constexpr int kDecStageBytes = 128 * 128;  // one (tile, 128-byte K chunk): 128 rows x 128 B
constexpr int kDecMaxStages = 12;
constexpr int kDecMaxTiles = 48;           // tiles per phase per CTA (host-checked bound)
constexpr int kDecMaxPairs = 64;           // M * K
constexpr int kDecMaxLastBlocks = 64;      // (unit, 64-row block) segments per CTA in the combine
constexpr int kDecBoxes = 4;               // TMA box heights 64, 32, 16, 8 rows
constexpr int kDecTmemCols = 512;
constexpr int kTracePointsDec = 16;

struct DecodeArgs {
    // TMA maps over the packed codes viewed as bytes [E * N rows, Kd / 4],
    // 128-byte swizzle, box 128 B x {64, 32, 16, 8} rows.
    CUtensorMap map_ug[kDecBoxes];
    CUtensorMap map_dn[kDecBoxes];
    const float* logits;     // [M, E] or nullptr (then inds_in / scores_in)
    const int32_t* inds_in;  // [M, K]
    const float* scores_in;
    int32_t* inds_out;       // optional copies of the routing (CTA 0 writes)
    float* scores_out;
    const uint16_t* x;       // [M, H]
    const uint16_t* s_ug;    // [E, 2I, H/gs]
    const uint16_t* b_ug;
    const uint16_t* s_dn;    // [E, H, I/gs]
    const uint16_t* b_dn;
    uint16_t* act;           // [M*K, I] staged SwiGLU output
    uint16_t* down;          // [M*K, H] staged down-projection output
    uint16_t* y;             // [M, H] output, or nullptr when h is set
    uint16_t* h;             // residual stream updated in place (may alias x)
    int32_t* ctrl;           // control words (see above)
    unsigned* block_ctr;     // [ceil(H/64)] completion counters, zero between calls
    const int32_t* stop;     // optional stop flag (non-zero: return MOMIJ_ERR_STOPPED)
    long long* trace;        // optional: kTracePointsDec %globaltimer stamps per CTA
    int M, H, I, E, K;
    int gs;
    int stages;              // ring stages (even)
    int spin_limit;          // polls of a bounded wait before it gives up
    float clamp;
    // dynamic shared-memory carve-up (byte offsets from the 1024-aligned base)
    int off_ring, off_b, off_fs, off_sb, off_logits;
    int b_bytes;             // bytes of the B region
};

// T: vectors per column set (1, 2, 4 or 8; the most pairs a unit holds).
template <int DT, int GS, int T>
__global__ void moe_decode_kernel(const __grid_constant__ DecodeArgs a);

// MMA N of a column set of T vectors x 4 digits (M = 128 needs N % 16 == 0).
__host__ __device__ constexpr int dec_mma_n(int T) { return T <= 4 ? 16 : 4 * T; }

// Bytes of B (digit operand) per group: two MMAs of N rows x 32 K-bytes.
__host__ __device__ constexpr int dec_b_group_bytes(int N) { return 64 * N; }

}  // namespace momij
