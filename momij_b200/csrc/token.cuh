// token.cuh -- arguments of the single-token MoE layer kernel (token.cu).
#pragma once

#include "decode.cuh"

namespace momij {

constexpr int kTokWarps = 16;                       // compute warps (MMA + epilogue)
constexpr int kTokCompute = 32 * kTokWarps;
constexpr int kTokThreads = kTokCompute + 128;      // + the producer warpgroup (one lane issues the TMA loads)
// Registers per thread: at launch (the launch-bounds maximum for 640 threads),
// then moved from the producer warpgroup to the compute warps by setmaxnreg.
constexpr int kTokRegsLaunch = 96, kTokRegsCompute = 112, kTokRegsProducer = 32;
static_assert(kTokCompute * kTokRegsCompute + 128 * kTokRegsProducer <= kTokThreads * kTokRegsLaunch,
              "register split exceeds the launch's registers");
constexpr int kTokStages = 4;                       // ring stages
constexpr int kTokStageBytes = 40960;               // codes (32 KB) + scales (4 KB) + biases (4 KB)
constexpr int kTokSOff = 32768, kTokBOff = 36864;   // scale and bias regions of a stage
constexpr int kTokMaxK = 8;                         // experts per token (a down stage holds all K)
constexpr int kTokMaxM = 8;                         // tokens per launch (processed one after another)
constexpr int kTokMaxTiles = 48;                    // up||gate tiles (8 row pairs) per CTA
constexpr int kTokMaxE = 512;                       // experts ranked by the kernel's own router
constexpr int kTokDnRows = 32;                      // output rows of a CTA (two 16-row MMA tiles)
constexpr int kTokMaps = 6;
// Digit operand (B) of one vector: 2 KB per 512 elements (one 128-byte code column).
__host__ __device__ constexpr int tok_b_bytes(int n) { return n * 4; }
// Partial-sum rows are padded by one float so that the rows of a tile
// written at one code column fall into distinct banks.
__host__ __device__ constexpr int tok_red_stride(int ncol) { return ncol + 1; }

struct TokenArgs {
    // tensor maps over this GPU's memory, loads into this CTA only:
    // [0] up||gate codes, 4D [128 B, I, H / 512 column chunks, 2E] box (128 B, 8, H / 512, 2),
    //     128-byte swizzle (one tile of 8 up rows + 8 gate rows, every column);
    // [1], [2] its scales / biases, box (row bytes, 8, 2) (swizzled when 128 B);
    // [3] down codes, 2D [E*H, I/4] box (128 B, rows_per_cta rows), 128-byte swizzle;
    // [4], [5] its scales / biases, box (16 B, rows_per_cta rows)
    CUtensorMap map[kTokMaps];
    const float* logits;     // [M, E] or nullptr (then inds_in / scores_in)
    const int32_t* inds_in;  // [M, K]
    const float* scores_in;
    int32_t* inds_out;       // optional copies of the routing (CTA 0 writes)
    float* scores_out;
    const uint16_t* x;       // [M, H]
    uint16_t* act;           // [M, K, I] staged SwiGLU output (workspace), one slice per token
    uint16_t* y;             // [M, H] output, or nullptr when h is set
    uint16_t* h;             // residual stream updated in place (may alias x)
    int32_t* ctrl;           // control words (kCtrl*): status, sticky error
    unsigned long long* bar64;  // grid-barrier arrivals: a multiple of the grid size between calls
    const int32_t* stop;     // optional stop flag (non-zero: return MOMIJ_ERR_STOPPED)
    long long* trace;        // optional: kTracePointsDec %globaltimer stamps per CTA
    int M, H, I, E, K;
    int spin_limit;          // polls of a bounded wait before it gives up
    int status_merge;        // 0: set the call's status word; 1: only record a non-OK status (a later
                             // token of a batch launched token by token)
    int rows_per_cta;        // output rows of a CTA in the down phase (<= kTokDnRows)
    float clamp;
    // dynamic shared-memory carve-up (byte offsets from the 1024-aligned base)
    int off_ring, off_logits;  // logits: max(threads, M * E) floats
    int off_xb, off_xfs, off_red_up;   // up phase: x digits, x group factors, partials
    int off_ab, off_afs, off_red_dn;   // down phase (aliases the up-phase region)
};

template <int DT>
__global__ void moe_token_kernel(const __grid_constant__ TokenArgs a);

}  // namespace momij
