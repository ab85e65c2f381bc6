// decode.cuh -- arguments and shared-memory plan of the fused decode-layer
// kernel (decode.cu): one MoE FFN layer for M <= 8 tokens in one launch, the
// 2-bit weights streamed by TMA and multiplied on the tcgen05 tensor cores.
#pragma once

#include <cuda.h>

#include "kernels.cuh"

namespace momij {

// Control words at the start of the workspace (the work-plan header of the
// multi-kernel path): [1] routing status, [2] sticky error word (a bounded
// wait that gave up), [3] grid-barrier arrivals, [4] grid-barrier generation,
// [6..7] the single-token kernel's 64-bit grid-barrier arrival count.
constexpr int kCtrlStatus = 1, kCtrlError = 2, kCtrlArrive = 3, kCtrlGen = 4, kCtrlBar64 = 6;

// Warp roles of the decode kernel (20 warps):
//   0-7   dequantise: warpgroup d (warps 4d..4d+3) turns the 16-code words of
//         groups [4d, 4d+4) of every stage into the MMA's A operand in TMEM;
//   8-23  epilogue: warp 8 + 8d + 4h + q reads the accumulators of MMA
//         issuer (d, h) for TMEM lane quarter q (tcgen05.ld), applies the
//         scales and biases (read from the stage, which both roles release),
//         writes outputs;
//   24-27 MMA issue (lane 0): warp 24+2d+h issues the MMAs of groups 2h, 2h+1
//         of warpgroup d's four (a thread issues one MMA per ~60 cycles, and
//         the issue rate grows with the number of issuing warps);
//   28-29 TMA producers (lane 0), alternate stages; 30-31 idle.
constexpr int kDecDeqWarps = 8;
constexpr int kDecEpiWarps = 16;
constexpr int kDecMmaWarps = 4;
constexpr int kDecProducers = 2;
constexpr int kDecIdleWarps = 2;  // complete the producers' warpgroup (registers move per warpgroup)
constexpr int kDecThreadsAll = 32 * (kDecDeqWarps + kDecEpiWarps + kDecMmaWarps + kDecProducers + kDecIdleWarps);
// Registers per thread after the role split (setmaxnreg): the epilogue
// warpgroups take what the dequantising and the MMA / producer warpgroups give
// up; the sum stays within the launch's 64 x kDecThreadsAll (1024 threads).
constexpr int kDecRegsLaunch = 64, kDecRegsEpi = 80, kDecRegsDeq = 56, kDecRegsCtl = 40;
static_assert(32 * kDecEpiWarps * kDecRegsEpi + 32 * kDecDeqWarps * kDecRegsDeq +
                      32 * (kDecMmaWarps + kDecProducers + kDecIdleWarps) * kDecRegsCtl <=
                  kDecRegsLaunch * kDecThreadsAll,
              "register split exceeds the launch's registers");
static_assert(kDecThreadsAll == 1024, "one CTA of 1024 threads per SM");
constexpr int kDecEpiThreads = 32 * kDecEpiWarps;
constexpr int kDecRouteThreads = 32 * (kDecMmaWarps + kDecProducers);  // route while the others encode x
constexpr int kDecCodeBytes = 128 * 128;   // a stage's codes: 128 rows x one 128-byte K chunk (8 groups)
constexpr int kDecSbBytes = 128 * 16;      // a stage's scales (and again biases): 128 rows x 16 B
constexpr int kDecStageBytes = kDecCodeBytes + 2 * kDecSbBytes;  // 20 KB, a multiple of 1 KB
constexpr int kDecMaxStages = 12;
constexpr int kDecMaxTiles = 96;           // tiles per phase per CTA (host-checked bound)
constexpr int kDecMaxPairs = 64;           // M * K
constexpr int kDecMaxLastBlocks = 128;     // (unit, 64-row block) segments per CTA in the combine
constexpr int kDecAslots = 2;              // A slots per warpgroup (64 TMEM columns each)
constexpr int kDecTmemCols = 512;
constexpr int kTracePointsDec = 32;
// TMA maps: 2D over [rows, row bytes] with box heights 64, 16, 8 (index 0..2),
// a box of 128 rows (index 3, down projection), and a 3D map whose box takes
// 64 rows of both the up and the gate half (index 4, up||gate).
constexpr int kDecMaps = 5;

struct DecodeArgs {
    // codes / scales / biases of the up||gate and the down projection, as
    // bytes [E * N rows, row bytes]: codes with 128-byte swizzle (box 128 B x
    // rows), scales and biases without (box 16 B x rows)
    CUtensorMap map_ug[kDecMaps], map_sug[kDecMaps], map_bug[kDecMaps];
    CUtensorMap map_dn[kDecMaps], map_sdn[kDecMaps], map_bdn[kDecMaps];
    const float* logits;     // [M, E] or nullptr (then inds_in / scores_in)
    const int32_t* inds_in;  // [M, K]
    const float* scores_in;
    int32_t* inds_out;       // optional copies of the routing (CTA 0 writes)
    float* scores_out;
    const uint16_t* x;       // [M, H]
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
    int slice_c0;            // CTA slices weigh a unit's rows c0 + its tokens (the epilogue's work)
    float clamp;
    // dynamic shared-memory carve-up (byte offsets from the 1024-aligned base)
    int off_ring, off_b, off_fs, off_red, off_logits;
    int b_bytes;             // bytes of the B region
};

// T: vectors per column set (1, 2, 4 or 8; the most pairs a unit holds).
template <int DT, int GS, int T>
__global__ void moe_decode_kernel(const __grid_constant__ DecodeArgs a);

// MMA N of a column set of T vectors x 4 digits (M = 128 needs N % 16 == 0).
__host__ __device__ constexpr int dec_mma_n(int T) { return T <= 4 ? 16 : 4 * T; }
// Groups sharing one accumulator pack (their column sets side by side): as
// many as fit in N, at most the two groups one issuing warp takes per chunk.
__host__ __device__ constexpr int dec_gp(int T) { return (dec_mma_n(T) / (4 * T)) < 2 ? 1 : 2; }

// Bytes of B (digit operand) per group: two MMAs of N rows x 32 K-bytes.
__host__ __device__ constexpr int dec_b_group_bytes(int N) { return 64 * N; }

}  // namespace momij
