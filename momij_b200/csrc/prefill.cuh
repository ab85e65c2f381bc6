// prefill.cuh -- the grouped (per-expert) GEMM path for prefill and large
// verify batches: tokens are permuted by expert (permute_kernel), cut into
// blocks of <= kBlockTokens sorted pairs of one expert, and every (block, 128
// weight rows) tile runs on the 5th-generation tensor cores (tcgen05, fp32
// accumulators in TMEM) with the 2-bit weights dequantised into bf16/f16
// shared-memory tiles.
#pragma once

#include "kernels.cuh"

namespace momij {

constexpr int kBlockTokens = 128;  // MMA N (tokens) per tile, at most
constexpr int kDequantWarps = 16;  // dequantise + epilogue
constexpr int kLoadWarps = 5;      // cp.async producers (4 token-row warps, 1 weight-chunk warp)
constexpr int kGroupedThreads = 32 * (kDequantWarps + kLoadWarps + 1);  // + one MMA-issuing warp

// Block list header (int32): [0] blocks.  Entries from +4: (expert, first
// sorted position, pairs, 0).
constexpr int kBlockHeader = 4;
__host__ __device__ constexpr size_t block_list_ints(int P, int E) {
    return kBlockHeader + 4 * ((size_t)P / kBlockTokens + (size_t)E + 1);
}

// Dynamic shared memory of grouped_gemm_kernel: two slots of dequantised
// weights (hi + lo, 32 KB each), five 16-KB token-row stages, four 10-KB
// weight chunks, 1 KB of alignment.
__host__ __device__ constexpr size_t grouped_smem_bytes() { return 2 * 32768 + 5 * 16384 + 4 * 10240 + 1024; }

struct GroupedArgs {
    const uint16_t* x;       // activation rows [rows, Kd], 16-element blocks in class order
    int x_per_pair;          // 1: row of pair p is p; 0: p / Ktop
    const uint32_t* w;       // [E, N, Kd/16]
    const uint16_t* s;       // [E, N, Kd/gs]
    const uint16_t* b;
    const int32_t* blocks;   // block list (see above)
    const int32_t* pairs;    // sorted pair ids
    int32_t* status;         // work-plan header: [1] routing status, [2] error word (both 0: run);
                             // a stuck MMA wait records MOMIJ_ERR_TIMEOUT in [2]
    uint16_t* out;           // up||gate mode: act [P, Ru] (columns in class order); rows mode: [P, N]
    int Kd, N, Ru, Ktop;     // Ru: up||gate mode: first gate row (= I)
    int E, P;                // experts, pairs (bounds of the block list entries)
    float clamp;
    // up||gate mode: outputs whose up or gate sum lies within fix_ulps fp32
    // ulps of a rounding midpoint of the 16-bit type are listed here for the
    // exact recomputation (act_fixup_kernel) instead of written: fix[0] =
    // count, then int4 entries (pair, row, which sums: bit 0 up, bit 1 gate,
    // the other sum's fp32 bits); entries past fix_cap are written as computed
    int32_t* fix;
    int fix_cap;
    int fix_ulps;
};

// Distance (in fp32 ulps of the value) below which an up or gate sum of the
// tensor-core GEMM is recomputed exactly.  The GEMM's fp32 accumulation is off
// by ~10 ulps (median; ~260 at the 99th percentile, the tail being sums with
// cancellation, whose small `act` values barely move a row) at K = 1024, and
// about twice that at K = 4096; a sum that close to a midpoint can round to
// the other 16-bit neighbour, and one moved `act` value shifts a whole down row.
__host__ __device__ constexpr int fix_ulps_for(int Kd) { return Kd >= 2048 ? 128 : 64; }

struct FixupArgs {
    const uint16_t* x;       // [M, Kd] token rows (natural order)
    const uint32_t* w;       // up||gate codes [E, 2I, Kd/16]
    const uint16_t* s;       // [E, 2I, Kd/gs]
    const uint16_t* b;
    const int32_t* inds;     // [P] expert of each (token, slot) pair
    const int32_t* fix;      // list written by the up||gate GEMM
    const int32_t* status;   // work-plan header ([1] routing status, [2] error word)
    uint16_t* act;           // [P, I], columns in class order
    int Kd, I, Ktop, fix_cap;
    float clamp;
};

// The listed (pair, row) outputs of the up||gate projection: the flagged
// sums recomputed exactly (per scale group, the code-weighted and the plain
// sums of the activations by error-free fp32 two-sum, combined with the
// group's scale and bias in float64), rounded once to the activation dtype
// like the oracle, and written through the staged clamped SwiGLU.
template <int DT, int GS>
__global__ void act_fixup_kernel(const FixupArgs a);

// y = x with each row's 16-element blocks in class order (element 4j + p of
// a block at 4p + j), the K order of the dequantised weight tiles; `blocks`
// = rows * K / 16.
__global__ void class_order_kernel(const uint4* x, uint4* y, long long blocks);

// Builds the block list from the per-expert offsets of permute_kernel.
__global__ void block_list_kernel(const int32_t* offsets, int E, int32_t* blocks,
                                  const int32_t* status);

// MODE kModeUpSwiglu: tile = 64 up rows + the matching 64 gate rows, output the
// staged clamped SwiGLU; kModeRows: 128 output rows.
template <int DT, int GS, int MODE>
__global__ void grouped_gemm_kernel(const GroupedArgs a);

}  // namespace momij
