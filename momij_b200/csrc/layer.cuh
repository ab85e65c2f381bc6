// layer.cuh -- arguments of the fused single-token MoE layer kernel (layer.cu).
#pragma once

#include "decode.cuh"

namespace momij {

// The control words (kCtrl*), the trace layout (kTracePointsDec stamps per
// CTA) and the per-64-row completion counters are those of the decode kernel.
constexpr int kLayerMaxLastBlocks = 64;
constexpr int kLayerThreads = 512;  // 16 warps that load and compute
constexpr int kLayerMaxPairs = 64;
// Ring slots per warp (items in flight + 1): one- and two-token units are
// memory-bound and keep 3 items in flight; larger units are compute-bound and
// need the shared memory for their tokens' digit planes.
__host__ __device__ constexpr int layer_stages(int tmax) { return tmax <= 2 ? 4 : 2; }

struct LayerArgs {
    const float* logits;     // [M, E] or nullptr (then inds_in/scores_in)
    const int32_t* inds_in;  // [M, K]
    const float* scores_in;
    int32_t* inds_out;       // optional copies of the routing (CTA 0 writes)
    float* scores_out;
    const uint16_t* x;       // [M, H]
    const uint32_t* w_ug;
    const uint16_t* s_ug;
    const uint16_t* b_ug;
    const uint32_t* w_dn;
    const uint16_t* s_dn;
    const uint16_t* b_dn;
    uint16_t* act;           // [M*K, I] staged SwiGLU output
    uint16_t* down;          // [M*K, H] staged down-projection output
    uint16_t* y;             // [M, H] output, or nullptr when h is set
    uint16_t* h;             // residual stream updated in place (may alias x)
    int32_t* ctrl;           // control words (kCtrl*)
    unsigned* block_ctr;     // [ceil(H/64)] completion counters, zero between calls
    const int32_t* stop;     // optional stop flag (non-zero: return MOMIJ_ERR_STOPPED)
    int M, H, I, E, K;
    int spin_limit;          // polls of the grid barrier before it gives up
    float clamp;
    int nK_up, nK_dn;        // 256-code chunks per row of each phase
    int batch_up, batch_dn;  // tiles per epilogue batch of each phase (multiples of item_tiles):
                             // red and scale buffers, shared by the phases
    int max_tiles, max_units, max_vec;  // capacities of the shared-memory tables
    long long* trace;  // optional: kTracePointsDec %globaltimer stamps per CTA (thread 0)
    // dynamic shared-memory carve-up (byte offsets)
    int off_logits, off_inds, off_scores, off_sorted, off_pflag, off_units;
    int off_tiles_up, off_lunits_up, off_upair_up, off_uslot_up, off_seg_up, off_xvecs;
    int off_tiles_dn, off_lunits_dn, off_upair_dn, off_uslot_dn, off_seg_dn, off_vecs_dn;
    int off_fs, off_dig, off_red, off_sb, off_stage;
};

template <int DT, int GS, int TMAX, int STAGES>
__global__ void moe_layer_kernel(const LayerArgs a);

}  // namespace momij
