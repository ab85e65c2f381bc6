/*
 * momij_moe.h -- C ABI of libmomij_moe.so, a B200 (sm_100a) implementation of
 * momij's 2-bit group-quantized MoE expert path.
 *
 * Every pointer argument is a device pointer owned by the caller (weights are
 * aliased, never copied), every size is a plain int, and every entry point
 * only enqueues work on `stream` (a cudaStream_t passed as void*; NULL is the
 * legacy default stream) and returns a status code.  This is the encode-only
 * convention of the reference's `into encoder:` overloads; the reference's
 * nil-encoder overloads (commit + wait) correspond to calling the entry point
 * and then momij_moe_synchronize().
 *
 * Weight format (MLX affine, transpose=true; momij WeightStore.swift:50-90):
 *   w   uint32 [E, N, Kdim/16]  code k of a row at bits [2(k%16), 2(k%16)+1]
 *   s,b dtype  [E, N, Kdim/gs]   dequantised weight = s*q + b, q in {0..3}
 *   up||gate projection: N = 2I, rows [0,I) up, rows [I,2I) gate.
 * Activations, scales, biases and outputs share one 16-bit dtype
 * (MOMIJ_DTYPE_BF16 or MOMIJ_DTYPE_F16); router logits and scores are fp32;
 * expert indices int32.  Accumulation is fp32 (exact integer dot products of
 * the codes, fp32 scale/bias epilogue); every gather-GEMV output is rounded
 * once to the activation dtype, as MLX gather_qmm outputs are.
 *
 * Supported shapes: gs in {64, 128}; Kdim % 256 == 0 and 256 <= Kdim <= 4096;
 * any N >= 1; M*Ktop <= MOMIJ_MAX_PAIRS; for shared-x calls M <= 8.
 */
#ifndef MOMIJ_MOE_H
#define MOMIJ_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* momij_stream_t; /* cudaStream_t */

/* Status codes; the first three mirror SeedlessError
 * (SeedlessMetal.swift:3718-3728). */
enum momij_status {
    MOMIJ_OK = 0,
    MOMIJ_ERR_UNSUPPORTED_SHAPE = 1, /* SeedlessError.unsupportedShape(N,K,gs) */
    MOMIJ_ERR_NOT_READY = 2,         /* SeedlessError.notReady */
    MOMIJ_ERR_NO_DEVICE = 3,         /* SeedlessError.noMetal */
    MOMIJ_ERR_INVALID_ARGUMENT = 4,  /* NULL pointer / negative size */
    MOMIJ_ERR_EXPERT_INDEX = 5,      /* an expert index outside [0, E) (device-detected) */
    MOMIJ_ERR_WORKSPACE = 6,         /* workspace too small */
    MOMIJ_ERR_CUDA = 7,              /* a CUDA runtime call failed */
    MOMIJ_ERR_NCCL = 8,              /* an NCCL call failed (expert parallel) */
    MOMIJ_ERR_TIMEOUT = 9,           /* a bounded device-side wait gave up */
    MOMIJ_ERR_STOPPED = 10           /* the stop flag was set */
};

enum momij_dtype { MOMIJ_DTYPE_BF16 = 0, MOMIJ_DTYPE_F16 = 1 };

#define MOMIJ_MAX_PAIRS 1024
/* momij_moe_expert_ffn / momij_moe_forward: M*Ktop up to this many pairs
 * through the grouped (prefill) path. */
#define MOMIJ_MAX_GROUPED_PAIRS 65536

/* Human-readable name of a status code (never NULL). */
const char* momij_status_string(int status);

/* Library/ABI version, e.g. 100 for 0.1.0. */
int momij_version(void);

/* Number of streaming multiprocessors of the current device, or -1. */
int momij_device_sm_count(void);

/* Stop flag: a device int32 (or NULL to clear) that every kernel of this
 * library reads when it starts; a non-zero value makes the call skip its work
 * and report MOMIJ_ERR_STOPPED through momij_moe_synchronize (outputs are then
 * undefined).  Process-wide, like the reference's single stop buffer; set it
 * before the calls it should affect are enqueued (a graph keeps the pointer it
 * was captured with).
 * Replaces: SeedlessMetal's stopFlag buffer, checked on entry by every
 * gqmm2 / router kernel (SeedlessMetal.swift:60, 69-70, 2185, 2730). */
int momij_set_stop_flag(const int32_t* device_flag);

/* Bound of the device-side waits (polls of an mbarrier or of the grid
 * barrier) before a kernel gives up with MOMIJ_ERR_TIMEOUT: 0 restores the
 * default (about a second), -1 makes every wait give up at once (for testing
 * the error path).  Process-wide; applies to calls enqueued afterwards.  No
 * counterpart in the reference (Metal command buffers have no such bound). */
int momij_set_spin_limit(int polls);

/* Waits for `stream`, then folds any device-detected error recorded in
 * `workspace` (may be NULL) into the returned status. */
int momij_moe_synchronize(momij_stream_t stream, const void* workspace);

/* Router: fp32 softmax over logits [M,E]; top-K by K rounds of argmax on the
 * logits (strict '>', so the lower index wins a tie); scores are the selected
 * gates renormalised by their sum.  inds [M,K] int32 in descending-score
 * order, scores [M,K] fp32.  K <= 32, E <= 1024.
 * Replaces: maple_route_top8 + SeedlessMetal.encodeRoute
 * (SeedlessMetal.swift:2720-2791, 1266-1281); MapleMoE.route
 * (MapleMoE.swift:41-56). */
int momij_moe_route(const float* logits, int M, int E, int K, int32_t* inds, float* scores,
                    momij_stream_t stream);

/* Per-expert token lists (counting sort by expert, ties by pair index):
 * offsets [E+1], pair [M*K] (pair index m*K+k), weight [M*K] (its score).
 * Replaces: nothing in the reference (MLX gather_qmm is called with
 * sortedIndices:false, MapleMoE.swift:68); it is the permute step the
 * grouped prefill GEMM and the expert-parallel dispatch consume. */
int momij_moe_permute(const int32_t* inds, const float* scores, int M, int K, int E,
                      int32_t* offsets, int32_t* pair, float* weight, momij_stream_t stream);

/* Workspace bytes needed by momij_moe_gqmm2 / up_swiglu / expert_ffn /
 * forward for these sizes (plan + staged intermediates).  The workspace must
 * be zero-filled once before its first use; the kernels leave it reusable. */
size_t momij_moe_workspace_size(int M, int Ktop, int H, int I);

/* 2-bit gather-GEMV:
 *   out[mk, n] = sum_k (s[e,n,k/gs]*q[e,n,k] + b[e,n,k/gs]) * x[row, k]
 * with e = inds[mk], mk in [0, M*Ktop), row = mk if lhs_per_expert else
 * mk / Ktop.  x [M or M*Ktop, Kdim], out [M*Ktop, N].  Each distinct expert's
 * rows are streamed once per call (tokens sharing an expert share the load).
 * inds[mk] == -1 marks an empty slot (expert-parallel receive buffers): its
 * output row is left untouched.  Same for momij_moe_gqmm2_up_swiglu.
 * Replaces: SeedlessMetal.gqmm2 (SeedlessMetal.swift:312-438, kernel
 * gqmm2_rows :2168-2221) and MLX.gatherQuantizedMM(transpose:true, bits:2,
 * mode:.affine) (MapleMoE.swift:65-75). */
int momij_moe_gqmm2(const void* x, const uint32_t* w, const void* scales, const void* biases,
                    const int32_t* inds, void* out, int M, int Ktop, int Kdim, int N, int E, int gs,
                    int lhs_per_expert, int dtype, void* workspace, size_t workspace_bytes,
                    momij_stream_t stream);

/* momij_moe_gqmm2 for callers that cannot allocate device memory (a binding
 * that owns only its inputs and outputs, or an engine that forbids allocation
 * inside its token loop because cudaMalloc can synchronize the device).  No
 * counterpart in the reference.  Same arguments and results as
 * momij_moe_gqmm2 minus the workspace: the work plan lives in a fixed
 * 20,736-byte array compiled into the library (held on every GPU that loads
 * it until exit), so the call allocates nothing.  Limits: M*Ktop <=
 * MOMIJ_NOALLOC_MAX_PAIRS, otherwise MOMIJ_ERR_WORKSPACE; every call shares
 * the array, so calls that overlap on the GPU race -- serialise them; the
 * first call on a device looks up the array's address (cudaGetSymbolAddress)
 * and should come before any stream capture on that device; the address is
 * cached per device for the life of the process, so after cudaDeviceReset
 * (or any other teardown of the device's primary context) the cached address
 * is stale: do not call this entry point again in that process; an expert
 * index out of range makes the call write nothing to `out`, and this entry
 * point has no way to report it (the next valid call rewrites the plan). */
#define MOMIJ_NOALLOC_MAX_PAIRS 1024
int momij_moe_gqmm2_noalloc(const void* x, const uint32_t* w, const void* scales,
                            const void* biases, const int32_t* inds, void* out, int M, int Ktop,
                            int Kdim, int N, int E, int gs, int lhs_per_expert, int dtype,
                            momij_stream_t stream);

/* Fused up||gate gather-GEMV + clamped SwiGLU:
 *   act[mk, j] = silu(min(g, clamp)) * clip(u, -clamp, clamp)
 * with u, g the up row j and gate row I+j outputs (each rounded to dtype
 * first).  x [M, H], w [E, 2I, H/16], act [M*Ktop, I].
 * Replaces: SeedlessMetal.gqmm2UpSwiglu (SeedlessMetal.swift:441-484, kernel
 * gqmm2_up_swiglu :2360-2433) and MapleMoE.clampedSwiglu over the split
 * gather output (MapleMoE.swift:35-39, 65-70). */
int momij_moe_gqmm2_up_swiglu(const void* x, const uint32_t* w, const void* scales,
                              const void* biases, const int32_t* inds, void* act, int M, int Ktop,
                              int H, int I, int E, int gs, float clamp, int dtype, void* workspace,
                              size_t workspace_bytes, momij_stream_t stream);

/* Elementwise clamped SwiGLU on ug [rows, 2I] (up || gate) -> act [rows, I].
 * Replaces: maple_clamped_swiglu / encodeClampedSwiglu
 * (SeedlessMetal.swift:2435-2450, 486-498). */
int momij_moe_clamped_swiglu(const void* ug, void* act, int rows, int I, float clamp, int dtype,
                             momij_stream_t stream);

/* y[m, h] = cast(sum_k float(down[m*Ktop+k, h]) * scores[m*Ktop+k]).
 * Replaces: maple_score_reduce / encodeScoreReduce (SeedlessMetal.swift:
 * 2452-2470, 652-667) and the combine of MapleMoE.swift:76-78. */
int momij_moe_score_reduce(const void* down, const float* scores, void* y, int M, int Ktop,
                           int H, int dtype, momij_stream_t stream);

/* h[m, h] = cast(float(h) + float(cast(acc))) with acc as in score_reduce.
 * Replaces: maple_score_resid / encodeScoreResid (SeedlessMetal.swift:
 * 2474-2493, 669-684). */
int momij_moe_score_resid(const void* down, const float* scores, void* h, int M, int Ktop,
                          int H, int dtype, momij_stream_t stream);

/* Whole expert FFN for given routing: up||gate gather + SwiGLU, down gather,
 * score-weighted combine.  If resid_h != NULL it is updated in place
 * (h += y, two-kernel rounding) and y may be NULL.
 * Replaces: SeedlessMetal.encodeFusedExpert / fusedExpertStep
 * (SeedlessMetal.swift:503-572) and SeedlessMoELayer.run
 * (MapleSeedlessMoE.swift:61-77). */
int momij_moe_expert_ffn(const void* x, const uint32_t* w_ug, const void* s_ug, const void* b_ug,
                         const uint32_t* w_dn, const void* s_dn, const void* b_dn,
                         const int32_t* inds, const float* scores, void* y, void* resid_h, int M,
                         int H, int I, int E, int Ktop, int gs, float clamp, int dtype,
                         void* workspace, size_t workspace_bytes, momij_stream_t stream);

/* Router + expert FFN from logits [M,E]: writes inds/scores (may be NULL to
 * keep them in the workspace only) and y (or updates resid_h).
 * Replaces: MapleMoE.callAsFunction (MapleMoE.swift:59-80) and the
 * route + fused-expert part of SeedlessMetal.encodeMoEBlock
 * (SeedlessMetal.swift:576-609). */
int momij_moe_forward(const float* logits, const void* x, const uint32_t* w_ug, const void* s_ug,
                      const void* b_ug, const uint32_t* w_dn, const void* s_dn, const void* b_dn,
                      int32_t* inds, float* scores, void* y, void* resid_h, int M, int H, int I,
                      int E, int Ktop, int gs, float clamp, int dtype, void* workspace,
                      size_t workspace_bytes, momij_stream_t stream);

/* Router logits [M, E] = x [M, H] W_gate [E, H]^T, fp32 accumulation (the
 * 16-bit x and W are widened; x_dtype and w_dtype are MOMIJ_DTYPE_*).
 * H % 256 == 0; rows 16-byte aligned.
 * Replaces: maple_batched_gemv / maple_gate_gemv (SeedlessMetal.swift:
 * 2542-2595) as encoded by SeedlessMetal.encodeGate (:1143-1202), and the
 * logits matmul of MapleMoE.route (MapleMoE.swift:52). */
int momij_moe_router_logits(const void* x, const void* w_gate, float* logits, int M, int H, int E,
                            int x_dtype, int w_dtype, momij_stream_t stream);

/* Fused router in one launch: the gate GEMV, then per token softmax
 * p_e = exp(l_e - max) / (sum + 1e-20), top-K over p, scores
 * p_k / (sum_k p_k + 1e-20); ties go as in the reference's scan (a lower
 * simdgroup, then the lane with the smaller bit-reversed index, then the lower
 * expert keeps a tie).  counter: one device uint32, zero before the first call
 * (each call leaves it zero; one counter per concurrently running call).
 * logits [M, E] is scratch (left holding the logits).  M <= 64, K <= 32,
 * E % 8 == 0, H % 256 == 0.
 * Replaces: MapleFused.fusedRouter (MapleFused.swift:79-255), which the
 * reference uses for one token and K = 8 (MapleMoE.swift:43-47); every token of
 * a batch is routed alike here. */
int momij_moe_fused_router(const void* x, const void* w_gate, uint32_t* counter, float* logits,
                           int32_t* inds, float* scores, int M, int H, int E, int K, int x_dtype,
                           int w_dtype, momij_stream_t stream);

/* RMSNorm: out[m] = round((x[m] * inv) * w), inv = 1 / sqrt(sum x^2 / H + eps),
 * fp32 arithmetic.
 * Replaces: maple_rms_norm (SeedlessMetal.swift:2496-2527) as encoded by
 * SeedlessMetal.encodeRms (:1071-1086). */
int momij_rms_norm(const void* x, const void* w, void* out, int M, int H, float eps, int dtype,
                   momij_stream_t stream);

/* Workspace bytes of momij_moe_block: momij_moe_workspace_size plus the
 * normalised activations [M, H] and the logits [M, E]; zero-filled once
 * before its first use, like the momij_moe_forward workspace. */
size_t momij_moe_block_workspace_size(int M, int Ktop, int H, int I, int E);

/* One MoE block from the residual stream h [M, H], updated in place:
 * xn = rmsnorm(h, norm_w, eps); logits = xn W_gate^T; top-K routing
 * (momij_moe_route); h += experts(xn) with the fused score-residual rounding
 * (momij_moe_forward with resid_h = h).  inds/scores may be NULL.
 * gate_dtype: dtype of W_gate.
 * Replaces: SeedlessMetal.encodeMoEBlock (SeedlessMetal.swift:576-609). */
int momij_moe_block(void* h, const void* norm_w, float eps, const void* w_gate, int gate_dtype,
                    const uint32_t* w_ug, const void* s_ug, const void* b_ug, const uint32_t* w_dn,
                    const void* s_dn, const void* b_dn, int32_t* inds, float* scores, int M, int H,
                    int I, int E, int Ktop, int gs, float clamp, int dtype, void* workspace,
                    size_t workspace_bytes, momij_stream_t stream);

/* Expert-parallel decode (experts sharded contiguously: rank r owns experts
 * [r*E/world, (r+1)*E/world)).  The caller runs the two all-to-all exchanges
 * with its own NCCL communicator (ncclSend/ncclRecv or all-to-all of equal
 * splits of `capacity` rows per rank):
 *   1. momij_moe_ep_dispatch: pair p = m*K + k of this rank's M tokens goes to
 *      rank dest = inds[p] / (E/world) at row slot_map[p] = dest*capacity +
 *      (its rank among the pairs bound for dest, in pair order) of send_x
 *      [world*capacity, H] (the token's row x[m]) and send_meta
 *      [world*capacity] (the expert's local index; -1 marks empty rows).
 *      capacity >= M*K.  *status (device int32): MOMIJ_OK or
 *      MOMIJ_ERR_EXPERT_INDEX.
 *   2. all-to-all(send_x -> recv_x), all-to-all(send_meta -> recv_meta);
 *   3. momij_moe_gqmm2_up_swiglu(recv_x, ..., recv_meta, act, M=world*capacity,
 *      Ktop=1) and momij_moe_gqmm2(act, ..., recv_meta, down, M=world*capacity,
 *      Ktop=1) with the rank's local experts (empty rows are skipped);
 *   4. all-to-all(down -> back);
 *   5. momij_moe_ep_combine: y[m] = sum_k scores[m,k] * back[slot_map[m*K+k]]
 *      in fp32 in k order, rounded once, or added into resid_h like
 *      momij_moe_score_resid -- the same bits as the single-GPU combine.
 * Replaces: no counterpart in the reference (it runs on one GPU); the expert
 * split follows north-star config 4 (experts sharded evenly, all-to-all
 * dispatch and combine over NVLink). */
int momij_moe_ep_dispatch(const int32_t* inds, const void* x, int M, int K, int E, int world,
                          int capacity, int H, void* send_x, int32_t* send_meta, int32_t* slot_map,
                          int32_t* status, momij_stream_t stream);
int momij_moe_ep_combine(const void* back, const float* scores, const int32_t* slot_map, void* y,
                         void* resid_h, int M, int K, int H, int dtype, const int32_t* status,
                         momij_stream_t stream);

/* Expert-parallel layer object: the communicator and the exchange buffers of
 * one rank (sized for max_tokens tokens of K slots per call).
 *   momij_moe_ep_init: nccl_comm points to the caller's ncclComm_t (world
 *     ranks, this GPU current), or is NULL and unique_id (the 128 bytes of a
 *     ncclUniqueId, e.g. from momij_nccl_unique_id on rank 0, shared by the
 *     caller) makes a communicator owned by the object; world == 1 needs
 *     neither.  E % world == 0, max_tokens*K + 1 <= H/2 and
 *     world*(max_tokens*K + 1) <= MOMIJ_MAX_PAIRS.
 *   momij_moe_ep_forward: one MoE layer for this rank's M <= max_tokens
 *     tokens: routing from logits [M,E] (or the given inds/scores when logits
 *     is NULL), dispatch, exchange, the rank's experts (w_* hold experts
 *     [rank*E/world, (rank+1)*E/world)), exchange back, combine into y or
 *     resid_h -- the same bits as the single-GPU path.  Enqueued on `stream`
 *     only (no host synchronisation; capturable in a CUDA graph); every rank
 *     calls it with the same M.
 *   momij_moe_ep_status: synchronises `stream` and returns the layer's
 *     status (expert index, workspace or timeout errors of its kernels).
 * NCCL is loaded at run time (libnccl.so.2); MOMIJ_ERR_NCCL when missing.
 * Replaces: no counterpart in the reference (one GPU); the exchange sequence
 * of north-star config 4 behind one call, for a caller without Python. */
typedef struct momij_ep momij_ep_t;
int momij_nccl_unique_id(void* out_128_bytes);
int momij_moe_ep_init(void* nccl_comm, const void* unique_id, int rank, int world, int E, int H, int I,
                      int K, int max_tokens, int gs, float clamp, int dtype, momij_ep_t** out);
int momij_moe_ep_forward(momij_ep_t* ep, const float* logits, const int32_t* inds, const float* scores,
                         const void* x, const uint32_t* w_ug, const void* s_ug, const void* b_ug,
                         const uint32_t* w_dn, const void* s_dn, const void* b_dn, void* y, void* resid_h,
                         int M, momij_stream_t stream);
int momij_moe_ep_status(momij_ep_t* ep, momij_stream_t stream);
int momij_moe_ep_destroy(momij_ep_t* ep);

/* Per-kernel GPU timing.  While enabled, each launch made by the entry points
 * above is bracketed by two CUDA events on its stream (also when the stream
 * is being captured into a CUDA graph; the pair then times the latest replay).
 * momij_profile_read sums the recorded pairs of one kernel id (it waits for
 * their events); momij_profile_reset releases all pairs.
 * Replaces: the MOMIJ_PROFILE_MOE phase timers (MapleSeedlessMoE.swift:81-107)
 * and the Metal GPU timestamps of the MoE benches (SeedlessMetal.swift:
 * 1050-1069). */
enum momij_kernel_id {
    MOMIJ_KERNEL_PLAN = 0,    /* router and/or work plan */
    MOMIJ_KERNEL_UP = 1,      /* up||gate gather-GEMV + SwiGLU */
    MOMIJ_KERNEL_ROWS = 2,    /* gather-GEMV (down projection, gqmm2) */
    MOMIJ_KERNEL_COMBINE = 3, /* score-weighted combine */
    MOMIJ_KERNEL_LAYER = 4    /* fused decode layer: route + up + down + combine */
};
int momij_profile_enable(int on);
int momij_profile_read(int kernel_id, double* total_ms, int* launches);
int momij_profile_reset(void);

/* Phase trace of the fused decode-layer kernel: while a device buffer is set,
 * each launch (also when captured into a graph) takes the next slot of
 * (SM count x 16) int64 %globaltimer stamps, one row per CTA, written by the
 * CTA's thread 0 at its phase boundaries (start, after the previous kernel,
 * routed, planned, up tables, tokens encoded, up done, down prefetch issued,
 * grid barrier passed, act encoded, down done, counters added, combined).
 * NULL disables.  Counterpart: the reference's per-phase timers
 * (PhaseMs, SeedlessDecodeEngine.swift:69-77). */
int momij_layer_trace(void* device_buffer, size_t bytes);

/* Deterministic synthetic inputs (the generator of momij_b200/synth.py, bit
 * for bit): kind 0 = packed 2-bit codes (uint32 words), 1 = a*u + c with u
 * uniform in [0,1) rounded to dtype, 2 = Irwin-Hall normal rounded to dtype,
 * 3 = Irwin-Hall normal as fp32.  Element i of dst gets index start + i.
 * Test-input generation only; no counterpart in the reference. */
int momij_synth_fill(void* dst, int64_t n, int kind, float a, float c, uint64_t seed,
                     uint64_t stream_id, int64_t start, int dtype, momij_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* MOMIJ_MOE_H */
