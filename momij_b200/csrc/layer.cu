// layer.cu -- one MoE FFN layer for a single decode token in a single
// persistent kernel (one CTA per SM, launched cooperatively so that all CTAs
// are co-resident), on the warp-level integer tensor-core engine of
// gemv_core.cuh (digit planes of the token, 16 consumer warps that each
// stream, dequantise and multiply their own items).  Batches of 2..8 tokens
// take the tcgen05 kernel of decode.cu instead.
//
//   1. every CTA routes the token itself (momij's maple_route_top8,
//      SeedlessMetal.swift:2720-2791, in its reduction-tree tie order:
//      route_tokens) and builds the unit plan in shared memory;
//   2. up||gate phase over the CTA's slice of the (unit, row pair) space:
//      its weight loads are issued before the tokens are encoded; the
//      epilogue applies the staged clamped SwiGLU and writes act[pair, I];
//   3. the down phase's first weight stages are issued during the up phase's
//      last stages, *before* the grid barrier that makes act complete, so HBM
//      keeps streaming across the barrier;
//   4. down phase over the CTA's slice of the (unit, output row) space writes
//      down[pair, H] (each value an activation-dtype gather output);
//   5. the CTA that completes the last unit of a 64-row block combines it:
//      y = cast(sum_k float(down_k) * score_k) in k order (MapleMoE.swift:
//      76-78), or h = cast(h + cast(acc)) (maple_score_resid).
// The arithmetic is exactly that of the multi-kernel path (gemv_core.cuh,
// combine_kernel), so both produce the same bits.
//
// Waits on other CTAs (the grid barrier) are bounded (the host's spin limit):
// a CTA that gives up records MOMIJ_ERR_TIMEOUT in the workspace error word,
// still adds its completion counts (so every counter returns to zero) and
// writes no output.  A set stop flag (the reference's stopFlag) skips the
// streaming work the same way and reports MOMIJ_ERR_STOPPED.
#include "gemv_core.cuh"
#include "layer.cuh"
#include "route_core.cuh"

namespace momij {

namespace {

// Phase timestamp (ns, %globaltimer) of this CTA, when tracing is enabled.
__device__ __forceinline__ void stamp(const LayerArgs& a, int i) {
    if (a.trace && threadIdx.x == 0) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        a.trace[(size_t)blockIdx.x * kTracePointsDec + i] = (long long)t;
    }
}

// Grid barrier of the consumer threads (grid_barrier_thread by thread 0).
// Every CTA arrives; `wait` false (this CTA already failed) arrives only.
__device__ bool layer_grid_barrier(const LayerArgs& a, unsigned g0, bool wait, int* s_flag) {
    bar_sync(kBarConsumers, kConsumerThreads);
    if (threadIdx.x == 0) {
        const bool ok = grid_barrier_thread(reinterpret_cast<unsigned*>(a.ctrl + kCtrlArrive),
                                            reinterpret_cast<unsigned*>(a.ctrl + kCtrlGen), g0, a.spin_limit, wait) &&
                        wait;
        if (!ok) atomicExch(a.ctrl + kCtrlError, MOMIJ_ERR_TIMEOUT);
        __threadfence();
        *s_flag = ok;
    }
    bar_sync(kBarConsumers, kConsumerThreads);
    return *s_flag != 0;
}

// Sort the P pairs by (expert, pair) and cut each expert's run into units of
// <= tmax pairs; P <= 64, one warp (lanes take pairs lane and lane + 32).
// Writes s_units / s_sorted / *s_nunits and *s_bad (an index outside [0, E)).
__device__ void plan_warp(const int* s_inds, int P, int E, int tmax, int4* s_units, int* s_sorted,
                          int4* s_qinfo, int* s_nunits, int* s_bad) {
    const int lane = threadIdx.x & 31;
    int bad = 0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int p = lane + 32 * h;
        if (p < P) {
            const int e = s_inds[p];
            bad |= (e < 0 || e >= E);
            int less = 0, before = 0, same = 0;
            for (int j = 0; j < P; ++j) {
                const int ej = s_inds[j];
                less += ej < e;
                before += (ej == e) & (j < p);
                same += ej == e;
            }
            s_sorted[less + before] = p;
            s_qinfo[less + before] = make_int4(e, before, same, 0);
        }
    }
    bad = __any_sync(0xffffffffu, bad);
    __syncwarp();
    unsigned mask[2];
    int4 info[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int q = lane + 32 * h;
        info[h] = q < P ? s_qinfo[q] : make_int4(0, 1, 0, 0);
        mask[h] = __ballot_sync(0xffffffffu, q < P && info[h].y % tmax == 0);
    }
    const unsigned below = (1u << lane) - 1u;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int q = lane + 32 * h;
        if ((mask[h] >> lane) & 1u) {
            const int u = __popc(mask[0] & (h ? 0xffffffffu : below)) + (h ? __popc(mask[1] & below) : 0);
            s_units[u] = make_int4(info[h].x, q, min(tmax, info[h].z - info[h].y), 0);
        }
    }
    if (lane == 0) {
        *s_nunits = __popc(mask[0]) + __popc(mask[1]);
        *s_bad = bad;
    }
}

// Shared-memory tables of one phase for the CTA's slice [r0, r1) of the
// flattened (unit, row) space: tiles (local unit, first row, rows), the local
// unit table, each (local unit, j)'s pair and digit slot, and (slot mode 1)
// the list of vectors to encode.  Slot mode 0: slot = token (pair / K).
struct PhaseSmemTables {
    int4* tiles;
    int4* lunits;
    int* upair;
    int* uslot;
    int* vecs;
    int4* seg;   // per local unit: (first tile, row lo, row hi, first slot)
    int* count;  // [0] tiles, [1] vectors, [2] local units, [3] overflow
};

// One warp: cuts the CTA's slice [r0, r1) of the flattened (unit, row) space
// into unit segments (lane ul: local unit ul; at most 64 units) with
// exclusive prefix sums of their tiles and (slot mode 1) vectors.
__device__ void build_segments(int r0, int r1, int Ru, int TR, int tmax, int slot_mode,
                               const int4* s_units, const PhaseSmemTables& tb, const LayerArgs& a) {
    const int lane = threadIdx.x & 31;
    int nu = 0, over = 0, nt = 0, nv = 0;
    if (r0 < r1) {
        const int u_first = r0 / Ru, u_last = (r1 - 1) / Ru;
        nu = u_last - u_first + 1;
        if (nu > a.max_units || nu > 64) over = 1;
        for (int base = 0; base < nu && !over; base += 32) {
            const int ul = base + lane;
            int ntl = 0, nvl = 0, lo = 0, hi = 0;
            int4 un = make_int4(0, 0, 0, 0);
            if (ul < nu) {
                const int u = u_first + ul;
                lo = max(r0, u * Ru) - u * Ru;
                hi = min(r1, (u + 1) * Ru) - u * Ru;
                un = s_units[u];
                ntl = (hi - lo + TR - 1) / TR;
                nvl = slot_mode == 1 ? un.z : 0;
            }
            if (__any_sync(0xffffffffu, ul < nu && un.z > tmax)) over = 1;
            int it = ntl, iv = nvl;  // inclusive warp prefix sums
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int t2 = __shfl_up_sync(0xffffffffu, it, o), v2 = __shfl_up_sync(0xffffffffu, iv, o);
                if (lane >= o) {
                    it += t2;
                    iv += v2;
                }
            }
            if (ul < nu) {
                tb.seg[ul] = make_int4(nt + it - ntl, lo, hi, nv + iv - nvl);
                tb.lunits[ul] = un;
            }
            nt += __shfl_sync(0xffffffffu, it, 31);
            nv += __shfl_sync(0xffffffffu, iv, 31);
        }
        if (nt > a.max_tiles || (slot_mode == 1 && nv > a.max_vec)) over = 1;
    }
    if (lane == 0) {
        tb.count[0] = over ? 0 : nt;
        tb.count[1] = over ? 0 : nv;
        tb.count[2] = over ? 0 : nu;
        tb.count[3] = over;
    }
}

// Block-wide, after build_segments: the tiles (local unit, first row, rows)
// and each (local unit, j)'s pair and digit slot (slot mode 0: the token
// pair / K; 1: consecutive vectors, listed in vecs).
__device__ void fill_tables(int TR, int tmax, int K, int slot_mode, const int* s_sorted,
                            const PhaseSmemTables& tb) {
    const int nt = tb.count[0], nu = tb.count[2];
    for (int tau = threadIdx.x; tau < nt; tau += blockDim.x) {
        int ul = 0;
        while (ul + 1 < nu && tb.seg[ul + 1].x <= tau) ++ul;
        const int4 sg = tb.seg[ul];
        const int rs = sg.y + (tau - sg.x) * TR;
        tb.tiles[tau] = make_int4(ul, rs, min(TR, sg.z - rs), 0);
    }
    for (int it = threadIdx.x; it < nu * tmax; it += blockDim.x) {
        const int ul = it / tmax, j = it % tmax;
        const int4 un = tb.lunits[ul];
        if (j >= un.z) continue;
        const int pr = s_sorted[un.y + j];
        tb.upair[it] = pr;
        if (slot_mode == 0) {
            tb.uslot[it] = pr / K;
        } else {
            const int slot = tb.seg[ul].w + j;
            tb.uslot[it] = slot;
            tb.vecs[slot] = pr;
        }
    }
}

template <int DT, int TMAX>
struct ActOut {  // up||gate phase: staged SwiGLU -> act[pair, I]
    const int* upair;
    uint16_t* act;
    int I;
    float clamp;
    __device__ void operator()(const int4& tile, int j, int r, float up, float gate) const {
        act[(size_t)upair[tile.x * TMAX + j] * I + tile.y + r] = swiglu_staged<DT>(up, gate, clamp);
    }
};

template <int DT, int TMAX>
struct DownOut {  // down phase: down[pair, H]
    const int* upair;
    uint16_t* down;
    int H;
    __device__ void operator()(const int4& tile, int j, int r, float v, float) const {
        down[(size_t)upair[tile.x * TMAX + j] * H + tile.y + r] = Half<DT>::from_f(v);
    }
};

}  // namespace

template <int DT, int GS, int TMAX, int STAGES>
__global__ void __launch_bounds__(kLayerThreads, 1) moe_layer_kernel(const LayerArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ int s_nunits, s_bad, s_flag, s_nlast, s_nseg, s_stopped;
    __shared__ unsigned s_gen0;
    __shared__ int s_nan[8];
    __shared__ __align__(8) uint64_t s_sbar_up, s_sbar_dn;
    __shared__ int s_cnt_up[4], s_cnt_dn[4];
    __shared__ int s_last[kLayerMaxLastBlocks];
    __shared__ int2 s_seg[kLayerMaxLastBlocks];
    stamp(a, 0);
    const int tid = threadIdx.x;
    const int P = a.M * a.K;

    float* s_logits = reinterpret_cast<float*>(smem + a.off_logits);
    int* s_inds = reinterpret_cast<int*>(smem + a.off_inds);
    float* s_scores = reinterpret_cast<float*>(smem + a.off_scores);
    int* s_sorted = reinterpret_cast<int*>(smem + a.off_sorted);
    int* s_pflag = reinterpret_cast<int*>(smem + a.off_pflag);
    int4* s_units = reinterpret_cast<int4*>(smem + a.off_units);
    const PhaseSmemTables up_tb{reinterpret_cast<int4*>(smem + a.off_tiles_up),
                                reinterpret_cast<int4*>(smem + a.off_lunits_up),
                                reinterpret_cast<int*>(smem + a.off_upair_up),
                                reinterpret_cast<int*>(smem + a.off_uslot_up),
                                reinterpret_cast<int*>(smem + a.off_xvecs),
                                reinterpret_cast<int4*>(smem + a.off_seg_up), s_cnt_up};
    const PhaseSmemTables dn_tb{reinterpret_cast<int4*>(smem + a.off_tiles_dn),
                                reinterpret_cast<int4*>(smem + a.off_lunits_dn),
                                reinterpret_cast<int*>(smem + a.off_upair_dn),
                                reinterpret_cast<int*>(smem + a.off_uslot_dn),
                                reinterpret_cast<int*>(smem + a.off_vecs_dn),
                                reinterpret_cast<int4*>(smem + a.off_seg_dn), s_cnt_dn};
    float2* s_fs = reinterpret_cast<float2*>(smem + a.off_fs);
    uint8_t* s_dig = reinterpret_cast<uint8_t*>(smem + a.off_dig);
    float* s_red = reinterpret_cast<float*>(smem + a.off_red);
    unsigned char* s_ring = smem + a.off_stage;

    pdl_wait();  // the previous kernel on the stream (e.g. the layer before) is complete
    pdl_launch_dependents();
    stamp(a, 1);

    // ---- 1. token encoding (it does not depend on the routing), routing ----
    const int nlog = a.logits ? a.M * a.E : 0;
    const float lg0 = tid < nlog ? __ldcg(a.logits + tid) : 0.f;  // in flight during the encoding
    const int stop0 = (tid == 0 && a.stop) ? __ldcg(a.stop) : 0;
    // the grid barrier's generation before this call's round (read early, off the critical path)
    const unsigned gen0 = tid == 0 ? ld_acquire_u32(reinterpret_cast<const unsigned*>(a.ctrl + kCtrlGen)) : 0u;
    if (tid < a.M) up_tb.vecs[tid] = tid;
    if (tid < 8) s_nan[tid] = 0;
    __syncthreads();
    digitize<DT>(a.x, up_tb.vecs, a.M, a.H, s_dig, s_fs, kConsumerThreads);
    if (tid == 0) {
        s_stopped = stop0 != 0;
        s_gen0 = gen0;
    }
    if (tid < nlog) {
        s_logits[tid] = lg0;
        if (isnan(lg0)) s_nan[tid / a.E] = 1;
    }
    for (int i = tid + blockDim.x; i < nlog; i += blockDim.x) {
        const float v = __ldcg(a.logits + i);
        s_logits[i] = v;
        if (isnan(v)) s_nan[i / a.E] = 1;
    }
    if (!a.logits) {
        for (int i = tid; i < P; i += blockDim.x) {
            s_inds[i] = a.inds_in[i];
            s_scores[i] = a.scores_in[i];
        }
    }
    __syncthreads();
    stamp(a, 2);
    // selection (ends with a block barrier), then the plan (warp 0) beside the scores (warps 1..M)
    if (a.logits) route_tokens(s_logits, s_nan, a.M, a.E, a.K, 0, kLayerThreads, 0, s_inds, s_scores,
                               nullptr, false);
    if (tid < 32) {
        plan_warp(s_inds, P, a.E, TMAX, s_units, s_sorted, reinterpret_cast<int4*>(s_pflag), &s_nunits, &s_bad);
    } else if (a.logits && (tid >> 5) <= a.M) {
        const int m = (tid >> 5) - 1;
        route_scores_warp(s_logits + m * a.E, a.E, a.K, s_inds + m * a.K, s_scores + m * a.K);
    }
    __syncthreads();
    const bool ok = s_bad == 0;
    const bool stopped = s_stopped != 0;
    if (blockIdx.x == 0 && tid == 0)
        a.ctrl[kCtrlStatus] = ok ? (stopped ? MOMIJ_ERR_STOPPED : MOMIJ_OK) : MOMIJ_ERR_EXPERT_INDEX;
    if (!ok) return;  // uniform: every CTA sees the same indices
    stamp(a, 3);
    const int U = s_nunits;
    const int G = gridDim.x, bx = blockIdx.x;
    const int Ru = U * a.I, Rd = U * a.H;
    const int r0 = (int)((long long)Ru * bx / G), r1 = (int)((long long)Ru * (bx + 1) / G);
    const int d0 = (int)((long long)Rd * bx / G), d1 = (int)((long long)Rd * (bx + 1) / G);
    if (tid < 32) build_segments(r0, r1, a.I, 8, TMAX, 0, s_units, up_tb, a);
    else if (tid < 64) build_segments(d0, d1, a.H, 16, TMAX, 1, s_units, dn_tb, a);
    __syncthreads();
    fill_tables(8, TMAX, a.K, 0, s_sorted, up_tb);
    fill_tables(16, TMAX, a.K, 1, s_sorted, dn_tb);
    if (tid == 0 && (s_cnt_up[3] || s_cnt_dn[3]))  // capacity guard; unreachable for host-sized tables
        atomicExch(a.ctrl + kCtrlError, MOMIJ_ERR_WORKSPACE);
    __syncthreads();
    if (stopped && tid == 0) {  // no items; the down segments still feed the completion counters
        s_cnt_up[0] = 0;
        s_cnt_dn[0] = 0;
        s_cnt_dn[1] = 0;
    }
    __syncthreads();
    stamp(a, 4);

    const PhaseWeights up_w{a.w_ug, a.s_ug, a.b_ug, 2 * a.I, a.I, a.H};
    const PhaseWeights dn_w{a.w_dn, a.s_dn, a.b_dn, a.H, 0, a.I};
    // one scale/bias buffer: the down phase's first batch is issued once the
    // up phase's last batch is computed
    uint16_t* s_sb = reinterpret_cast<uint16_t*>(smem + a.off_sb);
    sb_init(&s_sbar_up);
    sb_init(&s_sbar_dn);
    const PhaseTables up_tabs{up_tb.tiles, up_tb.lunits, up_tb.uslot, s_cnt_up[0]};
    GemvPhase<DT, GS, kModeUpSwiglu, TMAX, STAGES> up(up_tabs, up_w, s_ring, 0, a.nK_up, s_sb, a.batch_up,
                                                      &s_sbar_up, TMAX == 1);
    const PhaseTables dn_tabs{dn_tb.tiles, dn_tb.lunits, dn_tb.uslot, s_cnt_dn[0]};
    GemvPhase<DT, GS, kModeRows, TMAX, STAGES> dn(dn_tabs, dn_w, s_ring, up.count, a.nK_dn, s_sb, a.batch_dn,
                                                  &s_sbar_dn, TMAX == 1);

    // One item sequence per warp: its up items, then its down items, which
    // start streaming during the up phase's last items.
    auto ahead_up = [&]() {
        if (up.li.n < up.count) up.load_next();
        else dn.load_next();
    };
    auto ahead_dn = [&]() { dn.load_next(); };
    __syncthreads();  // tables
    // the first batch's scales and biases go out before the first code items
    if (s_cnt_up[0] > 0) up.issue_sb(0, min(s_cnt_up[0], a.batch_up));
    up.prefetch(ahead_up);

    // ---- 2. up||gate phase --------------------------------------------------
    stamp(a, 5);
    if (bx == 0) {
        for (int i = tid; i < P; i += kConsumerThreads) {
            if (a.inds_out) a.inds_out[i] = s_inds[i];
            if (a.scores_out) a.scores_out[i] = s_scores[i];
        }
    }
    {
        ActOut<DT, TMAX> out{up_tb.upair, a.act, a.I, a.clamp};
        if (!up.consume(s_dig, s_fs, s_red, true, out, ahead_up) && tid == 0)
            atomicExch(a.ctrl + kCtrlError, MOMIJ_ERR_TIMEOUT);
    }
    if (s_cnt_dn[0] > 0) dn.issue_sb(0, min(s_cnt_dn[0], a.batch_dn));  // lands during the grid barrier
    stamp(a, 6);
    stamp(a, 7);

    // ---- 3/4. down phase: its stages are already streaming --------------------
    // the combine's completion counters start at zero whatever the workspace
    // held (a call of another batch size carves it differently): CTA 0 clears
    // them before the grid barrier that precedes every count
    if (bx == 0)
        for (int i = tid; i < (a.H + 63) / 64; i += kConsumerThreads) a.block_ctr[i] = 0u;
    const bool fine = layer_grid_barrier(a, s_gen0, true, &s_flag);
    if (!fine) {
        ring_quiesce();  // the down items issued before the barrier
        if (s_cnt_dn[0] > 0) dn.wait_sb();
    }
    stamp(a, 8);
    if (fine) {
        digitize<DT>(a.act, dn_tb.vecs, s_cnt_dn[1], a.I, s_dig, s_fs, kConsumerThreads);
        bar_sync(kBarConsumers, kConsumerThreads);
        stamp(a, 9);
        DownOut<DT, TMAX> out{dn_tb.upair, a.down, a.H};
        if (!dn.consume(s_dig, s_fs, s_red, true, out, ahead_dn) && tid == 0)
            atomicExch(a.ctrl + kCtrlError, MOMIJ_ERR_TIMEOUT);
    }
    ring_quiesce();
    __threadfence();  // down rows written by this thread, before the block counters below
    stamp(a, 10);

    // ---- 5. last-arriver combine per 64-row block ----------------------------
    // Segments (unit, 64-row block) of this CTA's slice, one counter add each,
    // issued by as many threads in parallel.
    if (tid == 0) {
        int ns = 0;
        const int nu = s_cnt_dn[2];
        for (int ul = 0; ul < nu; ++ul) {
            const int lo = dn_tb.seg[ul].y, hi = dn_tb.seg[ul].z;
            for (int b = lo >> 6; b <= (hi - 1) >> 6 && ns < kLayerMaxLastBlocks; ++b) {
                const int bs = b * 64, be = min(a.H, bs + 64);
                s_seg[ns++] = make_int2(b, min(be, hi) - max(bs, lo));
            }
        }
        s_nseg = ns;
        s_nlast = 0;
    }
    bar_sync(kBarConsumers, kConsumerThreads);
    if (tid < s_nseg) {
        const int2 sg = s_seg[tid];
        const int bs = sg.x * 64, be = min(a.H, bs + 64);
        const unsigned target = (unsigned)U * (unsigned)(be - bs);
        const unsigned old = atomicAdd(a.block_ctr + sg.x, (unsigned)sg.y);
        if (old + (unsigned)sg.y == target) s_last[atomicAdd(&s_nlast, 1)] = sg.x;
    }
    bar_sync(kBarConsumers, kConsumerThreads);
    stamp(a, 11);
    const int nlast = s_nlast;
    if (nlast) {
        __threadfence();
        const int rowsmax = 64;
        for (int it = tid; it < nlast * a.M * rowsmax; it += kConsumerThreads) {
            const int q = it / (a.M * rowsmax), rem = it % (a.M * rowsmax);
            const int m = rem / rowsmax, r = rem % rowsmax;
            const int n = s_last[q] * 64 + r;
            if (n >= a.H) continue;
            // per 8 slots: the loads first (independent), then the fp32 sum in
            // k order (a short loop keeps the kernel's code small)
            float acc = 0.f;
#pragma unroll 1
            for (int k0 = 0; k0 < a.K; k0 += 8) {
                float dv[8];
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    dv[k] = (k0 + k < a.K)
                                ? Half<DT>::to_f(__ldcg(a.down + (size_t)(m * a.K + k0 + k) * a.H + n))
                                : 0.f;
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    if (k0 + k < a.K) acc = fmaf(dv[k], s_scores[m * a.K + k0 + k], acc);
            }
            const size_t off = (size_t)m * a.H + n;
            if (!fine || stopped) continue;  // counters only
            if (a.h) {
                const float delta = Half<DT>::to_f(Half<DT>::from_f(acc));
                a.h[off] = Half<DT>::from_f(Half<DT>::to_f(a.h[off]) + delta);
            } else {
                a.y[off] = Half<DT>::from_f(acc);
            }
        }
        if (tid < nlast) a.block_ctr[s_last[tid]] = 0u;  // ready for the next call
    }
    stamp(a, 12);
}

#define MOMIJ_LAYER_INST(DT, GS, TM, ST) \
    template __global__ void moe_layer_kernel<DT, GS, TM, ST>(const LayerArgs);
#define MOMIJ_LAYER_INST_TM(DT, GS) MOMIJ_LAYER_INST(DT, GS, 1, layer_stages(1))
MOMIJ_LAYER_INST_TM(MOMIJ_DTYPE_BF16, 64)
MOMIJ_LAYER_INST_TM(MOMIJ_DTYPE_BF16, 128)
MOMIJ_LAYER_INST_TM(MOMIJ_DTYPE_F16, 64)
MOMIJ_LAYER_INST_TM(MOMIJ_DTYPE_F16, 128)

}  // namespace momij
