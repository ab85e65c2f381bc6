// decode.cu -- one MoE FFN layer for a decode / verify batch (M <= 8 tokens)
// in a single persistent kernel (one CTA per SM, launched cooperatively so
// that all CTAs are co-resident), on the tcgen05 tensor cores:
//
//   1. every CTA routes the M tokens itself (the reference's maple_route_top8,
//      SeedlessMetal.swift:2720-2791) and plans the distinct experts ("units",
//      <= T pairs each) and its own slices of both projections;
//   2. two producer warps stream the slices' packed codes into a ring of
//      16-KB shared-memory stages with TMA (one stage = one tile of <= 128
//      weight rows x one 128-byte chunk of K), up||gate rows first, then the
//      down rows -- the down weights keep streaming while the CTAs wait at
//      the grid barrier that makes the SwiGLU output complete;
//   3. 16 warps (4 warpgroups, one per 32-byte quarter of every chunk) turn
//      each 16-code word into four "class" words with one AND each
//      (w & (0x03030303 << 2p): byte i holds code 4i+p of the word times 4^p)
//      and store them to tensor memory as the A operand of
//      tcgen05.mma.kind::i8 (u8 x s8 -> s32): the tensor core then forms
//      exact integer dot products with the activations, which are split per
//      64-element group into four balanced base-256 digits of
//      x * 2^(21-E) * 4^(3-p) (the 4^(3-p) evens the classes out, so all
//      classes accumulate into the same columns);
//   4. one thread issues the MMAs (A in TMEM, B = digit matrix in shared
//      memory) and commits them to mbarriers; the same 16 warps read the
//      accumulators back (tcgen05.ld) and apply the per-group scale and bias
//      in fp32:  acc += s * (sum_d 256^(3-d) D_d) * 2^(E-27) + b * sum(x);
//   5. tiles end with the staged clamped SwiGLU (up||gate, act[pair, I]) or
//      the rounded down rows (down[pair, H]); the CTA that completes the last
//      unit of a 64-row block does the fp32 score-weighted combine in k order
//      into y, or into the residual stream h (maple_score_resid rounding).
//
// Every wait is bounded (MOMIJ_ERR_TIMEOUT in the workspace error word).
#include "decode.cuh"
#include "route_core.cuh"
#include "tc.cuh"

namespace momij {

namespace {

constexpr int kBarDec = 1;         // named barrier of the 512 dequantising threads
constexpr int kDrainLimit = 1 << 24;  // polls while draining copies / MMAs on an error path
constexpr int kGridSpinNs = 64;

__device__ __forceinline__ void dstamp(const DecodeArgs& a, int i) {
    if (a.trace && threadIdx.x == 0) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        a.trace[(size_t)blockIdx.x * kTracePointsDec + i] = (long long)t;
    }
}

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Grid barrier over gridDim.x co-resident CTAs by one thread: an arrival
// counter that the last arriver resets, and a generation word it then
// increments; the others wait for the generation to change.  The counter
// never exceeds the grid size and the generation is compared for change only,
// so neither wraps into a wrong state.  Every CTA arrives even when it later
// gives up waiting, so the counter is back at zero after every call.
__device__ bool grid_barrier_thread(unsigned* arrive, unsigned* gen, int limit, bool wait) {
    __threadfence();
    const unsigned g0 = ld_acquire_u32(gen);
    const unsigned old = atomicAdd(arrive, 1u);
    if (old == gridDim.x - 1) {
        atomicExch(arrive, 0u);
        __threadfence();
        atomicAdd(gen, 1u);
        return true;
    }
    if (!wait) return false;
    for (int it = 0; it < limit; ++it) {
        if (ld_acquire_u32(gen) != g0) return true;
        __nanosleep(kGridSpinNs);
    }
    return ld_acquire_u32(gen) != g0;
}

// ---- routing ---------------------------------------------------------------
// Order of two candidates of the reference's reduction tree (see
// route_topk_tree): a larger value wins; equal values (signed zeros compare
// equal) go to the expert whose bit-reversed index (over the tree's width) is
// smaller.  `rb` is the bit count of the width (8 for E <= 256).
__device__ __forceinline__ uint32_t route_value_key(float v) {
    uint32_t u = __float_as_uint(v);
    if ((u & 0x7fffffffu) == 0) u = 0;  // -0 == +0
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ uint32_t rev_index(int e, int rb) { return __brev((uint32_t)e) >> (32 - rb); }

// Ranks all M*E candidates block-wide (tokens without NaN logits): candidate
// (m, e) lands at position r = #{e' : e' wins over e} when r < K.
__device__ void route_ranks(const float* s_logits, const int* s_nan, int M, int E, int K, int rb,
                            int nthreads, int* s_inds) {
    const int ncand = M * E;
    for (int c = threadIdx.x; c < ncand; c += nthreads) {
        const int m = c / E, e = c - m * E;
        if (s_nan[m]) continue;
        const float* lg = s_logits + m * E;
        const uint32_t ok = route_value_key(lg[e]);
        const uint32_t re = rev_index(e, rb);
        int r = 0;
        for (int j = 0; j < E; ++j) {
            const uint32_t oj = route_value_key(lg[j]);
            r += (oj > ok) | ((oj == ok) & (rev_index(j, rb) < re));
        }
        if (r < K) s_inds[m * K + r] = e;
    }
}

// ---- work plan ------------------------------------------------------------
// Sort the P <= 64 pairs by (expert, pair) and cut each expert's run into
// units of <= tmax pairs; one warp.  s_units[u] = (expert, first sorted
// position, pairs, token mask).
__device__ void plan_units_warp(const int* s_inds, int P, int E, int K, int tmax, int4* s_units,
                                int* s_sorted, int4* s_qinfo, int* s_nunits, int* s_bad) {
    const int lane = threadIdx.x & 31;
    int bad = 0;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        const int p = lane + 32 * hh;
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
    for (int hh = 0; hh < 2; ++hh) {
        const int q = lane + 32 * hh;
        info[hh] = q < P ? s_qinfo[q] : make_int4(0, 1, 0, 0);
        mask[hh] = __ballot_sync(0xffffffffu, q < P && info[hh].y % tmax == 0);
    }
    const unsigned below = (1u << lane) - 1u;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        const int q = lane + 32 * hh;
        if ((mask[hh] >> lane) & 1u) {
            const int u = __popc(mask[0] & (hh ? 0xffffffffu : below)) + (hh ? __popc(mask[1] & below) : 0);
            const int cnt = min(tmax, info[hh].z - info[hh].y);
            int tm = 0;
            for (int j = 0; j < cnt; ++j) tm |= 1 << (s_sorted[q + j] / K);
            s_units[u] = make_int4(info[hh].x, q, cnt, tm);
        }
    }
    if (lane == 0) {
        *s_nunits = __popc(mask[0]) + __popc(mask[1]);
        *s_bad = bad;
    }
}

// Cuts this CTA's slice [r0, r1) of a phase's flattened (unit, row) space
// into tiles (unit, first row, rows <= tile_rows) that do not cross units.
__device__ int make_tiles(int r0, int r1, int rows_per_unit, int tile_rows, int4* tiles, int max_tiles) {
    int nt = 0;
    for (int r = r0; r < r1;) {
        const int u = r / rows_per_unit, j = r - u * rows_per_unit;
        const int n = min(tile_rows, min(r1 - r, rows_per_unit - j));
        if (nt < max_tiles) tiles[nt] = make_int4(u, j, n, 0);
        ++nt;
        r += n;
    }
    return nt;
}

// ---- digit operand (B) -------------------------------------------------------
// B of group g (dec_b_group_bytes(N) bytes): MMA half h (code classes 2h,
// 2h+1) at h * 32N; N rows x 32 K-bytes, K-major, 8x16-byte core matrices
// (row group at +256, K half at +128).  Column n = gl*4T' + v*4 + d, where
// gl is the group's slot in its accumulator pack, v the vector, d the digit;
// K-byte k = 4c + b with column c = 4(p & 1) + i <-> element 16i + 4b + p.
__device__ __forceinline__ int b_off(int N, int h, int n, int k) {
    return h * 32 * N + (n >> 3) * 256 + (k >> 4) * 128 + (n & 7) * 16 + (k & 15);
}
// Slot of group g in its accumulator pack of GP groups: the packs of a
// warpgroup hold its consecutive groups (two per 8-group chunk).
__device__ __forceinline__ int pack_slot(int g, int GP) { return (2 * (g >> 3) + (g & 1)) & (GP - 1); }

// Balanced base-256 digits of |y| < 2^29: y = 2^24 d0 + 2^16 d1 + 2^8 d2 + d3.
__device__ __forceinline__ void split4(int y, int (&d)[4]) {
    d[3] = ((y + 128) & 255) - 128;
    int t = (y - d[3]) >> 8;
    d[2] = ((t + 128) & 255) - 128;
    t = (t - d[2]) >> 8;
    d[1] = ((t + 128) & 255) - 128;
    d[0] = (t - d[1]) >> 8;
}

// Writes the digits of vectors src[v] (row length Kd, `nvec` of them, vector
// v in column set v) into B (groups [0, Kd/64)) and their per-group factors
// fs[v * nG + g] = (2^(E-27), sum of the group).  Eight lanes per (vector,
// group); `nthreads` threads from thread 0 take part.  Loads bypass L1 (the
// vectors may have been written by other CTAs).
template <int DT>
__device__ void digitize_b(const uint16_t* const* src, int nvec, int Kd, int N, int T, unsigned char* B,
                           float2* fs, int nthreads) {
    const int nG = Kd >> 6;
    const int GP = N / (4 * T);
    const int total = nvec * nG * 8;
    const int lane = threadIdx.x & 31;
    const int gbytes = dec_b_group_bytes(N);
    for (int base = (threadIdx.x & ~31); base < total; base += nthreads) {
        const int idx = base + lane;
        const bool valid = idx < total;
        const int vg = idx >> 3, sub = idx & 7;
        const int v = valid ? vg / nG : 0, g = valid ? vg - v * nG : 0;
        float xv[8];
        float mx = 0.f, sum = 0.f;
        if (valid) {
            const uint4 raw = __ldcg(reinterpret_cast<const uint4*>(src[v] + (size_t)g * 64 + sub * 8));
            const uint32_t r[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                xv[2 * i] = Half<DT>::to_f(static_cast<uint16_t>(r[i] & 0xffffu));
                xv[2 * i + 1] = Half<DT>::to_f(static_cast<uint16_t>(r[i] >> 16));
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                mx = fmaxf(mx, fabsf(xv[i]));
                sum += xv[i];
            }
        }
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            sum += __shfl_xor_sync(0xffffffffu, sum, o);
        }
        if (!valid) continue;
        int E = (mx > 0.f) ? ilogbf(mx) : 0;
        E = max(E, -100);
        const float scale = ldexpf(1.f, 21 - E);
        unsigned char* Bg = B + (size_t)g * gbytes;
        const int nb = pack_slot(g, GP) * 4 * T + v * 4;
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            const int e = sub * 8 + t;
            const int i = e >> 4, b = (e >> 2) & 3, p = e & 3;
            const int h = p >> 1, c = 4 * (p & 1) + i, k = 4 * c + b;
            const int X = __float2int_rn(xv[t] * scale);
            int d[4];
            split4(X << (2 * (3 - p)), d);
#pragma unroll
            for (int dd = 0; dd < 4; ++dd) Bg[b_off(N, h, nb + dd, k)] = static_cast<unsigned char>(d[dd] & 0xff);
        }
        if (sub == 0) fs[v * nG + g] = make_float2(ldexpf(1.f, E - 27), sum);
    }
}


// Warp-uniform bounded wait: every lane polls, and the warp leaves together
// (all lanes saw the phase) or gives up together.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, int limit, const volatile int* abort) {
    for (int it = 0; it < limit; ++it) {
        if (__all_sync(0xffffffffu, mbar_try_wait(bar, parity))) return true;
        if ((it & 255) == 255 && __any_sync(0xffffffffu, *abort != 0)) return false;
    }
    return false;
}
// Bounded wait that ignores the abort flag (draining copies and MMAs in flight).
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
    for (int it = 0; it < kDrainLimit; ++it)
        if (mbar_try_wait(bar, parity)) return;
}

struct DecShared {
    int inds[kDecMaxPairs];
    float scores[kDecMaxPairs];
    int sorted[kDecMaxPairs];
    int4 qinfo[kDecMaxPairs];
    int4 units[kDecMaxPairs];
    int4 tiles_up[kDecMaxTiles];
    int4 tiles_dn[kDecMaxTiles];
    int2 seg[kDecMaxLastBlocks];
    int last[kDecMaxLastBlocks];
    int nan_tok[8];
    const uint16_t* vec_ptr[16];
    int nunits, bad, nt_up, nt_dn, udn0, nudn, nseg, nlast, flag, abort, stopped;
    uint32_t tmem;
    alignas(8) uint64_t full[kDecMaxStages];
    alignas(8) uint64_t empty[kDecMaxStages];
    alignas(8) uint64_t a_full[4][2];
    alignas(8) uint64_t a_empty[4][2];
    alignas(8) uint64_t d_full[4][4];
    alignas(8) uint64_t d_empty[4][4];
    alignas(8) uint64_t drain;
};

}  // namespace

template <int DT, int GS, int T>
__global__ void __launch_bounds__(kDecThreadsAll, 1) moe_decode_kernel(const __grid_constant__ DecodeArgs a) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ DecShared S;
    dstamp(a, 0);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int P = a.M * a.K;
    constexpr int N = dec_mma_n(T), GP = N / (4 * T), ND = 64 / N;
    const int nthreads = blockDim.x;
    volatile int* abort_flag = &S.abort;

    // ---- set-up (independent of the previous kernel) ---------------------------
    if (warp == 0) tmem_alloc(&S.tmem, kDecTmemCols);
    if (tid == 0) {
        for (int s = 0; s < a.stages; ++s) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.empty[s], kDecWarps);
        }
        for (int w = 0; w < 4; ++w) {
            for (int s = 0; s < 2; ++s) {
                mbar_init(&S.a_full[w][s], 4);
                mbar_init(&S.a_empty[w][s], 1);
            }
            for (int s = 0; s < 4; ++s) {
                mbar_init(&S.d_full[w][s], 1);
                mbar_init(&S.d_empty[w][s], 4);
            }
        }
        mbar_init(&S.drain, 1);
        mbar_fence_init();
        S.abort = 0;
        S.stopped = 0;
    }
    float* s_logits = reinterpret_cast<float*>(smem + a.off_logits);
    unsigned char* s_B = smem + a.off_b;
    float2* s_fs = reinterpret_cast<float2*>(smem + a.off_fs);
    uint32_t* s_sb = reinterpret_cast<uint32_t*>(smem + a.off_sb);  // scale/bias words; tile-end partials
    float* s_red = reinterpret_cast<float*>(smem + a.off_sb);
    unsigned char* s_ring = smem + a.off_ring;
    tc_before_sync();
    __syncthreads();
    tc_after_sync();
    const uint32_t tmem = S.tmem;

    // ---- routing and plan (after the previous kernel: logits may be its output)
    pdl_wait();
    pdl_launch_dependents();
    dstamp(a, 1);
    if (tid == 0 && a.stop && __ldcg(a.stop) != 0) S.stopped = 1;
    const int nlog = a.logits ? a.M * a.E : 0;
    if (tid < 8) S.nan_tok[tid] = 0;
    __syncthreads();
    // A set stop flag (the reference's stopFlag, read once per CTA) skips the
    // streaming work; the CTA still arrives at the grid barrier and adds its
    // completion counts, so a flag raised while CTAs start leaves the
    // workspace consistent for the next call.
    const bool stopped = S.stopped != 0;
    for (int i = tid; i < nlog; i += nthreads) {
        const float v = __ldcg(a.logits + i);
        s_logits[i] = v;
        if (isnan(v)) S.nan_tok[i / a.E] = 1;
    }
    if (!a.logits) {
        for (int i = tid; i < P; i += nthreads) {
            S.inds[i] = __ldcg(a.inds_in + i);
            S.scores[i] = __ldcg(a.scores_in + i);
        }
    }
    __syncthreads();
    if (a.logits) {
        const int rb = 31 - __clz(route_tree_width(a.E));
        route_ranks(s_logits, S.nan_tok, a.M, a.E, a.K, rb, nthreads, S.inds);
        if (warp < a.M && S.nan_tok[warp])  // NaN logits: the reference's tree, stage by stage
            route_topk_tree<8>(s_logits + warp * a.E, a.E, a.K, S.inds + warp * a.K);
        __syncthreads();
    }
    // plan (warp 0) while warps 1..M compute the routing scores
    if (warp == 0) {
        plan_units_warp(S.inds, P, a.E, a.K, T, S.units, S.sorted, S.qinfo, &S.nunits, &S.bad);
    } else if (a.logits && warp <= a.M) {
        const int m = warp - 1;
        route_scores_warp(s_logits + m * a.E, a.E, a.K, S.inds + m * a.K, S.scores + m * a.K);
    }
    __syncthreads();
    const bool ok = S.bad == 0;
    if (blockIdx.x == 0 && tid == 0) a.ctrl[kCtrlStatus] = ok ? MOMIJ_OK : MOMIJ_ERR_EXPERT_INDEX;
    if (stopped && ok && tid == 0) a.ctrl[kCtrlStatus] = MOMIJ_ERR_STOPPED;
    if (!ok) {  // uniform: every CTA sees the same indices
        if (warp == 0) tmem_dealloc(tmem, kDecTmemCols);
        return;
    }
    dstamp(a, 2);
    const int U = S.nunits;
    const int G = gridDim.x, bx = blockIdx.x;
    {
        const long long n8u = (long long)U * a.I / 8, n8d = (long long)U * a.H / 8;
        const int r0 = (int)(n8u * bx / G) * 8, r1 = (int)(n8u * (bx + 1) / G) * 8;
        const int d0 = (int)(n8d * bx / G) * 8, d1 = (int)(n8d * (bx + 1) / G) * 8;
        if (tid == 0) {
            S.nt_up = make_tiles(r0, r1, a.I, 64, S.tiles_up, kDecMaxTiles);
            S.nt_dn = make_tiles(d0, d1, a.H, 128, S.tiles_dn, kDecMaxTiles);
            S.udn0 = d0 < d1 ? d0 / a.H : 0;
            S.nudn = d0 < d1 ? (d1 - 1) / a.H - d0 / a.H + 1 : 0;
            if (S.nt_up > kDecMaxTiles || S.nt_dn > kDecMaxTiles || S.nudn > 2) {
                atomicExch(a.ctrl + kCtrlError, MOMIJ_ERR_WORKSPACE);  // host-sized; unreachable
                S.nt_up = S.nt_dn = 0;
                S.nudn = 0;
            }
        }
        if (bx == 0) {
            for (int i = tid; i < P; i += nthreads) {
                if (a.inds_out) a.inds_out[i] = S.inds[i];
                if (a.scores_out) a.scores_out[i] = S.scores[i];
            }
        }
    }
    __syncthreads();
    dstamp(a, 3);

    const int nG_up = a.H >> 6, nG_dn = a.I >> 6;
    const int nC_up = (nG_up + 7) >> 3, nC_dn = (nG_dn + 7) >> 3;
    // tiles streamed and computed (none when stopped); nt_dn_all also feeds the combine counts
    const int nt_up = stopped ? 0 : S.nt_up, nt_dn = stopped ? 0 : S.nt_dn, nt_dn_all = S.nt_dn;
    const int S_ = a.stages;

    if (warp >= kDecWarps && warp < kDecWarps + kDecProducers) {
        // ---- TMA producers: item i (phase, tile, chunk) fills stage i % S_; --------
        // ---- producer i % 2 (S_ is even, so a stage always has the same producer)
        if (lane == 0) {
            const int p = warp - kDecWarps;
            int item = 0;
            int issued_last[kDecMaxStages];
            for (int s = 0; s < kDecMaxStages; ++s) issued_last[s] = -1;
            bool okp = true;
            for (int ph = 0; ph < 2 && okp; ++ph) {
                const int nt = ph ? nt_dn : nt_up, nC = ph ? nC_dn : nC_up;
                const int4* tiles = ph ? S.tiles_dn : S.tiles_up;
                const CUtensorMap* maps = ph ? a.map_dn : a.map_ug;
                for (int t = 0; t < nt && okp; ++t) {
                    const int4 tl = tiles[t];
                    const int e = S.units[tl.x].x;
                    for (int c = 0; c < nC; ++c, ++item) {
                        if ((item & 1) != p) continue;
                        const int s = item % S_, use = item / S_;
                        if (use > 0 && !mbar_wait_bounded(&S.empty[s], (use - 1) & 1, a.spin_limit, abort_flag)) {
                            okp = false;
                            break;
                        }
                        const int nparts = ph ? 1 : 2;
                        mbar_expect_tx(&S.full[s], (uint32_t)(nparts * tl.z * 128));
                        const uint32_t st = smem_u32(s_ring + (size_t)s * kDecStageBytes);
                        for (int part = 0; part < nparts; ++part) {
                            // up||gate: up rows at stage rows [0, n), gate rows at [64, 64 + n)
                            int grow = ph ? e * a.H + tl.y : e * 2 * a.I + part * a.I + tl.y;
                            int srow = part * 64;
                            int left = tl.z;
                            while (left > 0) {
                                const int bi = left >= 64 ? 0 : left >= 32 ? 1 : left >= 16 ? 2 : 3;
                                const int br = 64 >> bi;
                                tma_load_2d(st + srow * 128, &maps[bi], c * 128, grow, &S.full[s]);
                                grow += br;
                                srow += br;
                                left -= br;
                            }
                        }
                        issued_last[s] = use;
                    }
                }
            }
            if (!okp) {
                *abort_flag = 1;
                atomicExch(a.ctrl + kCtrlError, MOMIJ_ERR_TIMEOUT);
            }
            // every issued stage has landed before the CTA can exit
            for (int s = 0; s < S_; ++s)
                if (issued_last[s] >= 0) mbar_drain(&S.full[s], issued_last[s] & 1);
        }
    } else if (warp == kDecWarps + kDecProducers) {
        // ---- MMA issuer ------------------------------------------------------
        if (lane == 0) {
            int ua[4] = {0, 0, 0, 0}, ud[4] = {0, 0, 0, 0};
            const uint32_t idesc = idesc_u8s8(N);
            const int gbytes = dec_b_group_bytes(N);
            bool okm = true;
            for (int ph = 0; ph < 2 && okm; ++ph) {
                const int nt = ph ? nt_dn : nt_up, nC = ph ? nC_dn : nC_up, nG = ph ? nG_dn : nG_up;
                const int4* tiles = ph ? S.tiles_dn : S.tiles_up;
                for (int t = 0; t < nt && okm; ++t) {
                    const int4 tl = tiles[t];
                    const uint32_t bbase =
                        smem_u32(s_B) + (ph ? (uint32_t)((tl.x - S.udn0) * nG_dn * gbytes) : 0u);
                    int q[4] = {0, 0, 0, 0};
                    int nGw[4];
#pragma unroll
                    for (int w = 0; w < 4; ++w) {
                        int n = 0;
                        for (int c = 0; c < nC; ++c) n += min(2, max(0, min(8, nG - 8 * c) - 2 * w));
                        nGw[w] = n;
                    }
                    for (int c = 0; c < nC && okm; ++c) {
                        const int ngc = min(8, nG - 8 * c);
#pragma unroll
                        for (int w = 0; w < 4; ++w) {
                            const int cnt = min(2, max(0, ngc - 2 * w));
                            if (cnt == 0 || !okm) continue;
                            const int slot = ua[w] & 1;
                            if (!mbar_wait_bounded(&S.a_full[w][slot], (ua[w] >> 1) & 1, a.spin_limit, abort_flag)) {
                                okm = false;
                                continue;
                            }
                            tc_after_sync();
                            const uint32_t tA = tmem + w * 128 + slot * 32;
                            for (int tt = 0; tt < cnt && okm; ++tt) {
                                const int g = 8 * c + 2 * w + tt;
                                const int qq = q[w]++;
                                const int gl = qq & (GP - 1);
                                const int buf = ud[w] % ND;
                                if (gl == 0 && ud[w] >= ND) {
                                    if (!mbar_wait_bounded(&S.d_empty[w][buf], ((ud[w] - ND) / ND) & 1, a.spin_limit,
                                                           abort_flag)) {
                                        okm = false;
                                        continue;
                                    }
                                    tc_after_sync();
                                }
                                const uint32_t tD = tmem + w * 128 + 64 + buf * N;
#pragma unroll
                                for (int h = 0; h < 2; ++h) {
                                    const uint64_t bd =
                                        sdesc_noswz(bbase + (uint32_t)(g * gbytes + h * 32 * N), 128, 256);
                                    mma_i8_ta(tD, tA + tt * 16 + h * 8, bd, idesc, (gl | h) ? 1u : 0u);
                                }
                                if (gl == GP - 1 || qq == nGw[w] - 1) {
                                    mma_commit(&S.d_full[w][buf]);
                                    ++ud[w];
                                }
                            }
                            if (!okm) continue;
                            mma_commit(&S.a_empty[w][slot]);
                            ++ua[w];
                        }
                    }
                }
            }
            if (!okm) {
                *abort_flag = 1;
                atomicExch(a.ctrl + kCtrlError, MOMIJ_ERR_TIMEOUT);
            }
            // every MMA issued has completed before the tensor memory is released
            mma_commit(&S.drain);
            mbar_drain(&S.drain, 0);
        }
    } else {
        // ---- 16 dequantising warps: warpgroup wg takes 16-byte chunks 2wg, 2wg+1 --
        // ---- (groups 8c + 2wg, 8c + 2wg + 1) of every stage; lane L = tile row ----
        const int wg = warp >> 2, wq = warp & 3, L = wq * 32 + lane;
        const uint32_t lane_off = tmem_lane_base(warp);
        const uint32_t tA0 = tmem + wg * 128, tD0 = tmem + wg * 128 + 64;
        const int gbytes = dec_b_group_bytes(N);
        int item = 0, ua = 0, ud = 0;
        bool okd = true;

        // the up phase's digit operand: every token's x (vector v = token)
        for (int i = tid; i < a.b_bytes / 16; i += kDecThreads)
            reinterpret_cast<uint4*>(s_B)[i] = make_uint4(0u, 0u, 0u, 0u);
        if (tid < a.M) S.vec_ptr[tid] = a.x + (size_t)tid * a.H;
        bar_sync(kBarDec, kDecThreads);
        if (!stopped) digitize_b<DT>(S.vec_ptr, a.M, a.H, N, T, s_B, s_fs, kDecThreads);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        bar_sync(kBarDec, kDecThreads);
        dstamp(a, 4);

        for (int ph = 0; ph < 2; ++ph) {
            const int nt = ph ? nt_dn : nt_up, nC = ph ? nC_dn : nC_up, nG = ph ? nG_dn : nG_up;
            const int4* tiles = ph ? S.tiles_dn : S.tiles_up;
            const uint16_t* sc = ph ? a.s_dn : a.s_ug;
            const uint16_t* bc = ph ? a.b_dn : a.b_ug;
            const int Nrows = ph ? a.H : 2 * a.I;
            const int nsb = (ph ? a.I : a.H) / GS;
            if (ph == 1) {
                // act complete on every CTA: grid barrier, then the down phase's digits
                __threadfence();
                bar_sync(kBarDec, kDecThreads);
                dstamp(a, 6);
                if (tid == 0) {
                    // every CTA arrives (also after an error), so the counter returns to zero
                    const bool wait = !*abort_flag;
                    S.flag = grid_barrier_thread(reinterpret_cast<unsigned*>(a.ctrl + kCtrlArrive),
                                                 reinterpret_cast<unsigned*>(a.ctrl + kCtrlGen), a.spin_limit,
                                                 wait) && wait;
                }
                bar_sync(kBarDec, kDecThreads);
                if (!S.flag) okd = false;
                dstamp(a, 7);
                if (okd) {
                    for (int i = tid; i < a.b_bytes / 16; i += kDecThreads)
                        reinterpret_cast<uint4*>(s_B)[i] = make_uint4(0u, 0u, 0u, 0u);
                }
                bar_sync(kBarDec, kDecThreads);
                for (int us = 0; us < S.nudn && okd && !stopped; ++us) {
                    const int4 un = S.units[S.udn0 + us];
                    if (tid < un.z) S.vec_ptr[tid] = a.act + (size_t)S.sorted[un.y + tid] * a.I;
                    bar_sync(kBarDec, kDecThreads);
                    digitize_b<DT>(S.vec_ptr, un.z, a.I, N, T, s_B + (size_t)us * nG_dn * gbytes,
                                   s_fs + (size_t)us * T * nG_dn, kDecThreads);
                    bar_sync(kBarDec, kDecThreads);
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                bar_sync(kBarDec, kDecThreads);
                dstamp(a, 8);
            }
            for (int t = 0; t < nt; ++t) {
                const int4 tl = tiles[t];
                const int4 un = S.units[tl.x];
                const int e = un.x;
                // the thread's weight row: up rows in lanes [0, 64), gate rows in [64, 128)
                const bool rvalid = ph ? (L < tl.z) : ((L & 63) < tl.z);
                const int grow = ph ? tl.y + L : ((L < 64) ? tl.y + L : a.I + tl.y + (L - 64));
                const size_t srow = ((size_t)e * Nrows + (rvalid ? grow : 0)) * nsb;
                const uint16_t* srp = sc + srow;
                const uint16_t* brp = bc + srow;
                // vectors of this tile: up -- the unit's tokens; down -- its pairs
                const int vmask = ph ? ((1 << un.z) - 1) : un.w;
                const float2* fsb = ph ? s_fs + (size_t)(tl.x - S.udn0) * T * nG_dn : s_fs;
                float acc[8];
#pragma unroll
                for (int v = 0; v < 8; ++v) acc[v] = 0.f;
                int nGw = 0;
                for (int c = 0; c < nC; ++c) nGw += min(2, max(0, min(8, nG - 8 * c) - 2 * wg));
                const int npk = (nGw + GP - 1) / GP;
                const int item0 = item;
                int pk_done = 0;  // packs of this tile whose epilogue ran
                int q = 0;        // groups of this tile dequantised by the warpgroup

                // epilogue of pack k of this tile (groups [k GP, min((k+1) GP, nGw)) of the warpgroup)
                auto epilogue = [&](int k) {
                    const int buf = ud % ND;
                    if (okd) okd = mbar_wait_warp(&S.d_full[wg][buf], (ud / ND) & 1, a.spin_limit, abort_flag);
                    ++ud;
                    if (!okd) return;
                    tc_after_sync();
                    uint32_t d0[16], d1[16];
                    tmem_ld16_nowait(tD0 + buf * N + lane_off, d0);
                    if (N == 32) tmem_ld16_nowait(tD0 + buf * N + 16 + lane_off, d1);
                    tmem_ld_wait();
                    tc_before_sync();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&S.d_empty[wg][buf]);
                    const int q0 = k * GP, q1 = min(q0 + GP, nGw);
#pragma unroll
                    for (int gl = 0; gl < 4; ++gl) {
                        const int qq = q0 + gl;
                        if (gl >= GP || qq >= q1) continue;
                        const int g = 8 * (qq >> 1) + 2 * wg + (qq & 1);
                        // this group's scale and bias words (copied at its chunk's dequantisation)
                        const int rp = ((item0 + (qq >> 1)) & 3) * 4 + wg;
                        const uint32_t sw = s_sb[(rp * 2 + 0) * 128 + L], bw = s_sb[(rp * 2 + 1) * 128 + L];
                        const int hs = (GS == 64) ? (qq & 1) : (wg & 1);
                        const float s = Half<DT>::to_f((uint16_t)(sw >> (16 * hs)));
                        const float b = Half<DT>::to_f((uint16_t)(bw >> (16 * hs)));
#pragma unroll
                        for (int v = 0; v < 8; ++v) {
                            if (v < T && ((vmask >> v) & 1)) {
                                const int nb = gl * 4 * T + v * 4;  // < 16 for T <= 4; < 32 for T = 8
                                int D[4];
#pragma unroll
                                for (int dd = 0; dd < 4; ++dd) {
                                    const int col = nb + dd;
                                    D[dd] = (int)(col < 16 ? d0[col & 15] : d1[col & 15]);
                                }
                                const float f =
                                    fmaf((float)D[0], 16777216.f, fmaf((float)D[1], 65536.f, (float)(D[2] * 256 + D[3])));
                                const float2 fsv = fsb[v * nG + g];
                                acc[v] += fmaf(s, f * fsv.x, b * fsv.y);
                            }
                        }
                    }
                };

                for (int c = 0; c < nC; ++c, ++item) {
                    const int s = item % S_;
                    if (okd) okd = mbar_wait_warp(&S.full[s], (item / S_) & 1, a.spin_limit, abort_flag);
                    const int cnt = min(2, max(0, min(8, nG - 8 * c) - 2 * wg));
                    if (cnt > 0 && okd) {
                        // scale and bias words of the chunk's two groups, for the epilogue
                        {
                            const int rp = (item & 3) * 4 + wg;
                            const int gw = (GS == 64) ? 8 * c + 2 * wg : ((8 * c + 2 * wg) / 2) & ~1;
                            cp_async4(smem_u32(s_sb + (rp * 2 + 0) * 128 + L), srp + gw, rvalid);
                            cp_async4(smem_u32(s_sb + (rp * 2 + 1) * 128 + L), brp + gw, rvalid);
                        }
                        const unsigned char* row = s_ring + (size_t)s * kDecStageBytes + L * 128;
                        uint4 raw[2];
#pragma unroll
                        for (int tt = 0; tt < 2; ++tt)
                            raw[tt] = tt < cnt ? *reinterpret_cast<const uint4*>(row + (((2 * wg + tt) ^ (L & 7)) << 4))
                                               : make_uint4(0u, 0u, 0u, 0u);
                        const int slot = ua & 1;
                        if (ua >= 2) okd = mbar_wait_warp(&S.a_empty[wg][slot], ((ua - 2) >> 1) & 1, a.spin_limit, abort_flag);
                        if (okd) {
                            tc_after_sync();
#pragma unroll
                            for (int tt = 0; tt < 2; ++tt) {
                                if (tt < cnt) {
                                    const uint32_t wv[4] = {raw[tt].x, raw[tt].y, raw[tt].z, raw[tt].w};
                                    uint32_t m[16];
#pragma unroll
                                    for (int p = 0; p < 4; ++p)
#pragma unroll
                                        for (int i = 0; i < 4; ++i) m[4 * p + i] = wv[i] & (0x03030303u << (2 * p));
                                    tmem_st16(tA0 + slot * 32 + tt * 16 + lane_off, m);
                                }
                            }
                            tmem_st_wait();
                            tc_before_sync();
                            __syncwarp();
                            if (lane == 0) mbar_arrive(&S.a_full[wg][slot]);
                        }
                        ++ua;
                    }
                    cp_async_commit();
                    q += cnt;
                    __syncwarp();
                    if (lane == 0 && okd) mbar_arrive(&S.empty[s]);
                    // packs closed before this chunk's groups: their MMAs were issued already
                    const int closed = (q - cnt) / GP;
                    if (pk_done < closed) cp_async_wait<1>();
                    while (pk_done < closed) epilogue(pk_done++);
                }
                cp_async_wait<0>();
                while (pk_done < npk) epilogue(pk_done++);
                // ---- tile end: warpgroup partials -> ((w0 + w1) + (w2 + w3)) ------
                // (the partials reuse the scale/bias buffer: no copy is in flight now)
                bar_sync(kBarDec, kDecThreads);
#pragma unroll
                for (int v = 0; v < 8; ++v)
                    if (v < T && ((vmask >> v) & 1)) s_red[((size_t)wg * T + v) * 128 + L] = acc[v];
                bar_sync(kBarDec, kDecThreads);
                if (okd) {
                    const size_t st = (size_t)T * 128;
                    auto red_sum = [&](int v, int l) {
                        const float* r = s_red + (size_t)v * 128 + l;
                        return (r[0] + r[st]) + (r[2 * st] + r[3 * st]);
                    };
                    if (ph == 0) {
                        for (int i = tid; i < un.z * 64; i += kDecThreads) {
                            const int j = i >> 6, l = i & 63;
                            if (l >= tl.z) continue;
                            const int pr = S.sorted[un.y + j];
                            const int m = pr / a.K;
                            a.act[(size_t)pr * a.I + tl.y + l] =
                                swiglu_staged<DT>(red_sum(m, l), red_sum(m, l + 64), a.clamp);
                        }
                    } else {
                        for (int i = tid; i < un.z * 128; i += kDecThreads) {
                            const int j = i >> 7, l = i & 127;
                            if (l >= tl.z) continue;
                            const int pr = S.sorted[un.y + j];
                            a.down[(size_t)pr * a.H + tl.y + l] = Half<DT>::from_f(red_sum(j, l));
                        }
                    }
                }
                bar_sync(kBarDec, kDecThreads);
            }
            if (ph == 0) dstamp(a, 5);
        }
        // a warp that gave up makes the others give up at their next wait
        if (!okd) *abort_flag = 1;
        bar_sync(kBarDec, kDecThreads);
        const bool all_ok = !*abort_flag;
        if (!all_ok && tid == 0) atomicExch(a.ctrl + kCtrlError, MOMIJ_ERR_TIMEOUT);
        dstamp(a, 9);

        // ---- last-arriver combine per 64-row block --------------------------------
        // (the counts are added also after an error or a stop, so that every
        // counter returns to zero; the status word then flags the output)
        {
            __threadfence();  // down rows written by this thread, before the block counters
            bar_sync(kBarDec, kDecThreads);
            if (tid == 0) {
                int ns = 0;
                for (int t = 0; t < nt_dn_all; ++t) {
                    const int4 tl = S.tiles_dn[t];
                    const int lo = tl.y, hi = tl.y + tl.z;
                    for (int b = lo >> 6; b <= (hi - 1) >> 6 && ns < kDecMaxLastBlocks; ++b) {
                        const int bs = b * 64, be = min(a.H, bs + 64);
                        S.seg[ns++] = make_int2(b, min(be, hi) - max(bs, lo));
                    }
                }
                S.nseg = ns;
                S.nlast = 0;
            }
            bar_sync(kBarDec, kDecThreads);
            if (tid < S.nseg) {
                const int2 sg = S.seg[tid];
                const int bs = sg.x * 64, be = min(a.H, bs + 64);
                const unsigned target = (unsigned)U * (unsigned)(be - bs);
                const unsigned old = atomicAdd(a.block_ctr + sg.x, (unsigned)sg.y);
                if (old + (unsigned)sg.y == target) S.last[atomicAdd(&S.nlast, 1)] = sg.x;
            }
            bar_sync(kBarDec, kDecThreads);
            const int nlast = S.nlast;
            if (nlast) {
                __threadfence();
                for (int it = tid; it < nlast * a.M * 64; it += kDecThreads) {
                    const int qb = it / (a.M * 64), rem = it % (a.M * 64);
                    const int m = rem / 64, r = rem % 64;
                    const int n = S.last[qb] * 64 + r;
                    if (n >= a.H) continue;
                    float accv = 0.f;
#pragma unroll 1
                    for (int k0 = 0; k0 < a.K; k0 += 8) {
                        float dvv[8];
#pragma unroll
                        for (int k = 0; k < 8; ++k)
                            dvv[k] = (k0 + k < a.K) ? Half<DT>::to_f(__ldcg(a.down + (size_t)(m * a.K + k0 + k) * a.H + n))
                                                    : 0.f;
#pragma unroll
                        for (int k = 0; k < 8; ++k)
                            if (k0 + k < a.K) accv = fmaf(dvv[k], S.scores[m * a.K + k0 + k], accv);
                    }
                    const size_t off = (size_t)m * a.H + n;
                    if (a.h) {
                        const float delta = Half<DT>::to_f(Half<DT>::from_f(accv));
                        if (all_ok && !stopped) a.h[off] = Half<DT>::from_f(Half<DT>::to_f(a.h[off]) + delta);
                    } else {
                        if (all_ok && !stopped) a.y[off] = Half<DT>::from_f(accv);
                    }
                }
                if (tid < nlast) a.block_ctr[S.last[tid]] = 0u;  // ready for the next call
            }
        }
        dstamp(a, 10);
    }
    tc_before_sync();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, kDecTmemCols);
}

#define MOMIJ_DECODE_INST(DT, GS, T) \
    template __global__ void moe_decode_kernel<DT, GS, T>(const __grid_constant__ DecodeArgs);
#define MOMIJ_DECODE_INST_T(DT, GS) \
    MOMIJ_DECODE_INST(DT, GS, 1) MOMIJ_DECODE_INST(DT, GS, 2) MOMIJ_DECODE_INST(DT, GS, 4) MOMIJ_DECODE_INST(DT, GS, 8)
MOMIJ_DECODE_INST_T(MOMIJ_DTYPE_BF16, 64)
MOMIJ_DECODE_INST_T(MOMIJ_DTYPE_BF16, 128)
MOMIJ_DECODE_INST_T(MOMIJ_DTYPE_F16, 64)
MOMIJ_DECODE_INST_T(MOMIJ_DTYPE_F16, 128)

}  // namespace momij
