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

__device__ __forceinline__ void dstamp_thread(const DecodeArgs& a, int i) {
    if (a.trace) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        a.trace[(size_t)blockIdx.x * kTracePointsDec + i] = (long long)t;
    }
}
__device__ __forceinline__ void dstamp(const DecodeArgs& a, int i) {
    if (threadIdx.x == 0) dstamp_thread(a, i);
}

__device__ __forceinline__ long long gtime() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return (long long)t;
}
// Accumulated wait time of one role, written to trace slot `i` (tracing only).
__device__ __forceinline__ void dwait_put(const DecodeArgs& a, int i, long long ns) {
    if (a.trace) a.trace[(size_t)blockIdx.x * kTracePointsDec + i] = ns;
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
#pragma unroll 8
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
// Slot of group g in its accumulator pack of GP (<= 4) groups: a warpgroup
// takes four consecutive groups of every 8-group chunk, so its packs hold
// consecutive groups.
__device__ __forceinline__ int pack_slot(int g, int GP) { return g & (GP - 1); }

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
// fs[v * nG + g] = (2^(E-27), sum of the group).  Sixteen lanes per (vector,
// group): lane (w, p) takes the elements 16w + 4b + p, b = 0..3 -- the four
// K-bytes of one column word of every digit row -- so each digit is one
// 32-bit store.  `nthreads` threads from thread t0 take part.  Loads bypass
// L1 (the vectors may have been written by other CTAs).
template <int DT>
__device__ void digitize_b(const uint16_t* const* src, int nvec, int Kd, int N, int T, int GP, unsigned char* B,
                           float2* fs, int nthreads, int t0 = 0) {
    const int nG = Kd >> 6;
    const int total = nvec * nG * 16;
    const int lane = threadIdx.x & 31;
    const int gbytes = dec_b_group_bytes(N);
    // the next pass's four elements are loaded while this pass computes
    auto load = [&](int bs, uint16_t (&raw)[4]) {
        const int idx = bs + lane;
        if (idx < total) {
            const int vg = idx >> 4, sub = idx & 15;
            const int vv = vg / nG, gg = vg - vv * nG;
            const uint16_t* xg = src[vv] + (size_t)gg * 64 + 16 * (sub >> 2) + (sub & 3);
#pragma unroll
            for (int b = 0; b < 4; ++b) raw[b] = __ldcg(xg + 4 * b);
        }
    };
    uint16_t nraw[4] = {0, 0, 0, 0};
    load((threadIdx.x - t0) & ~31, nraw);
    for (int base = ((threadIdx.x - t0) & ~31); base < total; base += nthreads) {
        const int idx = base + lane;
        const bool valid = idx < total;
        const int vg = idx >> 4, sub = idx & 15;
        const int w = sub >> 2, p = sub & 3;
        const int v = valid ? vg / nG : 0, g = valid ? vg - v * nG : 0;
        uint16_t raw[4] = {nraw[0], nraw[1], nraw[2], nraw[3]};
        if (base + nthreads < total) load(base + nthreads, nraw);
        float xv[4];
        float mx = 0.f, sum = 0.f;
        if (valid) {
#pragma unroll
            for (int b = 0; b < 4; ++b) xv[b] = Half<DT>::to_f(raw[b]);
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                mx = fmaxf(mx, fabsf(xv[b]));
                sum += xv[b];
            }
        }
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) {
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            sum += __shfl_xor_sync(0xffffffffu, sum, o);
        }
        if (!valid) continue;
        int E = (mx > 0.f) ? ilogbf(mx) : 0;
        E = max(E, -100);
        const float scale = ldexpf(1.f, 21 - E);
        uint32_t word[4] = {0u, 0u, 0u, 0u};
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int X = __float2int_rn(xv[b] * scale);
            int dg[4];
            split4(X << (2 * (3 - p)), dg);
#pragma unroll
            for (int dd = 0; dd < 4; ++dd) word[dd] |= (uint32_t)(dg[dd] & 0xff) << (8 * b);
        }
        // element 16w + 4b + p: MMA half h = p >> 1, column word c = 4 (p & 1) + w, byte b
        const int h = p >> 1, c = 4 * (p & 1) + w;
        const int nb = pack_slot(g, GP) * 4 * T + v * 4;
        unsigned char* Bh = B + (size_t)g * gbytes + h * 32 * N + (c >> 2) * 128 + (c & 3) * 4;
#pragma unroll
        for (int dd = 0; dd < 4; ++dd) {
            const int n = nb + dd;
            *reinterpret_cast<uint32_t*>(Bh + (n >> 3) * 256 + (n & 7) * 16) = word[dd];
        }
        if (sub == 0) fs[v * nG + g] = make_float2(ldexpf(1.f, E - 27), sum);
    }
}


// Warp-uniform bounded wait: every lane polls, and the warp leaves together
// (all lanes saw the phase) or gives up together.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, int limit, const volatile int* abort) {
    if (__all_sync(0xffffffffu, mbar_test_wait(bar, parity))) return true;  // usually complete already
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
    int wpre[kDecMaxPairs + 1];  // prefix of the units' slice weights
    int bnd[4];                  // this CTA's up and down slice bounds
    unsigned gen0;  // the grid barrier's generation before this call's round
    uint32_t tmem;
    alignas(8) uint64_t full[kDecMaxStages];
    alignas(8) uint64_t empty[kDecMaxStages];
    alignas(8) uint64_t a_full[2][kDecAslots];   // [warpgroup][slot]: its four warps wrote the slot
    alignas(8) uint64_t a_empty[2][kDecAslots];  // [warpgroup][slot]: both issuing warps commit
    alignas(8) uint64_t d_full[4][4];             // [issuing warp][pack buffer]
    alignas(8) uint64_t d_empty[4][4];
    alignas(8) uint64_t b_ready[2];
    alignas(8) uint64_t drain[4];
};

}  // namespace

template <int DT, int GS, int T>
__global__ void __launch_bounds__(kDecThreadsAll, 1) moe_decode_kernel(const __grid_constant__ DecodeArgs a) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ DecShared S;
    // GP groups per accumulator pack; ND pack buffers per issuing warp (64 TMEM columns)
    constexpr int N = dec_mma_n(T), GP = dec_gp(T), ND = 64 / N;
    constexpr int kBarEpi = 1, kBarRoute = 2, kBarEnc = 3;
    constexpr int kWarpEpi0 = kDecDeqWarps, kWarpMma0 = kDecDeqWarps + kDecEpiWarps,
                  kWarpProd0 = kWarpMma0 + kDecMmaWarps;
    constexpr int kTidEpi0 = 32 * kWarpEpi0;
    dstamp(a, 0);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int P = a.M * a.K;
    volatile int* abort_flag = &S.abort;

    // ---- set-up (independent of the previous kernel) ---------------------------
    if (warp == 0) tmem_alloc(&S.tmem, kDecTmemCols);
    if (tid == 0) {
        for (int s = 0; s < a.stages; ++s) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.empty[s], kDecDeqWarps + kDecEpiWarps);  // codes read; scales and biases read
        }
        for (int d = 0; d < 2; ++d) {
            for (int s = 0; s < kDecAslots; ++s) mbar_init(&S.a_full[d][s], 4);
            for (int s = 0; s < kDecAslots; ++s) mbar_init(&S.a_empty[d][s], 2);
        }
        for (int i = 0; i < 4; ++i) {
            for (int s = 0; s < 4; ++s) {
                mbar_init(&S.d_full[i][s], 1);
                mbar_init(&S.d_empty[i][s], 4);
            }
            mbar_init(&S.drain[i], 1);
        }
        mbar_init(&S.b_ready[0], 1);
        mbar_init(&S.b_ready[1], 1);
        mbar_fence_init();
        S.abort = 0;
        S.stopped = 0;
    }
    float* s_logits = reinterpret_cast<float*>(smem + a.off_logits);
    unsigned char* s_B = smem + a.off_b;
    float2* s_fs = reinterpret_cast<float2*>(smem + a.off_fs);
    float* s_red = reinterpret_cast<float*>(smem + a.off_red);      // [2][T][128] tile-end partials
    unsigned char* s_ring = smem + a.off_ring;
    tc_before_sync();
    __syncthreads();
    tc_after_sync();
    const uint32_t tmem = S.tmem;

    // ---- after the previous kernel: x and the logits may be its output ---------
    pdl_wait();
    pdl_launch_dependents();
    dstamp(a, 1);
    if (tid == 0 && a.stop && __ldcg(a.stop) != 0) S.stopped = 1;
    if (tid == 0) S.gen0 = ld_acquire_u32(reinterpret_cast<const unsigned*>(a.ctrl + kCtrlGen));
    if (tid < 8) S.nan_tok[tid] = 0;
    __syncthreads();
    // A set stop flag (the reference's stopFlag, read once per CTA) skips the
    // streaming work; the CTA still arrives at the grid barrier and adds its
    // completion counts, so a flag raised while CTAs start leaves the
    // workspace consistent for the next call.
    const bool stopped = S.stopped != 0;
    const int nG_up = a.H >> 6, nG_dn = a.I >> 6;
    const int gbytes = dec_b_group_bytes(N);
    // ---- the epilogue warps encode the tokens (the up phase's digit operand,
    // ---- independent of the routing) while warps 0-7 route and plan
    if (warp >= kWarpEpi0 && warp < kWarpMma0) {
        const int te = tid - kTidEpi0;
        for (int i = te; i < a.b_bytes / 16; i += kDecEpiThreads)
            reinterpret_cast<uint4*>(s_B)[i] = make_uint4(0u, 0u, 0u, 0u);
        if (te < a.M) S.vec_ptr[te] = a.x + (size_t)te * a.H;
        bar_sync(kBarEpi, kDecEpiThreads);
        if (!stopped) digitize_b<DT>(S.vec_ptr, a.M, a.H, N, T, GP, s_B, s_fs, kDecEpiThreads, kTidEpi0);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        bar_sync(kBarEpi, kDecEpiThreads);
        if (te == 0) {
            dstamp_thread(a, 3);
            mbar_arrive(&S.b_ready[0]);
        }
    } else if (warp < kDecDeqWarps) {
        // routing and plan by the first warpgroups (a named barrier over them)
        constexpr int nthr = 32 * kDecDeqWarps;
        const int nlog = a.logits ? a.M * a.E : 0;
        for (int i = tid; i < nlog; i += nthr) {
            const float v = __ldcg(a.logits + i);
            s_logits[i] = v;
            if (isnan(v)) S.nan_tok[i / a.E] = 1;
        }
        if (!a.logits) {
            for (int i = tid; i < P; i += nthr) {
                S.inds[i] = __ldcg(a.inds_in + i);
                S.scores[i] = __ldcg(a.scores_in + i);
            }
        }
        bar_sync(kBarRoute, nthr);
        if (tid == 0) dstamp_thread(a, 22);
        if (a.logits) {
            if (a.M == 1) {  // one token: ranks over the warps
                route_tokens(s_logits, S.nan_tok, a.M, a.E, a.K, 0, nthr, kBarRoute, S.inds, S.scores,
                             a.trace ? a.trace + (size_t)blockIdx.x * kTracePointsDec + 25 : nullptr);
            } else if (warp < a.M) {  // several: one warp per token replays the reduction tree
                route_token_warp(s_logits + warp * a.E, a.E, a.K, S.inds + warp * a.K, S.scores + warp * a.K);
            }
        }
        bar_sync(kBarRoute, nthr);
        if (tid == 0) dstamp_thread(a, 23);
        if (warp == 0) {
            plan_units_warp(S.inds, P, a.E, a.K, T, S.units, S.sorted, S.qinfo, &S.nunits, &S.bad);
            __syncwarp();
            // unit weights (c0 + tokens: the epilogue's work grows with them) and their prefix
            const int U = S.nunits;
            const int w0 = lane < U ? a.slice_c0 + __popc(S.units[lane].w) : 0;
            const int w1 = lane + 32 < U ? a.slice_c0 + __popc(S.units[lane + 32].w) : 0;
            int s0 = w0, s1 = w1;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int t0 = __shfl_up_sync(0xffffffffu, s0, o), t1 = __shfl_up_sync(0xffffffffu, s1, o);
                if (lane >= o) {
                    s0 += t0;
                    s1 += t1;
                }
            }
            const int tot0 = __shfl_sync(0xffffffffu, s0, 31);
            S.wpre[lane] = s0 - w0;
            S.wpre[lane + 32] = tot0 + s1 - w1;
            if (lane == 31) S.wpre[64] = tot0 + s1;
        }
        bar_sync(kBarRoute, nthr);
        if (tid == 0) dstamp_thread(a, 24);
        if (tid < 4) {
            // CTA bx takes the 8-row granules of the (unit, row) space whose
            // weight prefix falls in [W bx / G, W (bx + 1) / G)
            const int U = S.nunits, G = gridDim.x;
            const int rows = tid < 2 ? a.I : a.H, n = rows / 8;
            const long long pos = (long long)n * S.wpre[U] * (blockIdx.x + (tid & 1)) / G;
            int u = 0;
            while (u < U && (long long)n * S.wpre[u + 1] < pos) ++u;
            int b = U * rows;
            if (u < U) {
                const long long w = S.wpre[u + 1] - S.wpre[u], rem = pos - (long long)n * S.wpre[u];
                b = (u * n + (int)((rem + w - 1) / w)) * 8;
            }
            S.bnd[tid] = b;
        }
        bar_sync(kBarRoute, nthr);
        if (tid == 0) {
            const int r0 = S.bnd[0], r1 = S.bnd[1], d0 = S.bnd[2], d1 = S.bnd[3];
            S.nt_up = make_tiles(r0, r1, a.I, 64, S.tiles_up, kDecMaxTiles);
            S.nt_dn = make_tiles(d0, d1, a.H, 128, S.tiles_dn, kDecMaxTiles);
            S.udn0 = d0 < d1 ? d0 / a.H : 0;
            S.nudn = d0 < d1 ? (d1 - 1) / a.H - d0 / a.H + 1 : 0;
            if (S.bad == 0 && (S.nt_up > kDecMaxTiles || S.nt_dn > kDecMaxTiles || S.nudn > 2)) {
                atomicExch(a.ctrl + kCtrlError, MOMIJ_ERR_WORKSPACE);  // host-sized; unreachable
                S.nt_up = S.nt_dn = 0;
                S.nudn = 0;
            }
            if (a.trace) a.trace[(size_t)blockIdx.x * kTracePointsDec + 16] = gtime();
        }
        if (blockIdx.x == 0 && S.bad == 0) {
            for (int i = tid; i < P; i += nthr) {
                if (a.inds_out) a.inds_out[i] = S.inds[i];
                if (a.scores_out) a.scores_out[i] = S.scores[i];
            }
        }
    }
    __syncthreads();
    const bool ok = S.bad == 0;
    if (blockIdx.x == 0 && tid == 0)
        a.ctrl[kCtrlStatus] = ok ? (stopped ? MOMIJ_ERR_STOPPED : MOMIJ_OK) : MOMIJ_ERR_EXPERT_INDEX;
    if (!ok) {  // uniform: every CTA sees the same indices
        if (warp == 0) tmem_dealloc(tmem, kDecTmemCols);
        return;
    }
    dstamp(a, 2);
    const int U = S.nunits;
    const int nC_up = (nG_up + 7) >> 3, nC_dn = (nG_dn + 7) >> 3;
    // tiles streamed and computed (none when stopped); nt_dn_all also feeds the combine counts
    const int nt_up = stopped ? 0 : S.nt_up, nt_dn = stopped ? 0 : S.nt_dn, nt_dn_all = S.nt_dn;
    const int S_ = a.stages;
    // groups of warpgroup d in chunk c of a phase with nG groups (0 or 4: nG % 4 == 0)
    auto wg_groups = [](int nG, int c, int d) { return min(4, max(0, min(8, nG - 8 * c) - 4 * d)); };

    if (warp >= kWarpMma0) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kDecRegsCtl));
    else if (warp < kWarpEpi0) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kDecRegsDeq));
    else asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kDecRegsEpi));
    if (warp >= kWarpProd0 + kDecProducers) {
        // idle
    } else if (warp >= kWarpProd0) {
        // ---- TMA producers: item i (phase, tile, chunk) fills stage i % S_ -------------
        // ---- (codes, then scales, then biases); producer i % 2 (S_ is even) -----------
        if (lane == 0) {
            const int p = warp - kWarpProd0;
            int item = 0;
            int issued_last[kDecMaxStages];
            long long wait_ns = 0;
            for (int s = 0; s < kDecMaxStages; ++s) issued_last[s] = -1;
            bool okp = true;
            for (int ph = 0; ph < 2 && okp; ++ph) {
                const int nt = ph ? nt_dn : nt_up, nC = ph ? nC_dn : nC_up;
                const int4* tiles = ph ? S.tiles_dn : S.tiles_up;
                const CUtensorMap* mc = ph ? a.map_dn : a.map_ug;
                const CUtensorMap* ms = ph ? a.map_sdn : a.map_sug;
                const CUtensorMap* mb = ph ? a.map_bdn : a.map_bug;
                for (int t = 0; t < nt && okp; ++t) {
                    const int4 tl = tiles[t];
                    const int e = S.units[tl.x].x;
                    for (int c = 0; c < nC; ++c, ++item) {
                        if ((item & 1) != p) continue;
                        const int s = item % S_, use = item / S_;
                        const long long tw0 = a.trace ? gtime() : 0;
                        if (use > 0 && !mbar_wait_bounded(&S.empty[s], (use - 1) & 1, a.spin_limit, abort_flag)) {
                            okp = false;
                            break;
                        }
                        if (a.trace) wait_ns += gtime() - tw0;
                        const int rows = ph ? tl.z : 2 * tl.z;
                        mbar_expect_tx(&S.full[s], (uint32_t)(rows * (128 + 32)));
                        const uint32_t st = smem_u32(s_ring + (size_t)s * kDecStageBytes);
                        const uint32_t ss = st + kDecCodeBytes, sb = ss + kDecSbBytes;
                        const int xc = c * 128, xs = (GS == 64) ? 16 * c : 16 * (c >> 1);
                        if (ph == 0 && tl.z == 64) {  // a full up||gate tile: both halves in one box each
                            tma_load_3d(st, &mc[4], xc, tl.y, 2 * e, &S.full[s]);
                            tma_load_3d(ss, &ms[4], xs, tl.y, 2 * e, &S.full[s]);
                            tma_load_3d(sb, &mb[4], xs, tl.y, 2 * e, &S.full[s]);
                        } else if (ph == 1 && tl.z == 128) {
                            const int grow = e * a.H + tl.y;
                            tma_load_2d(st, &mc[3], xc, grow, &S.full[s]);
                            tma_load_2d(ss, &ms[3], xs, grow, &S.full[s]);
                            tma_load_2d(sb, &mb[3], xs, grow, &S.full[s]);
                        } else {
                            for (int part = 0; part < (ph ? 1 : 2); ++part) {
                                // up||gate: up rows at stage rows [0, n), gate rows at [64, 64 + n)
                                int grow = ph ? e * a.H + tl.y : e * 2 * a.I + part * a.I + tl.y;
                                int srow = part * 64;
                                int left = tl.z;
                                while (left > 0) {
                                    const int bi = left >= 64 ? 0 : left >= 16 ? 1 : 2;
                                    const int br = bi == 0 ? 64 : bi == 1 ? 16 : 8;
                                    tma_load_2d(st + srow * 128, &mc[bi], xc, grow, &S.full[s]);
                                    tma_load_2d(ss + srow * 16, &ms[bi], xs, grow, &S.full[s]);
                                    tma_load_2d(sb + srow * 16, &mb[bi], xs, grow, &S.full[s]);
                                    grow += br;
                                    srow += br;
                                    left -= br;
                                }
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
            if (p == 0) dwait_put(a, 11, wait_ns);
            // every issued stage has landed before the CTA can exit
            for (int s = 0; s < S_; ++s)
                if (issued_last[s] >= 0) mbar_drain(&S.full[s], issued_last[s] & 1);
        }
    } else if (warp >= kWarpMma0) {
        // ---- MMA issue: warp kWarpMma0 + 2d + hh issues groups 2hh, 2hh + 1 ---------
        // ---- of warpgroup d's four in every chunk ---------------------------------
        if (lane == 0) {
            const int iw = warp - kWarpMma0, d = iw >> 1, hh = iw & 1;
            int ua = 0, ud = 0;
            long long wait_a = 0, wait_d = 0, cy_issue = 0;
            const uint32_t idesc = idesc_u8s8(N);
            bool okm = true;
            const uint32_t tA0 = tmem + d * 256, tD0 = tmem + d * 256 + 128 + hh * 64;

            for (int ph = 0; ph < 2 && okm; ++ph) {
                const int nt = ph ? nt_dn : nt_up, nC = ph ? nC_dn : nC_up, nG = ph ? nG_dn : nG_up;
                const int4* tiles = ph ? S.tiles_dn : S.tiles_up;
                if (nt > 0) {  // the phase's digit operand
                    if (!mbar_wait_bounded(&S.b_ready[ph], 0, a.spin_limit, abort_flag)) {
                        okm = false;
                        break;
                    }
                }
                for (int t = 0; t < nt && okm; ++t) {
                    const int4 tl = tiles[t];
                    const uint32_t bbase = smem_u32(s_B) + (ph ? (uint32_t)((tl.x - S.udn0) * nG_dn * gbytes) : 0u);
                    for (int c = 0; c < nC && okm; ++c) {
                        if (wg_groups(nG, c, d) == 0) continue;
                        const int slot = ua % kDecAslots;
                        const long long tw0 = a.trace ? gtime() : 0;
                        // the four warps of the warpgroup have written the slot
                        if (!mbar_wait_bounded(&S.a_full[d][slot], (ua / kDecAslots) & 1, a.spin_limit, abort_flag)) {
                            okm = false;
                            break;
                        }
                        if (a.trace) wait_a += gtime() - tw0;
                        tc_after_sync();
                        const long long cyi = a.trace ? clock64() : 0;
                        const uint32_t tA = tA0 + slot * 64;
#pragma unroll
                        for (int jj = 0; jj < 2; ++jj) {
                            const int j = 2 * hh + jj;
                            const int g = 8 * c + 4 * d + j;
                            const int gl = jj & (GP - 1);
                            const int buf = ud % ND;
                            if (gl == 0 && ud >= ND) {
                                const long long tw1 = a.trace ? gtime() : 0;
                                if (!mbar_wait_bounded(&S.d_empty[iw][buf], ((ud - ND) / ND) & 1, a.spin_limit,
                                                       abort_flag)) {
                                    okm = false;
                                    break;
                                }
                                if (a.trace) wait_d += gtime() - tw1;
                                tc_after_sync();
                            }
                            const uint32_t tD = tD0 + buf * N;
#pragma unroll
                            for (int h = 0; h < 2; ++h) {
                                const uint64_t bd = sdesc_noswz(bbase + (uint32_t)(g * gbytes + h * 32 * N), 128, 256);
                                mma_i8_ta(tD, tA + j * 16 + h * 8, bd, idesc, (gl | h) ? 1u : 0u);
                            }
                            if (gl == GP - 1) {
                                mma_commit(&S.d_full[iw][buf]);
                                ++ud;
                            }
                        }
                        if (!okm) break;
                        mma_commit(&S.a_empty[d][slot]);
                        if (a.trace) cy_issue += clock64() - cyi;
                        ++ua;
                    }
                }
            }
            if (!okm) {
                *abort_flag = 1;
                atomicExch(a.ctrl + kCtrlError, MOMIJ_ERR_TIMEOUT);
            }
            if (iw == 0) {
                dwait_put(a, 12, wait_a);
                dwait_put(a, 13, wait_d);
                dwait_put(a, 19, cy_issue);
            }
            // every MMA issued has completed before the tensor memory is released
            mma_commit(&S.drain[iw]);
            mbar_drain(&S.drain[iw], 0);
        }
    } else if (warp < kWarpEpi0) {
        // ---- dequantising warpgroup d: groups [4d, 4d + 4) of every stage ---------------
        // ---- (16-byte chunks 4d .. 4d + 3 of a 128-byte stage row); lane L = tile row --
        // Software-pipelined: the next item's codes are read while this item's
        // tensor-memory stores complete.
        const int d = warp >> 2, L = (warp & 3) * 32 + lane;
        const uint32_t lane_off = tmem_lane_base(warp);
        const uint32_t tA0 = tmem + d * 256;
        bool okd = true;
        long long w_full = 0, w_a = 0;
        // stream position: item number and its (phase, tile, chunk)
        int item = 0, ph = 0, t = 0, c = 0;
        auto settle = [&]() {
            while (ph < 2 && t >= (ph ? nt_dn : nt_up)) {
                ++ph;
                t = 0;
            }
        };
        settle();
        // Reads the codes of the next item with groups for this warpgroup into
        // `raw` (and releases the stages of the items before it, which hold
        // nothing for it); false at the end of the stream.
        auto fetch = [&](uint4 (&raw)[4]) -> bool {
            while (ph < 2) {
                const int s = item % S_;
                const bool mine = wg_groups(ph ? nG_dn : nG_up, c, d) > 0;
                if (mine) {
                    const long long tw0 = a.trace ? gtime() : 0;
                    if (okd) okd = mbar_wait_warp(&S.full[s], (item / S_) & 1, a.spin_limit, abort_flag);
                    if (a.trace) w_full += gtime() - tw0;
                    if (okd) {
                        const unsigned char* row = s_ring + (size_t)s * kDecStageBytes + L * 128;
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            raw[j] = *reinterpret_cast<const uint4*>(row + (((4 * d + j) ^ (L & 7)) << 4));
                    }
                }
                __syncwarp();
                if (lane == 0 && okd) mbar_arrive(&S.empty[s]);  // in registers now (or nothing to read)
                ++item;
                if (++c == (ph ? nC_dn : nC_up)) {
                    c = 0;
                    ++t;
                    settle();
                }
                if (mine) return true;
            }
            return false;
        };
        uint4 raw[4];
        bool have = fetch(raw);
        for (int ua = 0; have; ++ua) {
            // the A operand: four class words per code word, 16 columns per group
            const int slot = ua % kDecAslots;
            const long long tw1 = a.trace ? gtime() : 0;
            if (okd && ua >= kDecAslots)
                okd = mbar_wait_warp(&S.a_empty[d][slot], ((ua - kDecAslots) / kDecAslots) & 1, a.spin_limit,
                                     abort_flag);
            if (a.trace) w_a += gtime() - tw1;
            if (okd) {
                tc_after_sync();
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint32_t wv[4] = {raw[j].x, raw[j].y, raw[j].z, raw[j].w};
                    uint32_t m[16];
#pragma unroll
                    for (int p = 0; p < 4; ++p)
#pragma unroll
                        for (int i = 0; i < 4; ++i) m[4 * p + i] = wv[i] & (0x03030303u << (2 * p));
                    tmem_st16(tA0 + slot * 64 + j * 16 + lane_off, m);
                }
            }
            have = fetch(raw);
            if (okd) {
                tmem_st_wait();
                tc_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.a_full[d][slot]);
            }
        }
        if (!okd) *abort_flag = 1;
        if (tid == 0) {
            dwait_put(a, 14, w_full);
            dwait_put(a, 15, w_a);
        }
    } else {
        // ---- epilogue warpgroup d: warpgroup d's accumulators -> partial row sums ---
        // epilogue warp (d, hh, quarter): the accumulators of MMA issuer 2d + hh
        const int ew = warp - kWarpEpi0, d = ew >> 3, hh = (ew >> 2) & 1, L = (warp & 3) * 32 + lane;
        const int iw = 2 * d + hh;
        const int te = tid - kTidEpi0;  // 0 .. kDecEpiThreads - 1
        const uint32_t lane_off = tmem_lane_base(warp);
        const uint32_t tD0 = tmem + d * 256 + 128;
        int ude = 0, item = 0;
        bool oke = true;
        long long w_d = 0, cy_epi = 0;
        const bool prof = a.trace != nullptr && te == 0;
        for (int ph = 0; ph < 2; ++ph) {
            const int nt = ph ? nt_dn : nt_up, nC = ph ? nC_dn : nC_up, nG = ph ? nG_dn : nG_up;
            const int4* tiles = ph ? S.tiles_dn : S.tiles_up;
            if (ph == 1) {
                // the combine's completion counters start at zero whatever the
                // workspace held (a call of another batch size carves it
                // differently): CTA 0 clears them before the grid barrier that
                // precedes every count
                if (blockIdx.x == 0)
                    for (int i = te; i < (a.H + 63) / 64; i += kDecEpiThreads) a.block_ctr[i] = 0u;
                // act complete on every CTA: grid barrier, then the down phase's digits
                bar_sync(kBarEpi, kDecEpiThreads);
                if (te == 0) dstamp_thread(a, 6);
                if (te == 0) {
                    // every CTA arrives (also after an error), so the counter returns to zero
                    const bool wait = !*abort_flag;
                    S.flag = grid_barrier_thread(reinterpret_cast<unsigned*>(a.ctrl + kCtrlArrive),
                                                 reinterpret_cast<unsigned*>(a.ctrl + kCtrlGen), S.gen0, a.spin_limit,
                                                 wait) && wait;
                }
                bar_sync(kBarEpi, kDecEpiThreads);
                if (!S.flag) oke = false;
                if (te == 0) dstamp_thread(a, 7);
                if (oke && !stopped) {
                    for (int i = te; i < a.b_bytes / 16; i += kDecEpiThreads)
                        reinterpret_cast<uint4*>(s_B)[i] = make_uint4(0u, 0u, 0u, 0u);
                    bar_sync(kBarEpi, kDecEpiThreads);
                    for (int us = 0; us < S.nudn; ++us) {
                        const int4 un = S.units[S.udn0 + us];
                        if (te < un.z) S.vec_ptr[te] = a.act + (size_t)S.sorted[un.y + te] * a.I;
                        bar_sync(kBarEpi, kDecEpiThreads);
                        // threads numbered from 0 within the epilogue warps
                        digitize_b<DT>(S.vec_ptr, un.z, a.I, N, T, GP, s_B + (size_t)us * nG_dn * gbytes,
                                       s_fs + (size_t)us * T * nG_dn, kDecEpiThreads, kTidEpi0);
                        bar_sync(kBarEpi, kDecEpiThreads);
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                }
                bar_sync(kBarEpi, kDecEpiThreads);
                if (te == 0) {
                    dstamp_thread(a, 8);
                    mbar_arrive(&S.b_ready[1]);
                }
            }
            for (int t = 0; t < nt; ++t) {
                const int4 tl = tiles[t];
                const int4 un = S.units[tl.x];
                // vectors of this tile: up -- the unit's tokens; down -- its pairs
                const int vmask = ph ? ((1 << un.z) - 1) : un.w;
                const float2* fsb = ph ? s_fs + (size_t)(tl.x - S.udn0) * T * nG_dn : s_fs;
                float acc[T];
#pragma unroll
                for (int v = 0; v < T; ++v) acc[v] = 0.f;
                for (int c = 0; c < nC; ++c, ++item) {
                    // this warpgroup's scales and biases of the item, from its stage
                    const int s = item % S_;
                    if (wg_groups(nG, c, d) == 0) {
                        __syncwarp();
                        if (lane == 0 && oke) mbar_arrive(&S.empty[s]);
                        continue;
                    }
                    uint4 sbw = make_uint4(0u, 0u, 0u, 0u);
                    if (oke) oke = mbar_wait_warp(&S.full[s], (item / S_) & 1, a.spin_limit, abort_flag);
                    if (oke) {
                        const unsigned char* sbrow = s_ring + (size_t)s * kDecStageBytes + kDecCodeBytes + L * 16;
                        if (GS == 64) {  // this warp's two groups 2hh, 2hh + 1 of warpgroup d's four
                            const uint32_t sw = *reinterpret_cast<const uint32_t*>(sbrow + 8 * d + 4 * hh);
                            const uint32_t bw = *reinterpret_cast<const uint32_t*>(sbrow + kDecSbBytes + 8 * d + 4 * hh);
                            sbw = hh ? make_uint4(0u, sw, 0u, bw) : make_uint4(sw, 0u, bw, 0u);
                        } else {  // gs 128: two scales (one word) of the chunk's half of the box
                            const int so = 8 * (c & 1) + 4 * d;
                            sbw.x = *reinterpret_cast<const uint32_t*>(sbrow + so);
                            sbw.z = *reinterpret_cast<const uint32_t*>(sbrow + kDecSbBytes + so);
                        }
                    }
                    __syncwarp();
                    if (lane == 0 && oke) mbar_arrive(&S.empty[s]);
                    {
#pragma unroll
                        for (int pk = 0; pk < 2 / GP; ++pk) {
                            const int buf = ude % ND;
                            const long long tw0 = a.trace ? gtime() : 0;
                            if (oke) oke = mbar_wait_warp(&S.d_full[iw][buf], (ude / ND) & 1, a.spin_limit, abort_flag);
                            if (a.trace) w_d += gtime() - tw0;
                            ++ude;
                            const long long cy0 = prof ? clock64() : 0;
                            if (oke) {
                                tc_after_sync();
                                uint32_t dv[N];
                                const uint32_t taddr = tD0 + hh * 64 + buf * N + lane_off;
                                if (N == 16) tmem_ld16_nowait(taddr, *reinterpret_cast<uint32_t(*)[16]>(dv));
                                else tmem_ld32_nowait(taddr, *reinterpret_cast<uint32_t(*)[32]>(dv));
                                tmem_ld_wait();
                                tc_before_sync();
                                __syncwarp();
                                if (lane == 0) mbar_arrive(&S.d_empty[iw][buf]);
#pragma unroll
                                for (int gl = 0; gl < GP; ++gl) {
                                    const int j = 2 * hh + pk * GP + gl;  // group of the warpgroup's four
                                    const int g = 8 * c + 4 * d + j;
                                    float sf, bf;
                                    if (GS == 64) {
                                        const uint32_t sw = (j < 2) ? sbw.x : sbw.y, bw = (j < 2) ? sbw.z : sbw.w;
                                        sf = Half<DT>::to_f((uint16_t)(sw >> (16 * (j & 1))));
                                        bf = Half<DT>::to_f((uint16_t)(bw >> (16 * (j & 1))));
                                    } else {
                                        sf = Half<DT>::to_f((uint16_t)(sbw.x >> (16 * (j >> 1))));
                                        bf = Half<DT>::to_f((uint16_t)(sbw.z >> (16 * (j >> 1))));
                                    }
#pragma unroll
                                    for (int v = 0; v < T; ++v) {
                                        if ((vmask >> v) & 1) {
                                            const int nb = gl * 4 * T + v * 4;
                                            const float f = fmaf((float)(int)dv[nb], 16777216.f,
                                                                 fmaf((float)(int)dv[nb + 1], 65536.f,
                                                                      (float)((int)dv[nb + 2] * 256 + (int)dv[nb + 3])));
                                            const float2 fsv = fsb[v * nG + g];
                                            acc[v] += fmaf(sf, f * fsv.x, bf * fsv.y);
                                        }
                                    }
                                }
                            }
                            if (prof) cy_epi += clock64() - cy0;
                        }
                    }
                }
                // ---- tile end: the four issuers' partials -> (p00 + p01) + (p10 + p11) ----
#pragma unroll
                for (int v = 0; v < T; ++v)
                    if ((vmask >> v) & 1) s_red[((size_t)iw * T + v) * 128 + L] = acc[v];
                bar_sync(kBarEpi, kDecEpiThreads);
                if (oke) {
                    const size_t st = (size_t)T * 128;
                    auto red_sum = [&](int v, int l) {
                        const float* r = s_red + (size_t)v * 128 + l;
                        return (r[0] + r[st]) + (r[2 * st] + r[3 * st]);
                    };
                    if (ph == 0) {
                        for (int i = te; i < un.z * 64; i += kDecEpiThreads) {
                            const int j = i >> 6, l = i & 63;
                            if (l >= tl.z) continue;
                            const int pr = S.sorted[un.y + j];
                            const int m = pr / a.K;
                            a.act[(size_t)pr * a.I + tl.y + l] =
                                swiglu_staged<DT>(red_sum(m, l), red_sum(m, l + 64), a.clamp);
                        }
                    } else {
                        for (int i = te; i < un.z * 128; i += kDecEpiThreads) {
                            const int j = i >> 7, l = i & 127;
                            if (l >= tl.z) continue;
                            const int pr = S.sorted[un.y + j];
                            a.down[(size_t)pr * a.H + tl.y + l] = Half<DT>::from_f(red_sum(j, l));
                        }
                    }
                }
                bar_sync(kBarEpi, kDecEpiThreads);
            }
            if (ph == 0 && te == 0) dstamp_thread(a, 5);
        }
        // a warp that gave up makes the others give up at their next wait
        if (!oke) *abort_flag = 1;
        bar_sync(kBarEpi, kDecEpiThreads);
        const bool all_ok = !*abort_flag;
        if (!all_ok && te == 0) atomicExch(a.ctrl + kCtrlError, MOMIJ_ERR_TIMEOUT);
        if (te == 0) dstamp_thread(a, 9);

        // ---- last-arriver combine per 64-row block --------------------------------
        // (the counts are added also after an error or a stop, so that every
        // counter returns to zero; the status word then flags the output)
        {
            __threadfence();  // down rows written by this thread, before the block counters
            bar_sync(kBarEpi, kDecEpiThreads);
            if (te == 0) {
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
            bar_sync(kBarEpi, kDecEpiThreads);
            if (te < S.nseg) {
                const int2 sg = S.seg[te];
                const int bs = sg.x * 64, be = min(a.H, bs + 64);
                const unsigned target = (unsigned)U * (unsigned)(be - bs);
                const unsigned old = atomicAdd(a.block_ctr + sg.x, (unsigned)sg.y);
                if (old + (unsigned)sg.y == target) S.last[atomicAdd(&S.nlast, 1)] = sg.x;
            }
            bar_sync(kBarEpi, kDecEpiThreads);
            const int nlast = S.nlast;
            if (nlast) {
                __threadfence();
                for (int it = te; it < nlast * a.M * 64; it += kDecEpiThreads) {
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
                if (te < nlast) a.block_ctr[S.last[te]] = 0u;  // ready for the next call
            }
        }
        if (te == 0) {
            dstamp_thread(a, 10);
            dwait_put(a, 17, w_d);
            dwait_put(a, 18, cy_epi);
        }
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
