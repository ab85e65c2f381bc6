// token.cu -- one MoE FFN layer for a decode token (or a batch of up to 8,
// one token after another) in one persistent kernel (one CTA per SM,
// launched cooperatively): a producer warpgroup
// streams the layer's expert weights by TMA into a ring of CTA-wide stages
// while 16 compute warps multiply them on the tensor cores; every step that
// is not streaming weights is short and parallel.
//
//   1. every CTA loads the logits and the token, ranks the experts (momij's
//      maple_route_top8, SeedlessMetal.swift:2720-2791: value order, ties in
//      its reduction-tree order -- the smaller bit-reversed index; a token
//      with a NaN logit replays the tree, route_tokens) and starts the weight
//      stream; it then encodes the token into the digit operand and computes
//      the renormalised scores while the first stages land.  A CTA takes an
//      even share of the up||gate tiles (8 row pairs of one expert slot) and
//      rows_per_cta output rows;
//   2. up||gate phase: one stage = two tiles x all of H (codes, scales,
//      biases; one 4D box per tile brings its 8 up and 8 gate rows, every
//      128-byte column); warp w takes column w & 7 of tile w >> 3; the
//      partial sums go to shared memory and each row pair then gets its
//      staged clamped SwiGLU -> act[slot, I];
//   3. grid barrier (act complete; the down weights are already streaming);
//   4. down phase: the CTA encodes the K act vectors, then warps 2k and
//      2k + 1 take expert slot k's two 16-row halves; one stage = one
//      128-byte code column of the CTA's rows for every expert slot; in the
//      epilogue the two lanes holding a row's digit columns fold 256 D0 + D1
//      and 256 D2 + D3 (|D| < 2^20) and exchange one word;
//   5. the CTA combines its own rows: y[n] = cast(sum_k float(down_k[n]) *
//      score_k) in k order (MapleMoE.swift:76-78), or h[n] = cast(h[n] +
//      cast(acc)) (maple_score_resid) -- no staging of the down outputs and no
//      cross-CTA completion counters.
// A launch may carry up to kTokMaxM tokens (a decode or verify batch): they
// are routed together, then steps 2-5 run for one token after another (act
// kept per token, one grid barrier per token) while the producer streams the
// next token's weights during the current token's serial tail; every token
// gets the bits of a single-token call.
//
// Arithmetic (exact integer inner products on the tensor cores): a 16-code
// word w gives the u8 operand of code class p (the code at bit offset 2p of
// every byte) as w & (0x03030303 << 2p) = q * 4^p.  Each 64-element group of
// the vector with largest magnitude in [2^E, 2^(E+1)) is X = rint(x *
// 2^(21-E)); the class-p elements enter as Y = X * 4^(3-p), split into four
// balanced base-256 s8 digits, so the four classes accumulate into the same
// s32 columns: sum_k q_k Y_k = 64 * sum_k q_k X_k.  mma.sync m16n8k32
// u8 x s8 -> s32: an MMA's K slab holds groups j and j + 4 of a 128-byte code
// column (16 code bytes each, one class), its 8 columns (group, digit) -- the
// pairing that makes the lanes' reads of the TMA's 128-byte swizzled rows
// conflict-free.  Per group and row the fp32 epilogue applies
//   s * (2^24 D0 + 2^16 D1 + 2^8 D2 + D3) * 2^(E-27) + b * sum(x)
// (the reference's gqmm2_rows form y = sum_g s_g sum(q x) + b_g sum(x),
// SeedlessMetal.swift:2145-2221), the same expression as the tcgen05 decode
// kernel's epilogue.
#include "route_core.cuh"
#include "tc.cuh"
#include "token.cuh"

namespace momij {

namespace {

__device__ __forceinline__ void tstamp(const TokenArgs& a, int i) {
    if (a.trace && threadIdx.x == 0) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        a.trace[(size_t)blockIdx.x * kTracePointsDec + i] = (long long)t;
    }
}

// Encoder tasks: EPT (8 or 16) consecutive elements of one 64-element group
// (vector v at src + v * Kd, Kd a multiple of 512); task = (v * nG + G) *
// (64 / EPT) + u, u the task's part of its group.
template <int EPT>
struct EncTask {
    static constexpr int kWords = EPT / 2;  // 16-bit elements in 32-bit words
    uint32_t w[kWords];
};

// Loads one task's elements; bypasses L1 (the vectors may have been written
// by other CTAs).
template <int EPT>
__device__ __forceinline__ void tok_load_task(const uint16_t* __restrict__ src, int Kd, int task, EncTask<EPT>& r) {
    const uint4* sp = reinterpret_cast<const uint4*>(src + (size_t)task * EPT);  // tasks tile the vectors in order
#pragma unroll
    for (int i = 0; i < EPT / 8; ++i) {
        const uint4 v = __ldcg(sp + i);
        r.w[4 * i] = v.x;
        r.w[4 * i + 1] = v.y;
        r.w[4 * i + 2] = v.z;
        r.w[4 * i + 3] = v.w;
    }
}

// Encodes one task into the digit operand.  The 64 / EPT tasks of a group sit
// in consecutive lanes (all 32 lanes call it; `valid` false only takes part
// in the shuffles).  Layout, per vector and 512-element code column c (2 KB):
// [slab s (4)][class pair (2)][active B lane L (16)][16 B], lane L's 16 bytes
// the fragments (b0, b1) of the pair's even then odd class, stored at entry
// (L & 8) | ((L & 7) ^ s) with the two 8-byte halves swapped when L >= 8 --
// so that the encoder's stores of a warp (its groups differ in slab and row)
// fall into distinct banks, while a reader's 16 lanes still cover one
// contiguous 256-byte block.  Group j of the
// column (G = 8c + j) feeds slab j & 3 through A lanes with t >> 1 = j >> 2;
// its in-group byte bb goes to A lane t & 1 = bb >> 3, register (bb >> 2) &
// 1, byte bb & 3, and its digit d to B lane L = 8 (j >> 2) + 4 (bb >> 3) + d.
// fs[v * nG + G] = (2^(E-27), sum of the group).  Digits: y = 2^24 d0 +
// 2^16 d1 + 2^8 d2 + d3 with d1..d3 in [-128, 127]; the bytes of (y +
// 0x808080) ^ 0x808080 are d3, d2, d1, d0 (each digit's byte is its
// carry-free remainder), and byte permutes gather digit dd of the task's
// class-p elements into one store.  Rounding: x * 2^(21-E) + 1.5 * 2^23 is
// rint(x * 2^(21-E)) + 1.5 * 2^23 exactly (|x * 2^(21-E)| < 2^22), so the
// integer bits of that sum, times 4^(3-p), plus the digit offset are one
// integer multiply-add: y + 0x808080 = bits * 4^(3-p) + (0x808080 -
// 0x4B400000 * 4^(3-p)) modulo 2^32.
template <int DT, int EPT>
__device__ __forceinline__ void tok_encode(const EncTask<EPT>& r, bool valid, int task, int Kd,
                                           unsigned char* __restrict__ B, float2* __restrict__ fs) {
    constexpr int TPG = 64 / EPT, NB = EPT / 4;  // tasks per group, code bytes per task
    float xv[EPT];
#pragma unroll
    for (int i = 0; i < EPT / 2; ++i) {
        xv[2 * i] = Half<DT>::to_f(static_cast<uint16_t>(r.w[i] & 0xffffu));
        xv[2 * i + 1] = Half<DT>::to_f(static_cast<uint16_t>(r.w[i] >> 16));
    }
    float mx = 0.f, sp[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        sp[p] = xv[p];
#pragma unroll
        for (int b = 1; b < NB; ++b) sp[p] += xv[4 * b + p];
#pragma unroll
        for (int b = 0; b < NB; ++b) mx = fmaxf(mx, fabsf(xv[4 * b + p]));
    }
    float W = (sp[0] + sp[1]) + (sp[2] + sp[3]);
#pragma unroll
    for (int o = 1; o < TPG; o <<= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        W += __shfl_xor_sync(0xffffffffu, W, o);
    }
    if (!valid) return;
    const int fe = (__float_as_int(mx) >> 23) & 0xff;
    int E = fe ? fe - 127 : (mx > 0.f ? ilogbf(mx) : 0);
    E = max(E, -100);
    const float scale = __int_as_float((148 - E) << 23);  // 2^(21 - E)
    const int vg = task / TPG, u = task - vg * TPG;
    const int nG = Kd >> 6, v = vg / nG, G = vg - v * nG, j = G & 7;
    const int bb0 = u * NB;  // first in-group byte of the task
    const int sl = j & 3, hi = j >> 2;  // slab, row of the entries (L >> 3)
    unsigned char* gb = B + (size_t)v * tok_b_bytes(Kd) + (G >> 3) * 2048 + sl * 512 + hi * 128 +
                        ((bb0 >> 2) & 1) * 4 + (bb0 & 3);
    const int ent0 = (bb0 >> 3) * 4;  // entry of digit 0 within the row, before the swizzle
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        constexpr uint32_t kMagic = 0x4B400000u;  // bits of 1.5 * 2^23
        const uint32_t mul = 1u << (2 * (3 - p)), add = 0x808080u - kMagic * mul;
        uint32_t e[NB];
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            const uint32_t bits = __float_as_uint(fmaf(xv[4 * b + p], scale, 12582912.f));
            e[b] = (bits * mul + add) ^ 0x808080u;
        }
        unsigned char* gp = gb + (p >> 1) * 256 + (((p & 1) ^ hi) * 8);
        auto ent = [&](int d) { return ((ent0 + d) ^ sl) * 16; };
        if (NB == 4) {
            const uint32_t t0 = __byte_perm(e[0], e[1], 0x5140), t1 = __byte_perm(e[2 % NB], e[3 % NB], 0x5140);
            const uint32_t t2 = __byte_perm(e[0], e[1], 0x7362), t3 = __byte_perm(e[2 % NB], e[3 % NB], 0x7362);
            *reinterpret_cast<uint32_t*>(gp + ent(3)) = __byte_perm(t0, t1, 0x5410);  // d3 (256^0)
            *reinterpret_cast<uint32_t*>(gp + ent(2)) = __byte_perm(t0, t1, 0x7632);  // d2
            *reinterpret_cast<uint32_t*>(gp + ent(1)) = __byte_perm(t2, t3, 0x5410);  // d1
            *reinterpret_cast<uint32_t*>(gp + ent(0)) = __byte_perm(t2, t3, 0x7632);  // d0 (256^3)
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i)  // digit 3 - i: byte i of both elements
                *reinterpret_cast<uint16_t*>(gp + ent(3 - i)) =
                    static_cast<uint16_t>(__byte_perm(e[0], e[1 % NB], i | ((4 + i) << 4)));
        }
    }
    if (u == 0)
        fs[v * nG + G] = make_float2(E > -100 ? __int_as_float((E + 100) << 23) : ldexpf(1.f, E - 27), W);
}

// Encodes vectors [v0, v0 + nvec) of src (row length Kd) by `nthr` threads
// (whole warps, thread index `tt` from 0), EPT elements per task, each thread
// loading all its tasks of a pass before it computes.
template <int DT, int EPT>
__device__ void tok_digitize(const uint16_t* __restrict__ src, int v0, int nvec, int Kd, unsigned char* __restrict__ B,
                             float2* __restrict__ fs, int tt, int nthr) {
    constexpr int NT = 2;
    const int total = nvec * Kd / EPT, first = v0 * Kd / EPT;
    const int lane = tt & 31;
    for (int base0 = tt & ~31; base0 < total; base0 += NT * nthr) {
        EncTask<EPT> raw[NT];
#pragma unroll
        for (int q = 0; q < NT; ++q) {
            const int task = base0 + q * nthr + lane;
            if (task < total) tok_load_task<EPT>(src, Kd, first + task, raw[q]);
        }
#pragma unroll
        for (int q = 0; q < NT; ++q) {
            const int base = base0 + q * nthr;
            if (base >= total) break;  // warp-uniform
            tok_encode<DT, EPT>(raw[q], base + lane < total, first + min(base + lane, total - 1), Kd, B, fs);
        }
    }
}

// Grid barrier by one thread per CTA (after a block barrier whose writes it
// publishes) on a 64-bit arrival counter that is a multiple of the grid size
// between calls (it starts at zero and every CTA of every call arrives once
// per barrier): a release reduction (no reply to wait for), then relaxed
// polls until the counter reaches `target` -- the value read at the start of
// the call plus the grid size per barrier so far -- at most `limit` polls,
// and one acquire fence after the poll that saw it.  The counter cannot wrap.
__device__ __forceinline__ bool tok_grid_barrier(unsigned long long* ctr, unsigned long long target, int limit) {
    asm volatile("red.release.gpu.global.add.u64 [%0], 1;\n" ::"l"(ctr) : "memory");
    for (int it = 0; it < limit; ++it) {
        unsigned long long v;
        asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];\n" : "=l"(v) : "l"(ctr) : "memory");
        if (v >= target) {
            asm volatile("fence.acq_rel.gpu;\n" ::: "memory");  // with the load: an acquire pattern
            return true;
        }
    }
    return false;
}

// 4D tensor-map load into this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const void* map, int x, int y, int z, int w, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
        "[%6];" ::"r"(dst),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
        : "memory");
}

constexpr int kDrainLimit = 1 << 20;  // polls while waiting for this CTA's own copies before it exits

}  // namespace

template <int DT>
__global__ void __launch_bounds__(kTokThreads, 1) moe_token_kernel(const __grid_constant__ TokenArgs a) {
    extern __shared__ unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t s_full[kTokStages], s_empty[kTokStages];
    __shared__ int s_inds[kTokMaxM * kTokMaxK];      // token m's experts at m * K
    __shared__ float s_scores[kTokMaxM * kTokMaxK];
    __shared__ float s_part[kTokWarps];
    __shared__ float s_max;
    __shared__ int s_nan[kTokMaxM];
    __shared__ int s_stop, s_flag;
    __shared__ unsigned long long s_bar0;
    __shared__ volatile int s_abort, s_never;
    __shared__ float s_dv[kTokDnRows * kTokMaxK];
    tstamp(a, 0);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int G = gridDim.x, bx = blockIdx.x;
    const int H = a.H, I = a.I, E = a.E, K = a.K, M = a.M;
    unsigned char* smem =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    unsigned char* s_ring = smem + a.off_ring;
    float* s_logits = reinterpret_cast<float*>(smem + a.off_logits);
    unsigned char* s_xb = smem + a.off_xb;
    float2* s_xfs = reinterpret_cast<float2*>(smem + a.off_xfs);
    float* s_red_up = reinterpret_cast<float*>(smem + a.off_red_up);
    unsigned char* s_ab = smem + a.off_ab;
    float2* s_afs = reinterpret_cast<float2*>(smem + a.off_afs);
    float* s_red_dn = reinterpret_cast<float*>(smem + a.off_red_dn);

    if (tid == 0) {
        for (int s = 0; s < kTokStages; ++s) {
            mbar_init(&s_full[s], 1);
            mbar_init(&s_empty[s], kTokWarps);
        }
        mbar_fence_init();
        s_abort = 0;
        s_never = 0;
    }

    // Before the wait (nothing here reads memory the previous kernel may write):
    // the tensor maps' descriptors, and the routing inputs pulled into L2 -- a
    // prefetch only moves lines into L2, the point of coherence, so a later
    // load still sees whatever the previous kernel writes there.
    if (warp == kTokWarps) {
        if (lane < kTokMaps) asm volatile("prefetch.tensormap [%0];" ::"l"(&a.map[lane]) : "memory");
        const char* rin = a.logits ? reinterpret_cast<const char*>(a.logits) : reinterpret_cast<const char*>(a.inds_in);
        const int rbytes = a.logits ? M * E * 4 : M * K * 4;
        for (int o = 128 * lane; o < rbytes; o += 32 * 128)
            asm volatile("prefetch.global.L2 [%0];" ::"l"(rin + o) : "memory");
        if (!a.logits && lane == 0) asm volatile("prefetch.global.L2 [%0];" ::"l"(a.scores_in) : "memory");
    }

    pdl_wait();  // the previous kernel on the stream (e.g. the layer before) is complete
    pdl_launch_dependents();
    tstamp(a, 1);

    // ---- 1. routing first (it gates the weight stream), the token's loads in flight
    const int xtasks = H / 8;  // 8-element encoder tasks of the token (<= kTokCompute: H <= 4096)
    EncTask<8> xraw;
    if (tid < xtasks) tok_load_task<8>(a.x, H, tid, xraw);
    if (tid == 0) s_stop = a.stop ? __ldcg(a.stop) : 0;
    // the barrier count before this call (the previous call on the stream is complete)
    if (tid == 0) s_bar0 = __ldcg(a.bar64);
    // one token: each thread holds one logit and the routing below ranks them
    // (its fast path); several: the logits go to shared memory and route_tokens
    // routes every token (with its scores)
    const float lc = (a.logits && M == 1 && tid < E) ? __ldcg(a.logits + tid) : -INFINITY;
    int flag;  // a NaN logit (routing from logits) or an expert index out of range (given indices)
    if (a.logits && M == 1) {
        s_logits[tid] = lc;  // E <= kTokThreads
        flag = __syncthreads_or(tid < E && isnan(lc));
    } else if (a.logits) {
        for (int i = tid; i < M * E; i += kTokThreads) s_logits[i] = __ldcg(a.logits + i);
        __syncthreads();
        if (warp < M) {
            int nan = 0;
            for (int e = lane; e < E; e += 32) nan |= isnan(s_logits[warp * E + e]);
            nan = __any_sync(0xffffffffu, nan);
            if (lane == 0) s_nan[warp] = nan;
        }
        __syncthreads();
        route_tokens(s_logits, s_nan, M, E, K, 0, kTokThreads, 1, s_inds, s_scores, nullptr, true);
        flag = 1;  // not the one-token fast path
    } else {
        int bad = 0;
        if (tid < M * K) {
            const int e = a.inds_in[tid];
            s_inds[tid] = e;
            s_scores[tid] = a.scores_in[tid];
            bad = e < 0 || e >= E;
        }
        flag = __syncthreads_or(bad);
        const int st0 = flag ? MOMIJ_ERR_EXPERT_INDEX : (s_stop ? MOMIJ_ERR_STOPPED : MOMIJ_OK);
        if (bx == 0 && tid == 0 && (!a.status_merge || st0 != MOMIJ_OK)) a.ctrl[kCtrlStatus] = st0;
        if (flag) return;  // uniform: every CTA sees the same indices
    }
    const bool fast = a.logits && M == 1 && !flag;  // one token routed by the ranking below
    if (fast) {
        // rank of candidate c over the P threads that share it: the number of
        // experts before it in value order, ties by the smaller bit-reversed index
        int P = 1;
        while (P < 32 && E * P * 2 <= kTokThreads) P <<= 1;
        const int c = tid / P, sub = tid & (P - 1);
        int r = 0;
        float lv = -INFINITY;
        if (c < E) {
            lv = s_logits[c];
            const unsigned rc = __brev((unsigned)c);
#pragma unroll 4
            for (int j = sub; j < E; j += P) {
                const float lj = s_logits[j];
                r += (lj > lv) | ((lj == lv) & (__brev((unsigned)j) < rc));
            }
        }
        for (int o = 1; o < P; o <<= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
        if (c < E && sub == 0 && r < K) {
            s_inds[r] = c;
            if (r == 0) s_max = lv;
        }
    } else if (a.logits && M == 1) {
        if (tid == 0) s_nan[0] = 1;
        __syncthreads();
        route_tokens(s_logits, s_nan, 1, E, K, 0, kTokThreads, 1, s_inds, s_scores, nullptr, false);
    }
    __syncthreads();
    const bool stopped = s_stop != 0;
    if (a.logits && bx == 0 && tid == 0 && (!a.status_merge || stopped))
        a.ctrl[kCtrlStatus] = stopped ? MOMIJ_ERR_STOPPED : MOMIJ_OK;
    tstamp(a, 2);

    // ---- work of this CTA ------------------------------------------------------
    const int tpe = I >> 3, T = K * tpe;  // up||gate tiles per expert slot, in all
    const int tl0 = (int)((long long)T * bx / G);
    const int ntiles = stopped ? 0 : (int)((long long)T * (bx + 1) / G) - tl0;
    const int rpc = a.rows_per_cta, n0 = rpc * bx;
    const int nrows = stopped ? 0 : max(0, min(rpc, H - n0));
    const int ncol_up = H >> 9, ncol_dn = I >> 9;  // 128-byte code columns per row
    const int srb_up = H / 32;                     // scale bytes per up||gate row (gs 64)
    const int n_up_st = (ntiles + 1) >> 1;
    const int n_st_tok = n_up_st + (nrows > 0 ? ncol_dn : 0);  // stages per token
    const int n_st = M * n_st_tok;
    const int RSU = tok_red_stride(ncol_up), RSD = tok_red_stride(ncol_dn);

    if (warp >= kTokWarps) {
        // ---- producer warpgroup: one lane issues every stage's TMA loads -------------
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kTokRegsProducer));
        if (warp == kTokWarps && lane == 0) {
            int issued = 0;
            for (int j = 0; j < n_st; ++j) {
                const int slot = j % kTokStages;
                if (j >= kTokStages &&
                    !mbar_wait_bounded(&s_empty[slot], ((j / kTokStages) + 1) & 1, a.spin_limit, &s_abort)) {
                    s_abort = 1;
                    break;
                }
                const uint32_t st = smem_u32(s_ring + (size_t)slot * kTokStageBytes);
                const int m = j / n_st_tok, jj = j - m * n_st_tok;  // token, its stage
                const int* inds = s_inds + m * K;
                if (jj < n_up_st) {
                    const int nt = min(2, ntiles - 2 * jj);
                    mbar_expect_tx(&s_full[slot], (uint32_t)(nt * (ncol_up * 2048 + 2 * 16 * srb_up)));
                    for (int q = 0; q < nt; ++q) {
                        const int gt = tl0 + 2 * jj + q, k = gt / tpe, i0 = (gt - k * tpe) * 8;
                        const int z = 2 * inds[k];
                        tma_load_4d(st + q * 16384, &a.map[0], 0, i0, 0, z, &s_full[slot]);
                        tma_load_3d(st + kTokSOff + q * 2048, &a.map[1], 0, i0, z, &s_full[slot]);
                        tma_load_3d(st + kTokBOff + q * 2048, &a.map[2], 0, i0, z, &s_full[slot]);
                    }
                } else {
                    const int c = jj - n_up_st;
                    mbar_expect_tx(&s_full[slot], (uint32_t)(K * rpc * (128 + 2 * 16)));
                    for (int k = 0; k < K; ++k) {
                        const int y = inds[k] * H + n0;
                        tma_load_2d(st + k * 4096, &a.map[3], c * 128, y, &s_full[slot]);
                        tma_load_2d(st + kTokSOff + k * 512, &a.map[4], c * 16, y, &s_full[slot]);
                        tma_load_2d(st + kTokBOff + k * 512, &a.map[5], c * 16, y, &s_full[slot]);
                    }
                }
                issued = j + 1;
            }
            // the CTA stays until every copy it issued has landed
            for (int j = max(0, issued - kTokStages); j < issued; ++j)
                if (!mbar_wait_bounded(&s_full[j % kTokStages], (j / kTokStages) & 1, kDrainLimit, &s_never)) break;
        }
        return;
    }
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kTokRegsCompute));

    // ---- the tokens one after another; the producer streams ahead across them ---------
    bool any_fail = false;  // a wait gave up or a grid barrier did not complete
#pragma unroll 1
    for (int m = 0; m < M; ++m) {
        const int* inds_m = s_inds + m * K;
        float* scores_m = s_scores + m * K;
        const int jm = m * n_st_tok;  // the token's first stage
        // ---- token encoding (and the one-token scores) while its first stages land ------
        if (tid < ((xtasks + 31) & ~31)) tok_encode<DT, 8>(xraw, tid < xtasks, min(tid, xtasks - 1), H, s_xb, s_xfs);
        if (fast) {
            // softmax denominator over all experts (max = the top-ranked logit);
            // the renormalised scores follow after the up||gate phase
            float ez = tid < E ? expf(lc - s_max) : 0.f;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ez += __shfl_xor_sync(0xffffffffu, ez, o);
            if (lane == 0) s_part[warp] = ez;
        }
        bar_sync(1, kTokCompute);
        tstamp(a, 3);

        // Digit operand fragments of a code column (bf[slab][class] = (b0, b1);
        // lanes whose column group is not their A group hold zeros) and the
        // factors of the lane's groups 8c + 4 (t >> 1) + s, s = 0..3.
        const bool bact = (g >> 2) == (t >> 1);
        const int bl = (t >> 1) * 8 + (t & 1) * 4 + (g & 3);  // the lane's entry L, before the swizzle
        const int hsw = (t >> 1) * 8;  // L >= 8: the entry's two 8-byte halves stored swapped
        uint2 bf[4][4];
        float2 fsl[4];
        auto load_b = [&](const unsigned char* col, const float2* fsg) {
#pragma unroll
            for (int s = 0; s < 4; ++s)
#pragma unroll
                for (int pp = 0; pp < 2; ++pp) {
                    uint2 ev = make_uint2(0u, 0u), od = make_uint2(0u, 0u);  // even, odd class
                    if (bact) {
                        const unsigned char* en = col + s * 512 + pp * 256 + (((bl & 8) | ((bl & 7) ^ s)) * 16);
                        ev = *reinterpret_cast<const uint2*>(en + hsw);
                        od = *reinterpret_cast<const uint2*>(en + (hsw ^ 8));
                    }
                    bf[s][2 * pp] = ev;
                    bf[s][2 * pp + 1] = od;
                }
            const float4 f0 = *reinterpret_cast<const float4*>(fsg + 4 * (t >> 1));
            const float4 f1 = *reinterpret_cast<const float4*>(fsg + 4 * (t >> 1) + 2);
            fsl[0] = make_float2(f0.x, f0.y);
            fsl[1] = make_float2(f0.z, f0.w);
            fsl[2] = make_float2(f1.x, f1.y);
            fsl[3] = make_float2(f1.z, f1.w);
        };

        // One 16-row tile of 128-byte swizzled code rows (row r < 8 at cb + 128 r,
        // row 8 + r at cb + hi + 128 r): rows g (even t) or g + 8 (odd t) of the
        // lane's four groups, summed as
        // (G_j0 + .. + G_j3) + (G_j4 + .. + G_j7); `sv`, `bv`: the four scales and
        // biases of the lane's row and groups.  Lanes t = 0, 1 return rows g, g + 8.
        const bool odd = t & 1;
        auto compute = [&](const unsigned char* cb, int hi, uint2 sv, uint2 bv) -> float {
            uint2 ra[4], rb[4];
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                const int off = (((s + 4 * (t >> 1)) ^ (g & 7)) << 4) + 8 * (t & 1);
                ra[s] = *reinterpret_cast<const uint2*>(cb + g * 128 + off);
                rb[s] = *reinterpret_cast<const uint2*>(cb + hi + g * 128 + off);
            }
            int acc[4][4];
#pragma unroll
            for (int s = 0; s < 4; ++s)
#pragma unroll
                for (int r = 0; r < 4; ++r) acc[s][r] = 0;
#pragma unroll
            for (int p = 0; p < 4; ++p) {
                const uint32_t m = 0x03030303u << (2 * p);
#pragma unroll
                for (int s = 0; s < 4; ++s)
                    mma_u8s8(acc[s], ra[s].x & m, rb[s].x & m, ra[s].y & m, rb[s].y & m, bf[s][p].x, bf[s][p].y);
            }
            const uint32_t sw[2] = {sv.x, sv.y}, bw[2] = {bv.x, bv.y};
            float v = 0.f;
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                // columns 2t, 2t+1 of rows g and g + 8: digits (D0, D1) on even t, (D2, D3) on
                // odd t; each lane folds its pairs (|D| < 2^20, so 256 D + D' fits), swaps one
                // with its neighbour and keeps row g (even t) or g + 8 (odd t)
                const int* c = acc[s];
                const int pg = c[0] * 256 + c[1], pg8 = c[2] * 256 + c[3];
                const int rv = __shfl_xor_sync(0xffffffffu, odd ? pg : pg8, 1);
                const int dh = odd ? rv : pg, dl = odd ? pg8 : rv;  // 256 D0 + D1, 256 D2 + D3
                const float f = fmaf((float)dh, 65536.f, (float)dl);
                const float sf = Half<DT>::to_f(static_cast<uint16_t>(sw[s >> 1] >> (16 * (s & 1))));
                const float bb = Half<DT>::to_f(static_cast<uint16_t>(bw[s >> 1] >> (16 * (s & 1))));
                v += fmaf(sf, f * fsl[s].x, bb * fsl[s].y);
            }
            v += __shfl_xor_sync(0xffffffffu, v, 2);
            return v;
        };

        bool okw = true;  // this warp's waits all succeeded
        // ---- 2. up||gate phase ---------------------------------------------------
        {
            const int q = warp >> 3, c = warp & 7;
            if (c < ncol_up) load_b(s_xb + (size_t)c * 2048, s_xfs + 8 * c);
            const int row = g + 8 * (t & 1);
#pragma unroll 1
            for (int jj = 0; jj < n_up_st; ++jj) {
                const int j = jm + jj, slot = j % kTokStages;
                okw = mbar_wait_bounded(&s_full[slot], (j / kTokStages) & 1, a.spin_limit, &s_abort);
                if (!okw) break;  // the slot stays held: the producer stops at it
                const int tau = 2 * jj + q;
                if (c < ncol_up && tau < ntiles) {
                    const unsigned char* st = s_ring + (size_t)slot * kTokStageBytes;
                    const unsigned char* sbr = st + q * 2048 + row * srb_up;
                    const int so = srb_up == 128 ? (((c ^ (row & 7)) << 4) + 8 * (t >> 1)) : (c * 16 + 8 * (t >> 1));
                    const uint2 sv = *reinterpret_cast<const uint2*>(sbr + kTokSOff + so);
                    const uint2 bv = *reinterpret_cast<const uint2*>(sbr + kTokBOff + so);
                    const float v = compute(st + q * 16384 + c * 1024, ncol_up * 1024, sv, bv);
                    if (t < 2) s_red_up[(tau * 16 + g + 8 * t) * RSU + c] = v;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&s_empty[slot]);
            }
        }
        if (!okw && lane == 0) s_abort = 1;
        bar_sync(1, kTokCompute);
        tstamp(a, 4);
        // staged SwiGLU of each row pair of the slice (code columns summed in order)
        if (tid < 8 * ntiles && !s_abort) {
            const int tau = tid >> 3, i = tid & 7;
            const int gt = tl0 + tau, k = gt / tpe, i0 = (gt - k * tpe) * 8;
            const float* ru = s_red_up + (tau * 16 + i) * RSU;
            const float* rg = ru + 8 * RSU;
            float up = 0.f, gate = 0.f;
            for (int c = 0; c < ncol_up; ++c) {
                up += ru[c];
                gate += rg[c];
            }
            a.act[((size_t)m * K + k) * I + i0 + i] = swiglu_staged<DT>(up, gate, a.clamp);
        }
        if (a.logits && M == 1 && warp == kTokWarps - 1) {
            if (fast) {
                // the selected gates renormalised by their sum in k order
                float z = 0.f;
                for (int w = 0; w < kTokWarps; ++w) z += s_part[w];
                const float gate = lane < K ? expf(s_logits[s_inds[lane]] - s_max) / z : 0.f;
                float sum = 0.f;
                for (int k = 0; k < K; ++k) sum += __shfl_sync(0xffffffffu, gate, k);
                if (lane < K) s_scores[lane] = gate / sum;
            } else {
                route_scores_warp(s_logits, E, K, s_inds, s_scores);
            }
        }
        // the residual rows this CTA updates at the end, in flight meanwhile
        const uint16_t hres = (a.h && tid < nrows) ? a.h[(size_t)m * H + n0 + tid] : (uint16_t)0;

        // ---- 3. grid barrier ------------------------------------------------------------
        bar_sync(1, kTokCompute);
        if (bx == 0 && tid < K) {
            if (a.inds_out) a.inds_out[m * K + tid] = inds_m[tid];
            if (a.scores_out) a.scores_out[m * K + tid] = scores_m[tid];
        }
        tstamp(a, 5);
        if (tid == 0) {
            // every CTA arrives once per token, also after a failure (then without waiting)
            const bool okb =
            tok_grid_barrier(a.bar64, s_bar0 + (unsigned long long)(m + 1) * G, s_abort ? 0 : a.spin_limit);
            if (!okb) s_abort = 1;
            s_flag = okb;
        }
        bar_sync(1, kTokCompute);
        const bool fine = s_flag != 0 && !s_abort;
        tstamp(a, 6);

        // ---- 4. down phase: the K act vectors encoded, then warp 2k + q takes
        // expert slot k's 16-row half q
        if (fine && nrows > 0) tok_digitize<DT, 16>(a.act + (size_t)m * K * I, 0, K, I, s_ab, s_afs, tid, kTokCompute);
        tstamp(a, 9);
        bar_sync(1, kTokCompute);
        // the next token's elements, in flight during this token's down phase
        if (m + 1 < M && tid < xtasks) tok_load_task<8>(a.x + (size_t)(m + 1) * H, H, tid, xraw);
        if (nrows > 0) {
            const int k = warp >> 1, q = warp & 1;
            const int row = g + 8 * (t & 1);
            const bool mine = k < K && 16 * q < nrows;
            okw = true;
#pragma unroll 1
            for (int c = 0; c < ncol_dn; ++c) {
                const int j = jm + n_up_st + c, slot = j % kTokStages;
                okw = mbar_wait_bounded(&s_full[slot], (j / kTokStages) & 1, a.spin_limit, &s_abort);
                if (!okw) break;
                if (fine && mine) {
                    load_b(s_ab + (size_t)k * tok_b_bytes(I) + (size_t)c * 2048, s_afs + (size_t)k * (I >> 6) + 8 * c);
                    const unsigned char* st = s_ring + (size_t)slot * kTokStageBytes;
                    const int so = k * 512 + (16 * q + row) * 16 + 8 * (t >> 1);
                    const uint2 sv = *reinterpret_cast<const uint2*>(st + kTokSOff + so);
                    const uint2 bv = *reinterpret_cast<const uint2*>(st + kTokBOff + so);
                    const float v = compute(st + k * 4096 + q * 2048, 1024, sv, bv);
                    const int r = 16 * q + g + 8 * t;
                    if (t < 2) {
                        if (c + 1 < ncol_dn) {
                            s_red_dn[(k * kTokDnRows + r) * RSD + c] = v;
                        } else {
                            // the last column: the expert's down value of the row, summed over
                            // the columns in order and rounded like a gather output
                            const float* rd = s_red_dn + (k * kTokDnRows + r) * RSD;
                            float dv = 0.f;
                            for (int cc = 0; cc < c; ++cc) dv += rd[cc];
                            dv += v;
                            if (r < nrows) s_dv[r * kTokMaxK + k] = Half<DT>::to_f(Half<DT>::from_f(dv));
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&s_empty[slot]);
            }
            if (!okw && lane == 0) s_abort = 1;
        }
        bar_sync(1, kTokCompute);
        tstamp(a, 7);
        any_fail = any_fail || s_abort || !s_flag;

        // ---- 5. combine of the CTA's rows ----------------------------------------------
        if (fine && !s_abort && nrows > 0) {
            if (tid < nrows) {
                float acc = 0.f;
                for (int k = 0; k < K; ++k) acc = fmaf(s_dv[tid * kTokMaxK + k], scores_m[k], acc);
                const size_t n = (size_t)m * H + n0 + tid;
                if (a.h) {
                    const float delta = Half<DT>::to_f(Half<DT>::from_f(acc));
                    a.h[n] = Half<DT>::from_f(Half<DT>::to_f(hres) + delta);
                } else {
                    a.y[n] = Half<DT>::from_f(acc);
                }
            }
        }
        tstamp(a, 8);
    }  // tokens
    if (tid == 0 && any_fail) atomicExch(a.ctrl + kCtrlError, MOMIJ_ERR_TIMEOUT);
}

template __global__ void moe_token_kernel<MOMIJ_DTYPE_BF16>(const __grid_constant__ TokenArgs);
template __global__ void moe_token_kernel<MOMIJ_DTYPE_F16>(const __grid_constant__ TokenArgs);

}  // namespace momij
