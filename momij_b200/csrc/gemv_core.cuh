// gemv_core.cuh -- the streaming 2-bit gather-GEMV engine shared by the
// standalone gather-GEMV kernel (gemv.cu) and the fused MoE layer kernel
// (layer.cu).
//
// Arithmetic: the reference's gqmm2_rows (momij SeedlessMetal.swift:
// 2145-2221) evaluates y = sum_g s_g*sum(q*x) + b_g*sum(x) with fp32 FMAs.
// Here the inner products sum(q*x) run on the tensor cores exactly:
//   * codes q become u8 operands: one AND per 4 codes per "class" p (the code
//     at bit offset 2p of every byte), i.e. the u8 value q*4^p; no shifts;
//   * each activation vector is split into 64-element digit groups; a group
//     with largest magnitude in [2^E, 2^(E+1)) is written as the integers
//     x*2^(21-E) = 65536*d0 + 256*d1 + d2 with balanced int8 digits (exact for
//     every element within 2^14 of the group maximum, otherwise rounded at
//     2^-22 of it -- below the fp32 rounding of the reference's accumulator);
//   * mma.sync m16n8k32 u8 x s8 -> s32 accumulates the four classes with a
//     Horner shift (D <<= 2 between classes), so each digit plane's dot
//     product is exact (units of several tokens shift the operand instead,
//     (w >> 2p) & 0x03030303, once for all their tokens, and scale the
//     result by 64 exactly);
//   * the N dimension of the MMA separates digit groups and digit planes:
//     an MMA's K slab holds the codes of two digit groups, and its 8 columns
//     are (group, digit 0|1|2|unused), so one MMA per class and K half gives
//     every group's three plane sums and the fp32 epilogue applies that
//     group's scale and bias:
//       acc += s * (65536*D0 + 256*D1 + D2) * 2^(E-27) + b * sum(x).
//
// Data movement: the phase's work is a list of *items*, each one 256-code
// chunk (the K range of one warp) of one tile of 16 MMA rows (16 output rows,
// or 8 up rows + the 8 matching gate rows).  Warp w takes items w, w + 16,
// ... (tile-major, so the 16 warps read neighbouring chunks of the same rows
// at the same time) and streams them through a private ring of STAGES slots
// with 16-B cp.async copies, STAGES - 1 items ahead, waiting with
// cp.async.wait_group: no warp waits for another while streaming, and no
// wait can spin.  The item sequence runs on across phases, so the first items
// of a phase stream while the previous phase ends.  Per-thread 16-B copies
// keep ~140 KB in flight per SM and stream faster than bulk (TMA) row copies
// at these row sizes.
#pragma once

#include "kernels.cuh"

namespace momij {

constexpr int kConsumerWarps = 16;
constexpr int kConsumerThreads = 32 * kConsumerWarps;
constexpr int kGemvThreads = kConsumerThreads;
constexpr int kBarConsumers = 1;  // named barrier id used by the consumer warps
constexpr int kWaitLimit = 1 << 22;  // bounded mbarrier waits (then MOMIJ_ERR_TIMEOUT)

// Balanced base-256 digits of |v| < 2^22: v = 65536*d[0] + 256*d[1] + d[2],
// d[1], d[2] in [-128, 127], d[0] in [-64, 64].
__device__ __forceinline__ void split3(int v, int (&d)[3]) {
    d[2] = ((v + 128) & 255) - 128;
    const int t = (v - d[2]) >> 8;
    d[1] = ((t + 128) & 255) - 128;
    d[0] = (t - d[1]) >> 8;
}

// Encode `nvec` vectors (vector i is row vecs[i] of x, Kd elements) into digit
// planes laid out for the B fragment: per digit group of 64 elements, byte
// 64 d + 16 p + 8 u + i holds digit d of element 4 (8 u + i) + p (code class
// p = element % 4; u, i: the half and byte of the group's 16 code bytes a
// lane reads), so one 8-byte load gives a lane both B registers of an MMA
// step.  8 lanes per group;
// `nthreads` threads (from thread 0) take part.  Loads bypass L1 (the vectors
// may have been written by other CTAs).
template <int DT>
__device__ void digitize(const uint16_t* __restrict__ x, const int* __restrict__ vecs, int nvec,
                         int Kd, uint8_t* __restrict__ dig, float2* __restrict__ fs, int nthreads) {
    const int nDG = Kd >> 6;
    const int total = nvec * nDG * 8;
    const int lane = threadIdx.x & 31;
    for (int base = (threadIdx.x & ~31); base < total; base += nthreads) {
        const int idx = base + lane;
        const bool valid = idx < total;
        const int dgi = idx >> 3, sub = idx & 7;
        const int slot = dgi / nDG, dg = dgi - slot * nDG;
        float v[8];
        float mx = 0.f, sum = 0.f;
        if (valid) {
            const uint16_t* src = x + (size_t)vecs[slot] * Kd + dg * 64 + sub * 8;
            const uint4 raw = __ldcg(reinterpret_cast<const uint4*>(src));
            const uint32_t r[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                v[2 * i] = Half<DT>::to_f(static_cast<uint16_t>(r[i] & 0xffffu));
                v[2 * i + 1] = Half<DT>::to_f(static_cast<uint16_t>(r[i] >> 16));
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                mx = fmaxf(mx, fabsf(v[i]));
                sum += v[i];
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
        uint8_t* gp = dig + (size_t)dgi * kDgStride;
        const int pos0 = 8 * (sub >> 2) + 2 * (sub & 3);
#pragma unroll
        for (int tt = 0; tt < 4; ++tt) {  // elements 8 sub + tt and 8 sub + tt + 4: class tt
            int dA[3], dB[3];
            split3(__float2int_rn(v[tt] * scale), dA);
            split3(__float2int_rn(v[tt + 4] * scale), dB);
            const int pos = 16 * tt + pos0;
#pragma unroll
            for (int d = 0; d < 3; ++d)
                *reinterpret_cast<uint16_t*>(gp + 64 * d + pos) =
                    static_cast<uint16_t>((dA[d] & 0xff) | ((dB[d] & 0xff) << 8));
        }
        if (sub == 0) fs[dgi] = make_float2(ldexpf(1.f, E - 27), sum);
    }
}

__device__ __forceinline__ uint4 lds128(const unsigned char* p) {
    return *reinterpret_cast<const uint4*>(p);
}
__device__ __forceinline__ uint2 lds64(const unsigned char* p) {
    return *reinterpret_cast<const uint2*>(p);
}

// Work description of one gather-GEMV phase, all in shared memory.
struct PhaseTables {
    const int4* tiles;  // (local unit, first row in the expert, rows, 0)
    const int4* units;  // per local unit: (expert, first sorted position, pairs, 0)
    const int* uslot;   // [local unit][TMAX]: digit slot of the unit's j-th pair
    int ntiles;
};

struct PhaseWeights {
    const uint32_t* w;  // [E, N, Kd/16]
    const uint16_t* s;  // [E, N, Kd/gs]
    const uint16_t* b;
    int N;              // rows per expert
    int Ru;             // up||gate: first gate row (= I); rows mode: unused
    int Kd;
};

// An item is one tile (16 MMA rows) x two adjacent 256-code chunks, i.e. 128
// code bytes -- one whole cache line -- per row: the copies of a warp then
// request four full lines per instruction.
__host__ __device__ constexpr int item_tiles(int) { return 1; }
constexpr int kItemChunks = 2;
// One warp's ring slot: the 16 rows x 128 code bytes of one item.
__host__ __device__ constexpr int slot_bytes(int) { return 16 * 128; }
// Scale/bias buffer of an epilogue batch: scales [tiles * 16][Kd/gs] then
// biases (halves); MMA row r of the batch's tile k at row 16 k + r.
// Row stride (halves) of the scale/bias buffer: the epilogue's lanes read
// one column of 16 rows at once, so rows are padded to a word count that
// spreads them over the banks (= 4 mod 8 words with 16-B rows, so rows r and
// r + 8 share a bank at most; an odd word count with 4-B rows).  With 16-B
// rows nsb % 8 == 0, so nsb / 2 words is 0 or 4 mod 8.
__host__ __device__ constexpr int sb_row_halves(int nsb, bool rows16) {
    return rows16 ? 2 * ((nsb / 2) % 8 == 4 ? nsb / 2 : nsb / 2 + 4) : 2 * (((nsb + 1) / 2) | 1);
}
// pad: rows padded by sb_row_halves (at most 8 halves more).  The fused
// layer kernel pads only for one-token units: with several tokens its shared
// memory is tight and smaller epilogue batches measured worse than the bank
// conflicts.
__host__ __device__ constexpr int sb_bytes_per_tile(int Kd, int gs, bool pad) {
    return 16 * (Kd / gs + (pad ? 8 : 0)) * 2 * 2;
}

// Red-buffer floats per tile: [chunk pairs][TMAX][16 rows], each the sum of
// one item's two chunks (chunk 2cp, then + chunk 2cp + 1), a chunk's value
// being ((G0 + G1) + (G2 + G3)) over its four digit groups.
// A red-buffer row (16 MMA rows of one chunk pair and token slot) takes
// red_row(TMAX) floats.  With one token the padding to 20 spreads the 8 lanes
// that sum one output over 8 chunk pairs across distinct banks; units of
// several tokens keep 16 (their larger buffers would cost epilogue batch
// size, which measured worse than the conflicts).
__host__ __device__ constexpr int red_row(int tmax) { return tmax == 1 ? 20 : 16; }
template <int TMAX>
__host__ __device__ constexpr int red_floats_per_tile(int nK) { return ((nK + 1) / 2) * TMAX * red_row(TMAX); }
// Sum of the partials of MMA row r (0..15) of token slot j of one tile over
// its n entries (chunk pairs), computed by L lanes (an aligned group; L = 1, 2, 4 or 8; lane
// `sub` of the group).  The association is fixed whatever L is:
// with S_v the sequential sum of the chunk values v, v + 8, ... (v = 0..7),
// the result is ((S0 + S1) + (S2 + S3)) + ((S4 + S5) + (S6 + S7)).
template <int TMAX, int L>
__device__ __forceinline__ float tile_sum(const float* red, int n, int j, int r, int sub) {
    constexpr int V = 8 / L;
    float part[V];
#pragma unroll
    for (int v = 0; v < V; ++v) {
        float acc = 0.f;
        for (int cc = sub * V + v; cc < n; cc += 8) acc += red[(cc * TMAX + j) * red_row(TMAX) + r];
        part[v] = acc;
    }
#pragma unroll
    for (int w = 1; w < V; w <<= 1)
#pragma unroll
        for (int v = 0; v < V; v += 2 * w) part[v] += part[v + w];
    float acc = part[0];
#pragma unroll
    for (int o = 1; o < L; o <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    return acc;
}

// Epilogue of tiles [tfirst, tlast) whose partials are in red_base (tile
// tau at (tau - tfirst) * per_tile), block-wide, 8 lanes per output (they
// read different chunks, so no bank conflicts between tiles):
// out(tile, j, r, v, v_gate) for every valid output (v_gate: the gate row's
// sum in up||gate mode).  Every thread of the block calls it.
template <int TMAX, int MODE, class Out>
__device__ void epilogue_tiles(int tfirst, int tlast, const float* red_base, int nK, const int4* tiles,
                               const int4* units, Out& out) {
    constexpr int TR = (MODE == kModeUpSwiglu) ? 8 : 16;
    const int per_tile = red_floats_per_tile<TMAX>(nK);
    const int items = (tlast - tfirst) * TMAX * TR;
    const int sub = threadIdx.x & 7;
    for (int base = 0; base < items; base += kConsumerThreads / 8) {
        const int it = base + (threadIdx.x >> 3);
        int tau = tfirst, j = 0, r = 0;
        bool valid = it < items;
        int4 tile = make_int4(0, 0, 0, 0);
        if (valid) {
            tau = tfirst + it / (TMAX * TR);
            j = (it / TR) % TMAX;
            r = it % TR;
            tile = tiles[tau];
            valid = j < units[tile.x].z && r < tile.z;
        }
        const float* red = red_base + (size_t)(tau - tfirst) * per_tile;
        const int ncp = (nK + 1) / 2;
        const float v = tile_sum<TMAX, 8>(red, ncp, j, r, sub);
        const float vg = (MODE == kModeUpSwiglu) ? tile_sum<TMAX, 8>(red, ncp, j, 8 + r, sub) : 0.f;
        if (valid && sub == 0) out(tile, j, r, v, vg);
    }
}

template <int DT, int GS, int MODE, int TMAX, int STAGES>
struct GemvPhase {
    static constexpr int TR = (MODE == kModeUpSwiglu) ? 8 : 16;  // output rows per tile
    static constexpr int DIST = STAGES - 1;  // items in flight ahead of the one computed
    static constexpr int SPC = 256 / GS;     // scale groups per row of a chunk
    static constexpr int SLOT = slot_bytes(TMAX);
    static constexpr bool kHorner = (TMAX == 1);  // class weights evened on the accumulators

    // Position in the warp's item sequence: tile and chunk pair.
    struct Iter {
        int tile, cp, n;  // n: items of this phase passed so far
    };

    PhaseTables T;
    PhaseWeights W;
    unsigned char* ring;  // this warp's STAGES slots
    int q0;               // ring position of this warp's first item of the phase
    int warp, lane, g, t, nK, ncp, count, dtile, dcp;
    uint64_t policy;
    Iter li, ci;  // next item to load, next item to compute
    float* red;   // partials of the current batch of tiles
    int tfirst;   // first tile of the current batch
    int per_tile;
    uint16_t* sb;   // the batch's scales, then biases (sb_bytes_per_tile per tile)
    int sb_tiles;   // tiles the scale/bias buffer holds (the batch size)
    uint64_t* sbar; // mbarrier of the batch's scale/bias copies
    int sb_par;     // its phase parity
    bool sb16;      // scale/bias rows and tensors 16-B aligned (16-B copies, else 4-B)
    int nsbp;       // row stride of the scale/bias buffer in halves (sb_row_halves)

    // ring_base: the block's rings (kConsumerWarps x STAGES x SLOT);
    // q0_: items this warp streamed through its ring in earlier phases;
    // sb_, sb_tiles_: the scale/bias buffer (batch size in tiles); sbar_: an
    // mbarrier initialised by sb_init.
    __device__ GemvPhase(const PhaseTables& tabs, const PhaseWeights& wts, unsigned char* ring_base,
                         int q0_, int nK_, uint16_t* sb_, int sb_tiles_, uint64_t* sbar_, bool pad_sb)
        : T(tabs), W(wts), q0(q0_), nK(nK_), sb(sb_), sb_tiles(sb_tiles_), sbar(sbar_), sb_par(0) {
        const int nsb = W.Kd / GS;
        sb16 = (nsb * 2) % 16 == 0 && (reinterpret_cast<uintptr_t>(W.s) % 16) == 0 &&
               (reinterpret_cast<uintptr_t>(W.b) % 16) == 0 && (reinterpret_cast<uintptr_t>(sb) % 16) == 0;
        nsbp = pad_sb ? sb_row_halves(nsb, sb16) : nsb;
        per_tile = red_floats_per_tile<TMAX>(nK_);
        warp = threadIdx.x >> 5;
        lane = threadIdx.x & 31;
        g = lane >> 2;
        t = lane & 3;
        ring = ring_base + (size_t)warp * STAGES * SLOT;
        ncp = (nK + kItemChunks - 1) / kItemChunks;
        const int nitems = T.ntiles * ncp;
        count = warp < nitems ? (nitems - warp + kConsumerWarps - 1) / kConsumerWarps : 0;
        dtile = kConsumerWarps / ncp;
        dcp = kConsumerWarps - dtile * ncp;
        li.tile = warp / ncp;
        li.cp = warp - li.tile * ncp;
        li.n = 0;
        ci = li;
        policy = l2_evict_first_policy();
    }

    // Item k of this warp is (tile, chunk pair) number warp + 16 k of the
    // phase, tile-major, so the 16 warps stream neighbouring chunks of the
    // same rows at the same time.
    __device__ __forceinline__ void advance(Iter& it) const {
        it.cp += dcp;
        it.tile += dtile;
        if (it.cp >= ncp) {
            it.cp -= ncp;
            ++it.tile;
        }
        ++it.n;
    }

    // Slot offset of 16-byte granule j (0..7) of MMA row r's 128 code bytes:
    // granules are permuted by j ^ f(r), f(r) = {0, 1, 4, 5}[r & 3], so the
    // 8-byte reads of four consecutive rows by a half-warp (two granules 2
    // apart per row) fall into distinct banks.
    static __device__ __forceinline__ int swz(int r, int j) {
        return r * 128 + 16 * (j ^ ((r & 1) | ((r & 2) << 1)));
    }

    // Global row of MMA row r (0..15) of tile `tile`, or -1 beyond the tile.
    __device__ __forceinline__ int tile_row(const int4& tile, int r) const {
        if (MODE == kModeUpSwiglu) {
            const int i = r & 7;
            if (i >= tile.z) return -1;
            return (r < 8) ? tile.y + i : W.Ru + tile.y + i;
        }
        return r < tile.z ? tile.y + r : -1;
    }

    // Copies the next item into its slot and commits one cp.async group (an
    // empty one past the end, so the group count stays in step with the
    // items).  Rows beyond the tile, and the second chunk when nK is odd, are
    // zero-filled.  Lane l copies granule l & 7 of rows (l >> 3) + 4 k.
    __device__ void load_next() {
        if (li.n < count) {
            const uint32_t dst = smem_u32(ring + ((q0 + li.n) % STAGES) * SLOT);
            const int4 tile = T.tiles[li.tile];
            const int part = lane & 7, r0 = lane >> 3;
            const bool pvalid = kItemChunks * li.cp + (part >> 2) < nK;
            const size_t rs = (size_t)(W.Kd >> 4);
            // rows r0 + 4k: up||gate: k = 0, 1 up rows, k = 2, 3 the gate rows
            const uint32_t* p0 =
                W.w + ((size_t)T.units[tile.x].x * W.N + tile.y + r0) * rs + (size_t)li.cp * 32 + part * 4;
            const uint32_t* p2 = (MODE == kModeUpSwiglu) ? p0 + (size_t)W.Ru * rs : p0 + 8 * rs;
            const int lim = (MODE == kModeUpSwiglu) ? tile.z : tile.z - 8;  // rows valid in p2's block
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int ri = r0 + 4 * (k & 1);
                const bool v = pvalid && ri < ((k < 2) ? tile.z : lim);
                const uint32_t* src = ((k < 2) ? p0 : p2) + (size_t)(4 * (k & 1)) * rs;
                cp_async16_hint(dst + swz(r0 + 4 * k, part), v ? src : W.w, v, policy);
            }
            advance(li);
        } else {
            ++li.n;
        }
        cp_async_commit();
    }

    // Scales and biases of tiles [tb0, tb1) into sb; every thread calls it
    // and then arrives on sbar (count kConsumerThreads) once its copies have
    // landed.  16-B cp.async pieces walk each row contiguously (4-B pieces
    // when rows or tensors are not 16-B aligned).
    __device__ void issue_sb(int tb0, int tb1) {
        constexpr int PARTS = (MODE == kModeUpSwiglu) ? 2 : 1;
        constexpr int PR = 16 / PARTS;  // MMA rows per part of a tile
        const int nsb = W.Kd / GS;
        const int psz = sb16 ? 16 : 4;
        const int ppr = nsb * 2 / psz;  // pieces per row
        const int per_tile = 2 * 16 * ppr;
        // this thread's pieces within a tile: i = threadIdx.x + 512 j
        for (int i = threadIdx.x; i < per_tile; i += kConsumerThreads) {
            const int tensor = i / (16 * ppr), rr = i - tensor * 16 * ppr;
            const int r = rr / ppr, pc = rr - r * ppr;
            const int part = r / PR, ri = r - part * PR;
            const uint16_t* gsrc = tensor ? W.b : W.s;
            const size_t goff = ((size_t)part * W.Ru + ri) * nsb;
            const uint32_t dst0 =
                smem_u32(sb + ((size_t)tensor * sb_tiles * 16 + r) * nsbp) + pc * psz;
            for (int k = tb0; k < tb1; ++k) {
                const int4 tile = T.tiles[k];
                if (ri >= tile.z) continue;
                const size_t grow = (size_t)T.units[tile.x].x * W.N + tile.y;
                const unsigned char* src =
                    reinterpret_cast<const unsigned char*>(gsrc + grow * nsb + goff) + pc * psz;
                const uint32_t dst = dst0 + (uint32_t)((k - tb0) * 16 * nsbp * 2);
                if (sb16) cp_async16(dst, src, true);
                else cp_async4(dst, src, true);
            }
        }
        mbar_arrive_cp_async(sbar);
    }
    // Before computing a batch: its scales and biases have landed (bounded
    // wait; false if it gave up).
    __device__ bool wait_sb() {
        const uint32_t par = sb_par & 1;
        ++sb_par;
        for (int it = 0; it < kWaitLimit; ++it)
            if (mbar_try_wait(sbar, par)) return true;
        return false;
    }

    // Issues the first DIST items of the warp's item sequence through
    // `ahead()`, which loads the sequence's next item (possibly of the next
    // phase).
    template <class Ahead>
    __device__ void prefetch(Ahead& ahead) {
#pragma unroll 1
        for (int j = 0; j < DIST; ++j) ahead();
    }

    // MMA layout.  The chunk's 64 code bytes per row are four digit groups
    // of 16 bytes.  For K half h and code class p, lane (g, t) holds the 8
    // bytes 8 (t & 1) + [0, 8) of digit group G = 2 (t >> 1) + h of MMA rows
    // g and g + 8 (MMA k = 4t + i <-> byte i, k = 16 + 4t + i <-> byte
    // 4 + i of those 8), so an MMA covers groups h and 2 + h.  B column n is
    // (local group n >> 2, digit n & 3), digit 3 unused: a lane's B registers
    // are non-zero only when its column's group is its own (n >> 2 == t >> 1).
    // The accumulator columns 2t, 2t + 1 of lane t are digits (0, 1) for even
    // t and (2, -) for odd t of group G; a lane's two groups (h = 0, 1) are
    // adjacent, so their scales and activation factors load together.

    // One-token units keep the B fragments of their digit slot in registers
    // (one set per chunk of the item) while the digit groups stay the same.
    uint2 bc[kItemChunks][2][4];
    int bc_key[kItemChunks] = {-1, -1};

    __device__ __forceinline__ uint2 load_b(const uint8_t* __restrict__ dig, int slotdg, int h, int p,
                                            bool bActive) const {
        if (!bActive) return make_uint2(0u, 0u);
        return lds64(dig + (slotdg + 2 * (t >> 1) + h) * kDgStride + (g & 3) * 64 + p * 16 + (t & 1) * 8);
    }

    // Chunk ch of the current compute item (its slot at sp; chunk c of tile
    // tau): exact group partial sums (a Horner chain per K half: D <<= 2
    // between code classes) -> per-row fp32 sums, set (ch 0) or added (ch 1)
    // into acc[j] of lanes t < 2 (row g for t = 0, g + 8 for t = 1).
    // (tile, nT, slot: the item's tile, its unit's pairs and their digit
    // slots times the digit groups per vector, shared by the item's chunks.)
    __device__ __forceinline__ void compute_chunk(const unsigned char* sp, int ch, int tau, int c,
                                                  int nT, const int (&slot)[TMAX],
                                                  const uint8_t* __restrict__ dig,
                                                  const float2* __restrict__ fs, float (&acc)[TMAX]) {
        const bool bActive = (g & 3) < 3 && (g >> 2) == (t >> 1);
        const int rA = g, rB = g + 8;
        uint2 wa[2], wb[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int j = 4 * ch + 2 * (t >> 1) + h;
            wa[h] = lds64(sp + swz(rA, j) + 8 * (t & 1));
            wb[h] = lds64(sp + swz(rB, j) + 8 * (t & 1));
        }
        int slotdg[TMAX];
        int D[TMAX][2][4];
#pragma unroll
        for (int j = 0; j < TMAX; ++j) {
            slotdg[j] = slot[j] + 4 * c;
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int r = 0; r < 4; ++r) D[j][h][r] = 0;
        }
        if (TMAX == 1 && bc_key[ch] != slotdg[0]) {
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int p = 0; p < 4; ++p) bc[ch][h][p] = load_b(dig, slotdg[0], h, p, bActive);
            bc_key[ch] = slotdg[0];
        }

#pragma unroll
        for (int p = 0; p < 4; ++p) {
            // One token: class p enters as q*4^p (one AND) and a Horner shift
            // of the accumulators between classes evens the weights out.
            // Several tokens: the shift moves to the operand (q itself, one
            // shift + AND per word, shared by the tokens) instead of being
            // paid on every token's accumulators; D is then 64x smaller,
            // which the epilogue restores exactly.
            if (kHorner && p) {
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int r = 0; r < 4; ++r) D[0][h][r] <<= 2;
            }
            const uint32_t mask = 0x03030303u << (2 * p);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t a0 = kHorner ? (wa[h].x & mask) : ((wa[h].x >> (2 * p)) & 0x03030303u);
                const uint32_t a1 = kHorner ? (wb[h].x & mask) : ((wb[h].x >> (2 * p)) & 0x03030303u);
                const uint32_t a2 = kHorner ? (wa[h].y & mask) : ((wa[h].y >> (2 * p)) & 0x03030303u);
                const uint32_t a3 = kHorner ? (wb[h].y & mask) : ((wb[h].y >> (2 * p)) & 0x03030303u);
#pragma unroll
                for (int j = 0; j < TMAX; ++j) {
                    if (j < nT) {
                        const uint2 bv = (TMAX == 1) ? bc[ch][h][p] : load_b(dig, slotdg[j], h, p, bActive);
                        mma_u8s8(D[j][h], a0, a1, a2, a3, bv.x, bv.y);
                    }
                }
            }
        }

        // Even lanes finish row g, odd lanes row g + 8, of their two groups;
        // then lanes t and t ^ 2 add up the chunk's four groups:
        // (G0 + G1) + (G2 + G3).
        const bool odd = t & 1;
        const int srow = (tau - tfirst) * 16 + (odd ? g + 8 : g);  // the lane's row in the batch
        const int nsb = W.Kd / GS;
        const uint16_t* sb_s = sb;
        const uint16_t* sb_b = sb + (size_t)sb_tiles * 16 * nsbp;
        float sc[2], bi[2];
        if (SPC == 4) {  // two adjacent groups' halves in one 4-byte load
            const int si = srow * nsbp + 4 * c + 2 * (t >> 1);
            const uint32_t sv = *reinterpret_cast<const uint32_t*>(sb_s + si);
            const uint32_t bv = *reinterpret_cast<const uint32_t*>(sb_b + si);
            sc[0] = Half<DT>::to_f((uint16_t)(sv & 0xffffu));
            sc[1] = Half<DT>::to_f((uint16_t)(sv >> 16));
            bi[0] = Half<DT>::to_f((uint16_t)(bv & 0xffffu));
            bi[1] = Half<DT>::to_f((uint16_t)(bv >> 16));
        } else {  // gs = 128: both groups share one scale
            const int si = srow * nsbp + SPC * c + (t >> 1);
            sc[0] = sc[1] = Half<DT>::to_f(sb_s[si]);
            bi[0] = bi[1] = Half<DT>::to_f(sb_b[si]);
        }
#pragma unroll
        for (int j = 0; j < TMAX; ++j) {
            if (j < nT) {
                const float4 fsv = *reinterpret_cast<const float4*>(fs + slotdg[j] + 2 * (t >> 1));
                float part[2];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int* cacc = D[j][h];
                    const int s1 = __shfl_xor_sync(0xffffffffu, odd ? cacc[0] : cacc[2], 1);
                    const int s2 = __shfl_xor_sync(0xffffffffu, cacc[3], 1);
                    const int d0 = odd ? s1 : cacc[0];
                    const int d1 = odd ? s2 : cacc[1];
                    const int d2 = odd ? cacc[2] : s1;
                    float v = fmaf((float)d0, 65536.f, fmaf((float)d1, 256.f, (float)d2));
                    if (!kHorner) v *= 64.f;  // the Horner chain's 4^3, exactly (a power of two)
                    const float F = h ? fsv.z : fsv.x, S = h ? fsv.w : fsv.y;
                    part[h] = fmaf(sc[h], v * F, bi[h] * S);
                }
                float pr = part[0] + part[1];
                pr += __shfl_xor_sync(0xffffffffu, pr, 2);
                acc[j] = ch ? acc[j] + pr : pr;
            }
        }
    }

    // Main loop (every thread calls it, after the warp's first DIST items
    // were issued): at each item the warp issues the item DIST ahead in its
    // sequence through `ahead()` (which may belong to the next phase), waits
    // for its own current item and computes it.  Batches of sb_tiles tiles
    // (the host makes one batch cover the phase when shared memory allows) start with a wait for their scales and biases and end
    // with the block-wide epilogue between two block barriers, during which
    // the next batch's scales and biases are issued; the loads in flight keep
    // streaming across.  first_issued: the caller issued batch 0's scales and
    // biases (issue_sb) already.  Returns false if a bounded wait gave up.
    template <class Out, class Ahead>
    __device__ bool consume(const uint8_t* dig, const float2* fs, float* red_base, bool first_issued,
                            Out& out, Ahead& ahead) {
        red = red_base;
        bool ok = true;
        const int batch_tiles = sb_tiles;
        if (!first_issued && T.ntiles > 0) issue_sb(0, min(T.ntiles, batch_tiles));
#pragma unroll 1
        for (int tb0 = 0; tb0 < T.ntiles; tb0 += batch_tiles) {
            const int tb1 = min(T.ntiles, tb0 + batch_tiles);
            tfirst = tb0;
            ok &= wait_sb();
#pragma unroll 1
            while (ci.n < count && ci.tile < tb1) {
                ahead();
                cp_async_wait<DIST>();
                __syncwarp();
                const unsigned char* sp = ring + ((q0 + ci.n) % STAGES) * SLOT;
                const int ul = T.tiles[ci.tile].x;
                const int nT = (TMAX == 1) ? 1 : T.units[ul].z;
                int slot[TMAX];
#pragma unroll
                for (int j = 0; j < TMAX; ++j) slot[j] = ((j < nT) ? T.uslot[ul * TMAX + j] : 0) * (W.Kd >> 6);
                float acc[TMAX];
#pragma unroll
                for (int ch = 0; ch < kItemChunks; ++ch) {
                    const int c = kItemChunks * ci.cp + ch;
                    if (c < nK) compute_chunk(sp, ch, ci.tile, c, nT, slot, dig, fs, acc);
                }
                float* red_tile = red + (size_t)(ci.tile - tfirst) * per_tile;
                if (t < 2) {
#pragma unroll
                    for (int j = 0; j < TMAX; ++j)
                        if (j < nT) red_tile[(ci.cp * TMAX + j) * red_row(TMAX) + t * 8 + g] = acc[j];
                }
                __syncwarp();
                advance(ci);
            }
            bar_sync(kBarConsumers, kConsumerThreads);
            if (tb1 < T.ntiles) issue_sb(tb1, min(T.ntiles, tb1 + batch_tiles));
            epilogue_tiles<TMAX, MODE>(tb0, tb1, red_base, nK, T.tiles, T.units, out);
            bar_sync(kBarConsumers, kConsumerThreads);
        }
        return ok;
    }
};

// Thread 0: initialises a phase's scale/bias mbarrier (one cp.async arrival
// per thread and batch); the block synchronises before its first use.
__device__ __forceinline__ void sb_init(uint64_t* bar) {
    if (threadIdx.x == 0) {
        mbar_init(bar, kConsumerThreads);
        mbar_fence_init();
    }
}

// Before the block exits, wait until every cp.async this thread issued has
// landed, so no copy is still writing into shared memory.
__device__ __forceinline__ void ring_quiesce() { cp_async_wait<0>(); }

}  // namespace momij
