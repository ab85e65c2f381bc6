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
//     product is exact;
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

// Tiles per item: one-/two-token units take two tiles (32 MMA rows) per
// item, which share the item's B fragments and bookkeeping; larger units one.
__host__ __device__ constexpr int item_tiles(int tmax) { return tmax <= 2 ? 2 : 1; }
// One warp's ring slot: the 16 * item_tiles MMA rows of one 256-code chunk
// (64 B each), then their scales [rows][256/gs] and biases (halves).
__host__ __device__ constexpr int slot_bytes(int tmax) { return item_tiles(tmax) * (16 * 64 + 2 * 16 * 4 * 2); }

// Red-buffer floats per tile: [nK][TMAX][16 rows], each the sum of the four
// lane groups' partials of one chunk, (t0 + t1) + (t2 + t3).
template <int TMAX>
__host__ __device__ constexpr int red_floats_per_tile(int nK) { return nK * TMAX * 16; }
// Sum of the partials of MMA row r (0..15) of token slot j of one tile over
// all chunks, computed by L lanes (an aligned group; L = 1, 2, 4 or 8; lane
// `sub` of the group).  The association is fixed whatever L is:
// with S_v the sequential sum of the chunk values v, v + 8, ... (v = 0..7),
// the result is ((S0 + S1) + (S2 + S3)) + ((S4 + S5) + (S6 + S7)).
template <int TMAX, int L>
__device__ __forceinline__ float tile_sum(const float* red, int nK, int j, int r, int sub) {
    constexpr int V = 8 / L;
    float part[V];
#pragma unroll
    for (int v = 0; v < V; ++v) {
        float acc = 0.f;
        for (int cc = sub * V + v; cc < nK; cc += 8) acc += red[(cc * TMAX + j) * 16 + r];
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
// tau at (tau - tfirst) * per_tile), block-wide, 8 lanes per output:
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
        const float v = tile_sum<TMAX, 8>(red, nK, j, r, sub);
        const float vg = (MODE == kModeUpSwiglu) ? tile_sum<TMAX, 8>(red, nK, j, 8 + r, sub) : 0.f;
        if (valid && sub == 0) out(tile, j, r, v, vg);
    }
}

template <int DT, int GS, int MODE, int TMAX, int STAGES>
struct GemvPhase {
    static constexpr int TR = (MODE == kModeUpSwiglu) ? 8 : 16;  // output rows per tile
    static constexpr int DIST = STAGES - 1;  // items in flight ahead of the one computed
    static constexpr int SPC = 256 / GS;     // scale groups per row of a chunk
    static constexpr int RT = item_tiles(TMAX);
    static constexpr int ROWS = 16 * RT;     // MMA rows per item
    static constexpr int CODE_BYTES = ROWS * 64;
    static constexpr int SLOT = slot_bytes(TMAX);

    // Position in the warp's item sequence: tile group (RT tiles) and chunk.
    struct Iter {
        int grp, c, n;  // n: items of this phase passed so far
    };

    PhaseTables T;
    PhaseWeights W;
    unsigned char* ring;  // this warp's STAGES slots
    int q0;               // ring position of this warp's first item of the phase
    int warp, lane, g, t, nK, count, dgrp, dc;
    bool sb8;  // scales/biases copied as 8-B pieces (else 4-B)
    uint64_t policy;
    Iter li, ci;  // next item to load, next item to compute
    float* red;   // partials of the current batch of tiles
    int tfirst;   // first tile of the current batch
    int per_tile;

    // ring_base: the block's rings (kConsumerWarps x STAGES x SLOT);
    // q0_: items this warp streamed through its ring in earlier phases.
    __device__ GemvPhase(const PhaseTables& tabs, const PhaseWeights& wts, unsigned char* ring_base,
                         int q0_, int nK_)
        : T(tabs), W(wts), q0(q0_), nK(nK_) {
        per_tile = red_floats_per_tile<TMAX>(nK_);
        warp = threadIdx.x >> 5;
        lane = threadIdx.x & 31;
        g = lane >> 2;
        t = lane & 3;
        ring = ring_base + (size_t)warp * STAGES * SLOT;
        const int nitems = ((T.ntiles + RT - 1) / RT) * nK;
        count = warp < nitems ? (nitems - warp + kConsumerWarps - 1) / kConsumerWarps : 0;
        dgrp = kConsumerWarps / nK;
        dc = kConsumerWarps - dgrp * nK;
        li.grp = warp / nK;
        li.c = warp - li.grp * nK;
        li.n = 0;
        ci = li;
        sb8 = SPC == 4 && (reinterpret_cast<uintptr_t>(W.s) % 8) == 0 &&
              (reinterpret_cast<uintptr_t>(W.b) % 8) == 0;
        policy = l2_evict_first_policy();
    }

    // Item k of this warp is (tile group, chunk) number warp + 16 k of the
    // phase, group-major, so the 16 warps stream neighbouring chunks of the
    // same rows at the same time.
    __device__ __forceinline__ void advance(Iter& it) const {
        it.c += dc;
        it.grp += dgrp;
        if (it.c >= nK) {
            it.c -= nK;
            ++it.grp;
        }
        ++it.n;
    }

    // Offset of 32-byte half h of MMA row r's 64 code bytes in a slot: the
    // halves of rows 2 and 3 (mod 4) are swapped, so the 8-byte reads of four
    // consecutive rows by a half-warp fall into distinct banks.
    static __device__ __forceinline__ int swz(int r, int h) { return 32 * (h ^ ((r >> 1) & 1)); }

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
    // items).  Rows beyond the tiles are zero-filled.
    __device__ void load_next() {
        if (li.n < count) {
            const uint32_t dst = smem_u32(ring + ((q0 + li.n) % STAGES) * SLOT);
            int4 tile[RT];
            size_t eb[RT];
#pragma unroll
            for (int rt = 0; rt < RT; ++rt) {
                const int tau = li.grp * RT + rt;
                tile[rt] = (tau < T.ntiles) ? T.tiles[tau] : make_int4(0, 0, 0, 0);
                eb[rt] = (size_t)T.units[tile[rt].x].x * W.N;
            }
            const int ra = lane >> 2, part = lane & 3;
            const size_t rs = (size_t)(W.Kd >> 4);
            const size_t co = (size_t)li.c * 16 + part * 4;
#pragma unroll
            for (int rt = 0; rt < RT; ++rt) {
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    const int row = tile_row(tile[rt], ra + 8 * hh);
                    const int mr = rt * 16 + ra + 8 * hh;
                    cp_async16_hint(dst + mr * 64 + swz(mr, part >> 1) + 16 * (part & 1),
                                    W.w + (row >= 0 ? (eb[rt] + row) * rs + co : 0), row >= 0,
                                    policy);
                }
            }
            // scales then biases of the item's rows: piece lane + 32 k ->
            // (tensor, row); 2 * ROWS = 32 * RT pieces
#pragma unroll
            for (int k = 0; k < RT; ++k) {
                const int it = lane + 32 * k;
                const int sb = it / ROWS, r = it - sb * ROWS;
                const bool second = RT > 1 && r >= 16;  // row of the item's second tile
                const int4 tl = second ? tile[RT - 1] : tile[0];
                const size_t ebr = second ? eb[RT - 1] : eb[0];
                const int row = tile_row(tl, r & 15);
                const uint16_t* src =
                    (sb ? W.b : W.s) +
                    (row >= 0 ? (ebr + row) * (size_t)(W.Kd / GS) + (size_t)li.c * SPC : 0);
                const uint32_t sdst = dst + CODE_BYTES + (sb * ROWS + r) * SPC * 2;
                if (sb8) {
                    cp_async8_hint(sdst, src, row >= 0, policy);
                } else {
#pragma unroll
                    for (int k = 0; k < SPC / 2; ++k) cp_async4(sdst + 4 * k, src + 2 * k, row >= 0);
                }
            }
            advance(li);
        } else {
            ++li.n;
        }
        cp_async_commit();
    }

    // Issues the first DIST items of the warp's item sequence through
    // `ahead()`, which loads the sequence's next item (possibly of the next
    // phase).
    template <class Ahead>
    __device__ void prefetch(Ahead& ahead) {
#pragma unroll 1
        for (int j = 0; j < DIST; ++j) ahead();
    }

    // MMA layout.  For K half h (code bytes 32h..32h+31 of the chunk, digit
    // groups 2h and 2h+1) and code class p, lane (g, t) holds the A bytes
    // 32h + 8t + [0, 8) of MMA rows g and g + 8 (MMA k = 4t + i <-> byte
    // 8t + i, k = 16 + 4t + i <-> byte 8t + 4 + i), i.e. bytes of digit group
    // 2h + (t >> 1).  B column n is (local group n >> 2, digit n & 3), digit 3
    // unused: a lane's B registers are non-zero only when its column's group is
    // its own (n >> 2 == t >> 1).  The accumulator columns 2t, 2t + 1 of lane t
    // are digits (0, 1) for even t and (2, -) for odd t of group 2h + (t >> 1).

    // One-token units keep the B fragments of their digit slot in registers
    // while the digit group stays the same.
    uint2 bc[2][4];
    int bc_key = -1;

    __device__ __forceinline__ uint2 load_b(const uint8_t* __restrict__ dig, int slotdg, int h, int p,
                                            bool bActive) const {
        if (!bActive) return make_uint2(0u, 0u);
        return lds64(dig + (slotdg + 2 * h + (t >> 1)) * kDgStride + (g & 3) * 64 + p * 16 + (t & 1) * 8);
    }

    // Tile rt of the current compute item (its slot at sp): exact group
    // partial sums (a Horner chain per K half: D <<= 2 between code classes)
    // -> per-row fp32 sums of the item's chunk into the batch's red buffer.
    __device__ __forceinline__ void compute_tile(const unsigned char* sp, int rt, int tau, int c,
                                                 const uint8_t* __restrict__ dig,
                                                 const float2* __restrict__ fs) {
        const int4 tile = T.tiles[tau];
        const int ul = tile.x;
        const int nT = T.units[ul].z;
        const int nDG = W.Kd >> 6;
        const bool bActive = (g & 3) < 3 && (g >> 2) == (t >> 1);
        const int rA = rt * 16 + g, rB = rA + 8;
        uint2 wa[2], wb[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            wa[h] = lds64(sp + rA * 64 + swz(rA, h) + 8 * t);
            wb[h] = lds64(sp + rB * 64 + swz(rB, h) + 8 * t);
        }
        int slotdg[TMAX];
        int D[TMAX][2][4];
#pragma unroll
        for (int j = 0; j < TMAX; ++j) {
            const int slot = (j < nT) ? T.uslot[ul * TMAX + j] : 0;
            slotdg[j] = slot * nDG + 4 * c;
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int r = 0; r < 4; ++r) D[j][h][r] = 0;
        }
        if (TMAX == 1 && bc_key != slotdg[0]) {
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int p = 0; p < 4; ++p) bc[h][p] = load_b(dig, slotdg[0], h, p, bActive);
            bc_key = slotdg[0];
        }

#pragma unroll
        for (int p = 0; p < 4; ++p) {
            if (p) {
#pragma unroll
                for (int j = 0; j < TMAX; ++j)
#pragma unroll
                    for (int h = 0; h < 2; ++h)
#pragma unroll
                        for (int r = 0; r < 4; ++r) D[j][h][r] <<= 2;
            }
            const uint32_t mask = 0x03030303u << (2 * p);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t a0 = wa[h].x & mask, a1 = wb[h].x & mask;
                const uint32_t a2 = wa[h].y & mask, a3 = wb[h].y & mask;
#pragma unroll
                for (int j = 0; j < TMAX; ++j) {
                    if (j < nT) {
                        const uint2 bv = (TMAX == 1) ? bc[h][p] : load_b(dig, slotdg[j], h, p, bActive);
                        mma_u8s8(D[j][h], a0, a1, a2, a3, bv.x, bv.y);
                    }
                }
            }
        }

        // Even lanes finish row g, odd lanes row g + 8, of their group per K
        // half; then the two lanes of a row with groups {t>>1, 2 + (t>>1)}
        // add up across t ^ 2.
        const bool odd = t & 1;
        const int row = odd ? rB : rA;
        const uint16_t* s16 = reinterpret_cast<const uint16_t*>(sp + CODE_BYTES);
        const uint16_t* b16 = s16 + ROWS * SPC;
        float sc[2], bi[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int gi = (64 * (2 * h + (t >> 1))) / GS;
            sc[h] = Half<DT>::to_f(s16[row * SPC + gi]);
            bi[h] = Half<DT>::to_f(b16[row * SPC + gi]);
        }
        float* red_tile = red + (size_t)(tau - tfirst) * per_tile;
#pragma unroll
        for (int j = 0; j < TMAX; ++j) {
            if (j < nT) {
                float part[2];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int* cacc = D[j][h];
                    const int s1 = __shfl_xor_sync(0xffffffffu, odd ? cacc[0] : cacc[2], 1);
                    const int s2 = __shfl_xor_sync(0xffffffffu, cacc[3], 1);
                    const int d0 = odd ? s1 : cacc[0];
                    const int d1 = odd ? s2 : cacc[1];
                    const int d2 = odd ? cacc[2] : s1;
                    const float v = fmaf((float)d0, 65536.f, fmaf((float)d1, 256.f, (float)d2));
                    const float2 fsv = fs[slotdg[j] + 2 * h + (t >> 1)];
                    part[h] = fmaf(sc[h], v * fsv.x, bi[h] * fsv.y);
                }
                float pr = part[0] + part[1];
                pr += __shfl_xor_sync(0xffffffffu, pr, 2);
                if (t < 2) red_tile[(c * TMAX + j) * 16 + t * 8 + g] = pr;
            }
        }
    }

    // Main loop (every thread calls it, after the warp's first DIST items
    // were issued): at each item the warp issues the item DIST ahead in its
    // sequence through `ahead()` (which may belong to the next phase), waits
    // for its own current item and computes it.  Batches of `batch_tiles`
    // tiles (a multiple of RT; the host makes one batch cover the phase when
    // the red buffer allows) are each followed by the block-wide epilogue
    // between two block barriers; the loads in flight keep streaming across.
    template <class Out, class Ahead>
    __device__ void consume(const uint8_t* dig, const float2* fs, float* red_base, int batch_tiles,
                            Out& out, Ahead& ahead) {
        red = red_base;
#pragma unroll 1
        for (int tb0 = 0; tb0 < T.ntiles; tb0 += batch_tiles) {
            const int tb1 = min(T.ntiles, tb0 + batch_tiles);
            tfirst = tb0;
#pragma unroll 1
            while (ci.n < count && ci.grp * RT < tb1) {
                ahead();
                cp_async_wait<DIST>();
                __syncwarp();
                const unsigned char* sp = ring + ((q0 + ci.n) % STAGES) * SLOT;
#pragma unroll
                for (int rt = 0; rt < RT; ++rt) {
                    const int tau = ci.grp * RT + rt;
                    if (tau < T.ntiles) compute_tile(sp, rt, tau, ci.c, dig, fs);
                }
                __syncwarp();
                advance(ci);
            }
            bar_sync(kBarConsumers, kConsumerThreads);
            epilogue_tiles<TMAX, MODE>(tb0, tb1, red_base, nK, T.tiles, T.units, out);
            bar_sync(kBarConsumers, kConsumerThreads);
        }
    }
};

// Before the block exits, wait until every cp.async this thread issued has
// landed, so no copy is still writing into shared memory.
__device__ __forceinline__ void ring_quiesce() { cp_async_wait<0>(); }

}  // namespace momij
