// prefill.cu -- grouped GEMM of the 2-bit experts on the tcgen05 tensor cores
// for prefill / large verify batches (tokens per expert large enough that the
// weights are re-used across tokens).
//
// Per tile (one block of <= 128 sorted pairs of one expert x 128 weight rows):
//   D[row, token] = sum_k dequant(W[e])[row, k] * X[token, k]
// with D (fp32) in tensor memory.  Each k-block of 64 elements is staged in
// shared memory as K-major 128-byte-swizzled tiles: the 128 weight rows
// dequantised (w = s*q + b in fp32) and split into two activation-dtype tiles
// A_hi = round(w) and A_lo = round(w - A_hi), so A_hi + A_lo carries w to
// ~2^-17 (a single 16-bit rounding of w would cost ~2^-9 per weight, several
// times the tolerance after two projections); B = the block's token rows.
// The four values a (row, group) can take are tabulated once per k-block and
// codes become packed halves by byte permutes, four codes of one bit
// position ("class") at a time, so the tiles hold each 16-element block of K
// in class order (element 4j + p at 4p + j) and the activations are reordered
// alike (class_order_kernel; the up GEMM writes act in that order).
// Pipeline per CTA: a ring of load stages (token rows, codes, scale and bias
// words) filled by cp.async four k-blocks ahead, two slots of dequantised A;
// one thread issues eight tcgen05.mma.kind::f16 (M=128, N=tokens rounded up
// to 16, K=16; hi then lo into the same fp32 accumulator) per k-block and
// commits them to the slot's mbarrier while the other threads dequantise the
// next k-block.  The epilogue reads TMEM (tcgen05.ld) and writes per-pair
// rows: the staged clamped SwiGLU of up||gate (tile = 64 up rows + the
// matching 64 gate rows), or the down projection.
//
// Reference semantics: MLX gatherQuantizedMM for M*Ktop rows (MapleMoE.swift:
// 65-75) with sortedIndices false; the grouping by expert is this build's
// (the reference reuses its GEMV for prefill, SeedlessDecodeEngine.swift:
// 516-545).  Outputs are per (token, slot) pair like gqmm2, so the same
// combine kernel applies.
#include "common.cuh"
#include "prefill.cuh"

namespace momij {

namespace {

// Shared memory: a ring of load stages (per k-block: the token rows B in the
// MMA layout), a ring of weight chunks (codes, scales and biases of four
// k-blocks), both filled by cp.async, and two slots of dequantised weights
// (A hi, A lo) that alternate between the dequantising threads and the
// tensor core.
constexpr int kStageA = 128 * 128;           // 128 weight rows x 64 elements x 2 B (one of hi / lo)
constexpr int kSlotA = 2 * kStageA;          // A hi + A lo
constexpr int kASlots = 2;
constexpr int kStageB = kBlockTokens * 128;  // tokens x 64 elements x 2 B
constexpr int kLoadBytes = kStageB;          // a load stage holds one k-block's token rows
constexpr int kLoadStages = 5;
// Weight chunks (4 k-blocks): the 128 rows' codes (64 B each), then their
// scales and biases (8 B per row: the chunk's groups); a ring of four.
constexpr int kChunkKB = 4;
constexpr int kChunkCodes = 0;
constexpr int kChunkScales = 128 * 64;
constexpr int kChunkBiases = kChunkScales + 128 * 8;
constexpr int kChunkBytes = kChunkBiases + 128 * 8;  // 10 KB
constexpr int kChunks = 4;
constexpr int kRowThreads = 128;   // loader threads copying token rows (8 x 16 B each per k-block)
constexpr int kChunkThreads = 32;  // loader threads copying weight chunks
static_assert(kRowThreads + kChunkThreads == 32 * kLoadWarps, "the loader warps form the two streams");
constexpr int kTmemCols = kBlockTokens;      // fp32 accumulator columns
static_assert(kLoadBytes % 1024 == 0 && kSlotA % 1024 == 0, "stages keep the 1024-B swizzle alignment");
static_assert(grouped_smem_bytes() ==
                  (size_t)kASlots * kSlotA + (size_t)kLoadStages * kLoadBytes + (size_t)kChunks * kChunkBytes + 1024,
              "host and kernel agree on the shared-memory size");
constexpr int kMmaWaitLimit = 1 << 22;

// tcgen05 shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row
// groups 1024 B apart (leading byte offset unused for swizzled K-major).
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor, kind::f16: fp32 D, A and B bf16 (or f16), both
// K-major, M = 128, N = n.
template <int DT>
__device__ __forceinline__ uint32_t idesc_f16(int n) {
    const uint32_t ab = (DT == MOMIJ_DTYPE_BF16) ? 1u : 0u;
    return (1u << 4) | (ab << 7) | (ab << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}
// Byte offset of element (r, k), k < 64, in a K-major tile with 128-byte
// rows and 128-byte swizzle (16-byte chunk c of row r at c ^ (r & 7)).
__device__ __forceinline__ uint32_t sw128(int r, int k) {
    return (r >> 3) * 1024 + (r & 7) * 128 + ((((k * 2) >> 4) ^ (r & 7)) << 4) + ((k * 2) & 15);
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Two fp32 values -> two activation-dtype values packed (first in the low half).
template <int DT>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    uint32_t r;
    if (DT == MOMIJ_DTYPE_BF16)
        asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    else
        asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}
// Column of element c in class order: within each block of 16 elements,
// element 4j + p moves to 4p + j (the order the dequantised weight tiles use).
// Whether v lies within `ulps` fp32 ulps of a rounding midpoint of the
// 16-bit type (normal range of the type).
template <int DT>
__device__ __forceinline__ bool near_half_midpoint(float v, int ulps) {
    const uint32_t u = __float_as_uint(v);
    if (DT == MOMIJ_DTYPE_BF16) return abs((int)(u & 0xffffu) - 0x8000) < ulps;
    return abs((int)(u & 0x1fffu) - 0x1000) < ulps;
}

// s + e = a + b exactly (Knuth's two-sum), e accumulated.
__device__ __forceinline__ void two_sum_acc(float& s, float& e, float b) {
    const float t = s + b;
    const float bv = t - s;
    e += (s - (t - bv)) + (b - bv);
    s = t;
}

// float64 -> 16-bit value, rounded once (ties to even), as the oracle does.
template <int DT>
__device__ __forceinline__ uint16_t half_from_f64(double d) {
    constexpr int kMant = (DT == MOMIJ_DTYPE_BF16) ? 7 : 10;
    constexpr int kEmin = (DT == MOMIJ_DTYPE_BF16) ? -126 : -14;
    if (isnan(d)) return Half<DT>::from_f(__int_as_float(0x7fc00000));
    const double m = fabs(d);
    if (m == 0.0) return Half<DT>::from_f((float)d);
    const int e = max(ilogb(m), kEmin);
    const double q = ldexp(1.0, e - kMant);
    const double v = copysign(rint(m / q) * q, d);  // representable in the 16-bit type (or overflowing to inf)
    return Half<DT>::from_f((float)v);              // exact conversion
}

__device__ __forceinline__ int class_order16(int c) {
    return (c & ~15) | ((c & 3) << 2) | ((c >> 2) & 3);
}
// Named barrier `id` over `count` threads that also ANDs a predicate.
__device__ __forceinline__ bool bar_and(int id, int count, bool v) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, %2, %3, p;\n"
        " selp.u32 %0, 1, 0, q;\n}\n"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(id), "r"(count)
        : "memory");
    return r != 0;
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
        "[%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
          "=r"(v[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

}  // namespace

__global__ void block_list_kernel(const int32_t* offsets, int E, int32_t* blocks, const int32_t* status) {
    const int lane = threadIdx.x & 31;
    pdl_wait();  // offsets and status are written by permute_kernel
    if (threadIdx.x >= 32) return;
    if (status && *status != MOMIJ_OK) {
        if (lane == 0) blocks[0] = 0;
        return;
    }
    int carry = 0;
    for (int base = 0; base < E; base += 32) {
        const int e = base + lane;
        const int lo = e < E ? offsets[e] : 0, hi = e < E ? offsets[e + 1] : 0;
        const int nb = (hi - lo + kBlockTokens - 1) / kBlockTokens;
        int incl = nb;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        const int first = carry + incl - nb;
        for (int j = 0; j < nb; ++j) {
            int32_t* ent = blocks + kBlockHeader + 4 * (first + j);
            ent[0] = e;
            ent[1] = lo + j * kBlockTokens;
            ent[2] = min(kBlockTokens, hi - lo - j * kBlockTokens);
            ent[3] = 0;
        }
        carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) blocks[0] = carry;
    pdl_launch_dependents();
}

// y = x with every row's 16-element blocks in class order (class_order16);
// one thread per block of 16 halves.
__global__ void class_order_kernel(const uint4* __restrict__ x, uint4* __restrict__ y, long long blocks) {
    pdl_wait();
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < blocks;
         i += (long long)gridDim.x * blockDim.x) {
        const uint4 u = x[2 * i], v = x[2 * i + 1];
        const uint32_t w[8] = {u.x, u.y, u.z, u.w, v.x, v.y, v.z, v.w};
        uint32_t o[8];
#pragma unroll
        for (int p = 0; p < 4; ++p)
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
                // output halves 4p + 2jj, 4p + 2jj + 1 <- elements 4 (2jj) + p, 4 (2jj + 1) + p
                const int e0 = 8 * jj + p, e1 = 8 * jj + 4 + p;
                const uint32_t h0 = (w[e0 >> 1] >> (16 * (e0 & 1))) & 0xffffu;
                const uint32_t h1 = (w[e1 >> 1] >> (16 * (e1 & 1))) & 0xffffu;
                o[2 * p + jj] = h0 | (h1 << 16);
            }
        y[2 * i] = make_uint4(o[0], o[1], o[2], o[3]);
        y[2 * i + 1] = make_uint4(o[4], o[5], o[6], o[7]);
    }
    pdl_launch_dependents();
}

// Warp roles: warps [0, 16) dequantise (thread (ra, wq): 16 codes of row ra
// per k-block) and run the epilogue; warps [16, 20) copy the token rows of
// each k-block, warp 20 the weight chunks (codes, scales, biases of four
// k-blocks); the last warp's
// lane 0 issues the MMAs.  Hand-offs per k-block g (stage g % kLoadStages,
// A slot g % kASlots) are mbarriers:
//   load_full[st]   loaders -> dequant + MMA   (128 arrivals, after each
//                   loader's copies landed and a generic->async proxy fence)
//   a_full[as]      dequant -> MMA             (16 warp arrivals, after the fence)
//   a_empty[as]     MMA commit -> dequant      (slot reusable)
//   load_empty[st]  MMA commit -> loaders (stage reusable)
//   chunk_full[cs]  loaders -> dequant (the 4 k-blocks' codes, scales, biases)
//   chunk_empty[cs] 16 dequant warps -> loaders
//   done            MMA commit -> epilogue      (per tile)
//   tmem_free       16 epilogue warps -> MMA    (accumulator reusable)
// Every wait is bounded; a timeout sets the kernel's error word and ends the
// waiting role, whose partners then time out too.
template <int DT, int GS, int MODE>
__global__ void __launch_bounds__(kGroupedThreads, 1) grouped_gemm_kernel(const GroupedArgs a) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint32_t s_tmem;
    __shared__ __align__(8) uint64_t bar_full[kLoadStages], bar_lempty[kLoadStages];
    __shared__ __align__(8) uint64_t bar_afull[kASlots], bar_aempty[kASlots];
    __shared__ __align__(8) uint64_t bar_cfull[kChunks], bar_cempty[kChunks];
    __shared__ __align__(8) uint64_t bar_done, bar_tmem, bar_fin;
    __shared__ int s_timeout;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    pdl_wait();
    if (a.status[1] != MOMIJ_OK || a.status[2] != MOMIJ_OK) return;
    const int nblocks = a.blocks[0];
    if (nblocks < 0 || nblocks > a.P / kBlockTokens + a.E + 1) {  // cannot come from block_list_kernel
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicExch(a.status + 2, MOMIJ_ERR_WORKSPACE);
        return;
    }
    const int nrb = (MODE == kModeUpSwiglu) ? a.Ru / 64 : a.N / 128;
    const int ntiles = nblocks * nrb;
    if ((int)blockIdx.x >= ntiles) return;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid == 0) {
        for (int s = 0; s < kLoadStages; ++s) {
            mbar_init(&bar_full[s], kRowThreads);
            mbar_init(&bar_lempty[s], 1);
        }
        for (int s = 0; s < kChunks; ++s) {
            mbar_init(&bar_cfull[s], kChunkThreads);
            mbar_init(&bar_cempty[s], kDequantWarps);
        }
        for (int s = 0; s < kASlots; ++s) {
            mbar_init(&bar_afull[s], kDequantWarps);
            mbar_init(&bar_aempty[s], 1);
        }
        mbar_init(&bar_done, 1);
        mbar_init(&bar_tmem, kDequantWarps);
        mbar_init(&bar_fin, 1);
        mbar_fence_init();
        s_timeout = 0;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;

    const int KB = a.Kd / 64;
    const int nsb = a.Kd / GS;
    const int4* blist = reinterpret_cast<const int4*>(a.blocks + kBlockHeader);
    unsigned char* const ring = smem + kASlots * kSlotA;
    unsigned char* const chunks = ring + kLoadStages * kLoadBytes;
    // bounded wait; once any role of the CTA gave up, every later wait fails
    // at once, so all roles wind down quickly
    volatile int* timed_out = &s_timeout;
    auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
        for (int it = 0; it < kMmaWaitLimit; ++it) {
            if (mbar_try_wait(bar, parity)) return true;
            if ((it & 1023) == 1023 && *timed_out) return false;
        }
        *timed_out = 1;
        return false;
    };
    // a malformed entry (it cannot come from block_list_kernel) is an error, not an access
    auto tile_ok = [&](const int4& blk) {
        return !(blk.x < 0 || blk.x >= a.E || blk.y < 0 || blk.z < 1 || blk.z > kBlockTokens ||
                 blk.y + blk.z > a.P);
    };
    // weight row of tile row r (0..127) of row block rb
    auto weight_row = [&](int e, int rb, int r) -> size_t {
        int gr;
        if (MODE == kModeUpSwiglu) gr = (r < 64) ? rb * 64 + r : a.Ru + rb * 64 + (r - 64);
        else gr = rb * 128 + r;
        return (size_t)e * a.N + gr;
    };

    if (warp == kDequantWarps + kLoadWarps) {
        // ---- MMA issue (one thread) ------------------------------------------
        if (lane == 0) {
            int g = 0, tcount = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
                const int4 blk = blist[t / nrb];
                if (!tile_ok(blk)) continue;
                const int nmma = (blk.z + 15) & ~15;
                if (tcount > 0) ok = wait(&bar_tmem, (tcount - 1) & 1);  // the epilogue has read TMEM
                tc_fence_after();
                const uint32_t idesc = idesc_f16<DT>(nmma);
                for (int kb = 0; kb < KB && ok; ++kb, ++g) {
                    const int st = g % kLoadStages, as = g % kASlots;
                    ok = wait(&bar_afull[as], (g / kASlots) & 1) && wait(&bar_full[st], (g / kLoadStages) & 1);
                    if (!ok) break;
                    // the token rows were written by other threads' cp.async
                    // (generic proxy): order them before the tensor core reads
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    tc_fence_after();
                    unsigned char* sA = smem + as * kSlotA;
                    unsigned char* sL = sA + kStageA;
                    unsigned char* sB = ring + st * kLoadBytes;
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint64_t bd = sdesc_sw128(smem_u32(sB) + kk * 32);
#pragma unroll
                        for (int part = 0; part < 2; ++part) {  // D += A_hi B, then D += A_lo B
                            const uint64_t ad = sdesc_sw128(smem_u32(part ? sL : sA) + kk * 32);
                            const uint32_t accum = (kb > 0 || kk > 0 || part > 0) ? 1u : 0u;
                            asm volatile(
                                "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                                " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
                                "l"(ad), "l"(bd), "r"(idesc), "r"(accum));
                        }
                    }
                    asm volatile(
                        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                            smem_u32(&bar_aempty[as])));
                    asm volatile(
                        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                            smem_u32(&bar_lempty[st])));
                }
                if (!ok) break;
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                    smem_u32(&bar_done)));
                ++tcount;
            }
            // every MMA issued has completed before TMEM is released
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                smem_u32(&bar_fin)));
            wait(&bar_fin, 0);
        }
    } else if (warp >= kDequantWarps) {
        // ---- loaders ------------------------------------------------------------
        // Two streams on separate threads, so neither waits for the other's
        // copies: warps 16-19 copy token rows (stage per k-block), warp 20
        // weight chunks.  No loader thread waits on its own copies:
        // every stage's / chunk's barrier gets a cp.async-tracked arrival from
        // each thread of its stream (it fires once that thread's earlier
        // copies have landed).
        const int pl = tid - 32 * kDequantWarps;  // 0..159
        const bool rows_stream = pl < kRowThreads;
        const int ps = rows_stream ? pl : pl - kRowThreads;
        int g = 0, gc = 0;  // k-blocks and chunks issued
        bool ok = true;
        for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
            const int bi = t / nrb, rb = t - bi * nrb;
            const int4 blk = blist[bi];
            if (!tile_ok(blk)) continue;
            const int e = blk.x, start = blk.y, cnt = blk.z;
            if (rows_stream) {
                // thread ps copies 16-B part ps & 7 of tokens 16 j + (ps >> 3),
                // so a warp's copy covers four whole 128-B row segments; the
                // source rows and the swizzled destinations are set per tile
                const int nmma = (cnt + 15) & ~15, part = ps & 7;
                const uint16_t* src[8];
                uint32_t dst[8];
                int nv = 0;  // copies of this thread: tokens < nmma (the first nv of j)
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int n = 16 * j + (ps >> 3);
                    int xr = 0;
                    if (n < cnt) {
                        const int p = min(max(a.pairs[start + n], 0), a.P - 1);
                        xr = a.x_per_pair ? p : p / a.Ktop;
                    }
                    src[j] = a.x + (size_t)xr * a.Kd + part * 8;
                    dst[j] = sw128(n, part * 8) | (n < cnt ? 0u : 0x80000000u);  // top bit: zero-fill
                    nv += n < nmma;
                }
                for (int kb = 0; kb < KB && ok; ++kb, ++g) {
                    const int st = g % kLoadStages;
                    if (g >= kLoadStages && !(ok = wait(&bar_lempty[st], (g / kLoadStages - 1) & 1))) break;
                    const uint32_t sp = smem_u32(ring + st * kLoadBytes);
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        if (j < nv)
                            cp_async16(sp + (dst[j] & 0x7fffffffu), src[j] + kb * 64, !(dst[j] >> 31));
                    mbar_arrive_cp_async(&bar_full[st]);
                }
            } else {
                // chunk ci: k-blocks 4 ci .. 4 ci + 3; codes 64 B per row (four
                // threads per row), then the rows' scale and bias words
                const int nch = KB / kChunkKB;
                for (int ci = 0; ci < nch && ok; ++ci, ++gc) {
                    const int cs = gc % kChunks;
                    if (gc >= kChunks && !(ok = wait(&bar_cempty[cs], (gc / kChunks - 1) & 1))) break;
                    unsigned char* cp = chunks + cs * kChunkBytes;
                    const int kb = ci * kChunkKB;
#pragma unroll 4
                    for (int j = 0; j < 16; ++j) {
                        const int i = ps + 32 * j, r = i >> 2, pt = i & 3;
                        cp_async16(smem_u32(cp + kChunkCodes + r * 64 + pt * 16),
                                   a.w + weight_row(e, rb, r) * (size_t)(a.Kd / 16) + kb * 4 + pt * 4, true);
                    }
#pragma unroll 4
                    for (int h = 0; h < 4; ++h) {
                        const int r = ps + 32 * h;
                        const size_t gw = weight_row(e, rb, r) * nsb + (size_t)kb * 64 / GS;  // first group of the chunk
                        if (GS == 64) {
                            cp_async8(smem_u32(cp + kChunkScales + r * 8), a.s + gw, true);
                            cp_async8(smem_u32(cp + kChunkBiases + r * 8), a.b + gw, true);
                        } else {
                            cp_async4(smem_u32(cp + kChunkScales + r * 8), a.s + gw, true);
                            cp_async4(smem_u32(cp + kChunkBiases + r * 8), a.b + gw, true);
                        }
                    }
                    mbar_arrive_cp_async(&bar_cfull[cs]);
                }
            }
        }
        cp_async_commit();
        cp_async_wait<0>();  // no copy in flight when the CTA ends
    } else {
        // ---- dequantise + epilogue ------------------------------------------------
        const int ra = tid >> 2, wq = tid & 3;  // row ra, codes 16 wq + [0, 16) of each k-block
        int g = 0, gc = 0, tcount = 0;  // k-blocks, chunks consumed, tiles
        bool ok = true;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
            const int bi = t / nrb, rb = t - bi * nrb;
            const int4 blk = blist[bi];
            if (!tile_ok(blk)) {
                if (tid == 0) atomicExch(a.status + 2, MOMIJ_ERR_WORKSPACE);
                continue;
            }
            const int start = blk.y, cnt = blk.z;
            // no early exit inside the tile: the 16 warps meet at named
            // barriers below, so a failed wait only skips the work
            for (int kb = 0; kb < KB; ++kb, ++g) {
                const int as = g % kASlots, cs = gc % kChunks, kq = kb % kChunkKB;
                if (ok && g >= kASlots) ok = wait(&bar_aempty[as], (g / kASlots - 1) & 1);
                if (ok && kq == 0) ok = wait(&bar_cfull[cs], (gc / kChunks) & 1);
                if (kq == kChunkKB - 1) ++gc;
                if (!ok) continue;
                const unsigned char* cp = chunks + cs * kChunkBytes;
                unsigned char* sA = smem + as * kSlotA;  // hi
                unsigned char* sL = sA + kStageA;        // lo
                const uint32_t cw = *reinterpret_cast<const uint32_t*>(cp + kChunkCodes + ra * 64 + kq * 16 + wq * 4);
                const int gi = (kb * 64) / GS - ((kb - kq) * 64) / GS;  // the group within the chunk
                const float sc = Half<DT>::to_f(*reinterpret_cast<const uint16_t*>(cp + kChunkScales + ra * 8 + gi * 2));
                const float bi2 = Half<DT>::to_f(*reinterpret_cast<const uint16_t*>(cp + kChunkBiases + ra * 8 + gi * 2));
                // The row's group takes four weight values w_q = s*q + b: their
                // hi and lo halves as byte tables (low bytes of entries 0..3,
                // high bytes), so a byte permute turns two codes into two
                // packed halves.
                const float w0 = bi2, w1 = fmaf(sc, 1.f, bi2), w2 = fmaf(sc, 2.f, bi2), w3 = fmaf(sc, 3.f, bi2);
                const uint32_t h01 = pack2<DT>(w0, w1), h23 = pack2<DT>(w2, w3);
                const uint32_t l01 = pack2<DT>(w0 - Half<DT>::to_f((uint16_t)(h01 & 0xffffu)),
                                               w1 - Half<DT>::to_f((uint16_t)(h01 >> 16)));
                const uint32_t l23 = pack2<DT>(w2 - Half<DT>::to_f((uint16_t)(h23 & 0xffffu)),
                                               w3 - Half<DT>::to_f((uint16_t)(h23 >> 16)));
                const uint32_t thA = __byte_perm(h01, h23, 0x6420), thB = __byte_perm(h01, h23, 0x7531);
                const uint32_t tlA = __byte_perm(l01, l23, 0x6420), tlB = __byte_perm(l01, l23, 0x7531);
                // class order within the word's 16 codes: column 4p + j holds
                // code 4j + p (the activations are permuted alike)
                uint32_t hi[8], lo[8];
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    const uint32_t m = (cw >> (2 * p)) & 0x03030303u;  // byte j: code 4j + p
                    const uint32_t sel = m | (m << 4) | 0x40404040u;   // nibbles (q, q + 4) per code
                    const uint32_t sel2 = sel >> 16;
                    hi[2 * p] = __byte_perm(thA, thB, sel);
                    hi[2 * p + 1] = __byte_perm(thA, thB, sel2);
                    lo[2 * p] = __byte_perm(tlA, tlB, sel);
                    lo[2 * p + 1] = __byte_perm(tlA, tlB, sel2);
                }
                const int k0 = wq * 16;
                const uint32_t o0 = sw128(ra, k0), o1 = sw128(ra, k0 + 8);
                *reinterpret_cast<uint4*>(sA + o0) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                *reinterpret_cast<uint4*>(sA + o1) = make_uint4(hi[4], hi[5], hi[6], hi[7]);
                *reinterpret_cast<uint4*>(sL + o0) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                *reinterpret_cast<uint4*>(sL + o1) = make_uint4(lo[4], lo[5], lo[6], lo[7]);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor core
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&bar_afull[as]);
                    if (kq == kChunkKB - 1) mbar_arrive(&bar_cempty[cs]);  // the chunk's codes are read
                }
            }
            if (ok) ok = wait(&bar_done, tcount & 1);
            ok = bar_and(1, 32 * kDequantWarps, ok);  // the same decision in every dequantising thread
            if (!ok) break;
            tc_fence_after();

            // ---- epilogue: warp w reads TMEM lanes 32 (w & 3) + lane, columns
            // 32 (w >> 2) + [0, 32); the A slots (all MMAs done) stage the gate sums
            const int r = 32 * (warp & 3) + lane;  // A row = TMEM lane
            const int c0 = 32 * (warp >> 2);
            const uint32_t taddr = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + c0;
            if (MODE == kModeUpSwiglu) {
                float* sG = reinterpret_cast<float*>(smem);  // [token][64] gate sums
                if (r >= 64) {
#pragma unroll 1
                    for (int cc = 0; cc < 32; cc += 16) {
                        uint32_t v[16];
                        tmem_ld16(taddr + cc, v);
#pragma unroll
                        for (int j = 0; j < 16; ++j) sG[(c0 + cc + j) * 64 + (r - 64)] = __uint_as_float(v[j]);
                    }
                }
                bar_sync(1, 32 * kDequantWarps);
                if (r < 64) {
#pragma unroll 1
                    for (int cc = 0; cc < 32; cc += 16) {
                        uint32_t v[16];
                        tmem_ld16(taddr + cc, v);
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const int n = c0 + cc + j;
                            if (n < cnt) {  // act columns in class order for the down GEMM
                                const int p = min(max(__ldg(a.pairs + start + n), 0), a.P - 1);
                                const float uf = __uint_as_float(v[j]), gf = sG[n * 64 + r];
                                const int which = a.fix ? (near_half_midpoint<DT>(uf, a.fix_ulps) ? 1 : 0) |
                                                              (near_half_midpoint<DT>(gf, a.fix_ulps) ? 2 : 0)
                                                        : 0;
                                if (which) {
                                    const int q = atomicAdd(a.fix, 1);
                                    if (q < a.fix_cap) {
                                        reinterpret_cast<int4*>(a.fix + 4)[q] = make_int4(
                                            p, rb * 64 + r, which, __float_as_int(which == 1 ? gf : uf));
                                        continue;  // act_fixup_kernel writes it
                                    }
                                }
                                a.out[(size_t)p * a.Ru + class_order16(rb * 64 + r)] =
                                    swiglu_staged<DT>(uf, gf, a.clamp);
                            }
                        }
                    }
                }
            } else {
#pragma unroll 1
                for (int cc = 0; cc < 32; cc += 16) {
                    uint32_t v[16];
                    tmem_ld16(taddr + cc, v);
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int n = c0 + cc + j;
                        if (n < cnt) {
                            const int p = min(max(__ldg(a.pairs + start + n), 0), a.P - 1);
                            a.out[(size_t)p * a.N + rb * 128 + r] = Half<DT>::from_f(__uint_as_float(v[j]));
                        }
                    }
                }
            }
            tc_fence_before();
            // TMEM read and the gate sums consumed before the next tile's MMAs
            // and dequantisation reuse them
            bar_sync(1, 32 * kDequantWarps);
            if (lane == 0) mbar_arrive(&bar_tmem);
            ++tcount;
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    if (tid == 0 && s_timeout) atomicExch(a.status + 2, MOMIJ_ERR_TIMEOUT);
    pdl_launch_dependents();
}

template <int DT, int GS>
__global__ void __launch_bounds__(256) act_fixup_kernel(const FixupArgs a) {
    pdl_wait();  // the up||gate GEMM (the list, act) is complete
    pdl_launch_dependents();
    if (__ldcg(a.status + 1) != 0 || __ldcg(a.status + 2) != 0) return;  // routing failed or a wait gave up
    const int n = min(__ldcg(a.fix), a.fix_cap);
    const int lane = threadIdx.x & 31, wpb = blockDim.x >> 5;
    constexpr int kWpg = GS / 16;  // code words per scale group
    const int ng = a.Kd / GS;
    for (int it = blockIdx.x * wpb + (threadIdx.x >> 5); it < n; it += gridDim.x * wpb) {
        const int4 ent = __ldcg(reinterpret_cast<const int4*>(a.fix + 4) + it);
        const int p = ent.x, i = ent.y, which = ent.z, e = a.inds[p];
        const uint16_t* xr = a.x + (size_t)(p / a.Ktop) * a.Kd;
        float sums[2] = {__int_as_float(ent.w), __int_as_float(ent.w)};  // [up, gate]
#pragma unroll 1
        for (int h = 0; h < 2; ++h) {
            if (!((which >> h) & 1)) continue;
            const size_t row = (size_t)e * 2 * a.I + (size_t)h * a.I + i;
            const uint32_t* wr = a.w + row * (a.Kd / 16);
            const uint16_t* sr = a.s + row * ng;
            const uint16_t* br = a.b + row * ng;
            double acc = 0.0;
            for (int g = lane; g < ng; g += 32) {  // lane: whole scale groups
                float sq = 0.f, eq = 0.f, sx = 0.f, ex = 0.f;
#pragma unroll
                for (int wq = 0; wq < kWpg; ++wq) {
                    const uint32_t c = __ldg(wr + g * kWpg + wq);
                    const uint4* xv = reinterpret_cast<const uint4*>(xr + (size_t)g * GS + wq * 16);
                    const uint4 x0 = __ldg(xv), x1 = __ldg(xv + 1);
                    const uint32_t xw[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const float xf = Half<DT>::to_f((uint16_t)(xw[j >> 1] >> (16 * (j & 1))));
                        const uint32_t q = (c >> (2 * j)) & 3u;
                        const float qx = ((q & 1u) ? xf : 0.f) + ((q & 2u) ? xf + xf : 0.f);  // exact
                        two_sum_acc(sq, eq, qx);
                        two_sum_acc(sx, ex, xf);
                    }
                }
                const double sc = Half<DT>::to_f(__ldg(sr + g)), bi = Half<DT>::to_f(__ldg(br + g));
                acc = fma(sc, (double)sq + (double)eq, fma(bi, (double)sx + (double)ex, acc));
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
            sums[h] = Half<DT>::to_f(half_from_f64<DT>(acc));
        }
        if (lane == 0) a.act[(size_t)p * a.I + class_order16(i)] = swiglu_staged<DT>(sums[0], sums[1], a.clamp);
    }
}

#define MOMIJ_GROUPED_INST(DT, GS)                                               \
    template __global__ void grouped_gemm_kernel<DT, GS, kModeUpSwiglu>(const GroupedArgs); \
    template __global__ void grouped_gemm_kernel<DT, GS, kModeRows>(const GroupedArgs); \
    template __global__ void act_fixup_kernel<DT, GS>(const FixupArgs);
MOMIJ_GROUPED_INST(MOMIJ_DTYPE_BF16, 64)
MOMIJ_GROUPED_INST(MOMIJ_DTYPE_BF16, 128)
MOMIJ_GROUPED_INST(MOMIJ_DTYPE_F16, 64)
MOMIJ_GROUPED_INST(MOMIJ_DTYPE_F16, 128)

}  // namespace momij
