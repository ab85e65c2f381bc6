// gemv.cu -- 2-bit gather-GEMV for decode / verify batches (M*Ktop pairs).
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
//   * the N dimension of the MMA separates the four lane groups (= four
//     digit groups of 64 codes) and the digit planes: MMA #1 of a token holds
//     (lane group, d0|d1) in its 8 columns, MMA #2 holds d2 of a token pair,
//     so every lane ends with its own group's three partial sums and the fp32
//     epilogue applies that group's scale and bias:
//       acc += s * (65536*D0 + 256*D1 + D2) * 2^(E-27) + b * sum(x).
// Data movement: each CTA owns a contiguous slice of the flattened
// (unit, row) space, so HBM work is balanced to one row; every warp owns a
// 256-code chunk of K and streams, per lane, 16 B from each of two rows plus
// 8 B of scales/biases through a private cp.async ring of STAGES tiles.
#include "kernels.cuh"

namespace momij {

namespace {

// Balanced base-256 digits of |v| < 2^22: v = 65536*d[0] + 256*d[1] + d[2],
// d[1], d[2] in [-128, 127], d[0] in [-64, 64].
__device__ __forceinline__ void split3(int v, int (&d)[3]) {
    d[2] = ((v + 128) & 255) - 128;
    const int t = (v - d[2]) >> 8;
    d[1] = ((t + 128) & 255) - 128;
    d[0] = (t - d[1]) >> 8;
}

// Encode `nvec` vectors into digit planes (layout matched to the B fragment:
// per digit group, plane d at +64*d (d = 0, 1, 2), byte 8*s + 4*half + b
// holds element 16*(2*(s>>2) + half) + 4*b + (s&3) for MMA step s).  8 lanes
// per group.
template <int DT>
__device__ void digitize(const uint16_t* __restrict__ x, const int* __restrict__ vecs, int nvec,
                         int Kd, uint8_t* __restrict__ dig, float2* __restrict__ fs) {
    const int nDG = Kd >> 6;
    const int total = nvec * nDG * 8;
    const int lane = threadIdx.x & 31;
    for (int base = (threadIdx.x & ~31); base < total; base += blockDim.x) {
        const int idx = base + lane;
        const bool valid = idx < total;
        const int dgi = idx >> 3, sub = idx & 7;
        const int slot = dgi / nDG, dg = dgi - slot * nDG;
        float v[8];
        float mx = 0.f, sum = 0.f;
        if (valid) {
            const uint16_t* src = x + (size_t)vecs[slot] * Kd + dg * 64 + sub * 8;
            uint4 raw = *reinterpret_cast<const uint4*>(src);
            uint32_t r[4] = {raw.x, raw.y, raw.z, raw.w};
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
        const int w = sub >> 1;
#pragma unroll
        for (int tt = 0; tt < 4; ++tt) {
            int dA[3], dB[3];
            split3(__float2int_rn(v[tt] * scale), dA);
            split3(__float2int_rn(v[tt + 4] * scale), dB);
            const int j = 8 * (sub & 1) + tt;
            const int pos = 8 * (4 * (w >> 1) + (j & 3)) + 4 * (w & 1) + (j >> 2);
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

}  // namespace

template <int DT, int GS, int MODE, int TMAX, int STAGES>
__global__ void __launch_bounds__(512, 1) gemv_kernel(const GemvArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ int s_ntiles, s_nvec, s_overflow;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    constexpr int TR = (MODE == kModeUpSwiglu) ? 8 : 16;  // output rows per tile
    constexpr int SBN = 256 / GS;                          // scales per row per chunk

    pdl_wait();
    const int U = a.plan[0];
    if (a.plan[1] != MOMIJ_OK || U <= 0) return;
    const int Ru = a.rows_per_unit;
    const long long R = (long long)U * Ru;
    const long long r0 = R * blockIdx.x / gridDim.x, r1 = R * (blockIdx.x + 1) / gridDim.x;
    if (r0 >= r1) return;

    int4* s_tiles = reinterpret_cast<int4*>(smem + a.off_tiles);
    int4* s_units = reinterpret_cast<int4*>(smem + a.off_units);
    int* s_upair = reinterpret_cast<int*>(smem + a.off_upair);
    int* s_uslot = reinterpret_cast<int*>(smem + a.off_uslot);
    int* s_vecs = reinterpret_cast<int*>(smem + a.off_vecs);
    float2* s_fs = reinterpret_cast<float2*>(smem + a.off_fs);
    uint8_t* s_dig = reinterpret_cast<uint8_t*>(smem + a.off_dig);
    float* s_red = reinterpret_cast<float*>(smem + a.off_red);
    unsigned char* s_stage = smem + a.off_stage;

    const int32_t* units_g = a.plan + kPlanHeader;
    const int32_t* sorted_g = a.plan + kPlanHeader + 4 * a.P;

    if (tid == 0) {
        const int u_first = (int)(r0 / Ru), u_last = (int)((r1 - 1) / Ru);
        int nt = 0, nv = 0, over = (u_last - u_first + 1) > a.max_units;
        if (a.digit_all_tokens) {
            for (int m = 0; m < a.M; ++m) s_vecs[m] = m;
            nv = a.M;
        }
        for (int u = u_first; u <= u_last && !over; ++u) {
            const int ul = u - u_first;
            int4 un = make_int4(units_g[4 * u], units_g[4 * u + 1], units_g[4 * u + 2], 0);
            s_units[ul] = un;
            if (un.z > TMAX || (!a.digit_all_tokens && nv + un.z > a.max_vec)) {
                over = 1;
                break;
            }
            for (int j = 0; j < un.z; ++j) {
                int pr = sorted_g[un.y + j];
                int vec = a.x_per_pair ? pr : pr / a.Ktop;
                s_upair[ul * TMAX + j] = pr;
                if (a.digit_all_tokens) {
                    s_uslot[ul * TMAX + j] = vec;
                } else {
                    s_vecs[nv] = vec;
                    s_uslot[ul * TMAX + j] = nv++;
                }
            }
            long long lo = max(r0, (long long)u * Ru) - (long long)u * Ru;
            long long hi = min(r1, (long long)(u + 1) * Ru) - (long long)u * Ru;
            for (long long rs = lo; rs < hi && !over; rs += TR) {
                if (nt >= a.max_tiles) { over = 1; break; }
                s_tiles[nt++] = make_int4(ul, (int)rs, (int)min((long long)TR, hi - rs), 0);
            }
        }
        s_ntiles = nt;
        s_nvec = nv;
        s_overflow = over;
    }
    __syncthreads();
    // capacity guard: the host sizes shared memory from worst-case bounds, so
    // this never triggers for valid plans; if it does, the error word is set
    // and nothing is written
    if (s_overflow) {
        if (tid == 0) atomicExch(a.plan + 2, MOMIJ_ERR_WORKSPACE);
        return;
    }
    const int ntiles = s_ntiles;
    digitize<DT>(a.x, s_vecs, s_nvec, a.Kd, s_dig, s_fs);
    __syncthreads();

    const int nK = a.nK, ptile = a.ptile;
    const int c = warp % nK, tl = warp / nK;
    const int nDG = a.Kd >> 6;
    const int wordsPerRow = a.Kd >> 4;
    const int sbPerRow = a.Kd / GS;
    const int nrounds = (ntiles + ptile - 1) / ptile;
    unsigned char* my_stage = s_stage + (size_t)warp * STAGES * kStageBytes;
    const uint32_t my_stage_s = smem_u32(my_stage);

    auto issue = [&](int k) {
        const int tau = k * ptile + tl;
        if (k < nrounds && tau < ntiles) {
            const int4 tile = s_tiles[tau];
            const int e = s_units[tile.x].x;
            int rowA, rowB;
            bool vA, vB;
            if (MODE == kModeUpSwiglu) {
                rowA = tile.y + g;
                rowB = Ru + tile.y + g;
                vA = vB = g < tile.z;
            } else {
                rowA = tile.y + g;
                rowB = tile.y + 8 + g;
                vA = g < tile.z;
                vB = g + 8 < tile.z;
            }
            const size_t rbase = (size_t)e * a.N;
            const uint32_t st = my_stage_s + (k % STAGES) * kStageBytes;
            const uint32_t* wA = a.w + (rbase + rowA) * wordsPerRow + c * 16 + t * 4;
            const uint32_t* wB = a.w + (rbase + rowB) * wordsPerRow + c * 16 + t * 4;
            cp_async16(st + lane * 16, vA ? (const void*)wA : (const void*)a.w, vA);
            cp_async16(st + 512 + lane * 16, vB ? (const void*)wB : (const void*)a.w, vB);
            const int row = (t & 1) ? rowB : rowA;
            const bool v = (t & 1) ? vB : vA;
            const uint16_t* sbase = (t & 2) ? a.b : a.s;
            const uint16_t* src = sbase + (rbase + row) * sbPerRow + c * SBN;
            if (GS == 64) cp_async8(st + 1024 + lane * 8, v ? (const void*)src : (const void*)sbase, v);
            else cp_async4(st + 1024 + lane * 8, v ? (const void*)src : (const void*)sbase, v);
        }
        cp_async_commit();
    };

#pragma unroll 1
    for (int k = 0; k < STAGES - 1; ++k) issue(k);

    const bool bActive = (g >> 1) == t;
    const int dsel = g & 1;
    const int dg = 4 * c + t;
    const int tq = (GS == 64) ? t : (t >> 1);

#pragma unroll 1
    for (int kb = 0; kb < nrounds; kb += a.batch_rounds) {
        const int kend = min(nrounds, kb + a.batch_rounds);
#pragma unroll 1
        for (int k = kb; k < kend; ++k) {
            issue(k + STAGES - 1);
            cp_async_wait<STAGES - 1>();
            __syncwarp();
            const int tau = k * ptile + tl;
            if (tau < ntiles) {
                const int4 tile = s_tiles[tau];
                const int ul = tile.x;
                const int T = s_units[ul].z;
                const unsigned char* st = my_stage + (k % STAGES) * kStageBytes;
                const uint4 wa4 = lds128(st + lane * 16);
                const uint4 wb4 = lds128(st + 512 + lane * 16);
                const uint32_t wa[4] = {wa4.x, wa4.y, wa4.z, wa4.w};
                const uint32_t wb[4] = {wb4.x, wb4.y, wb4.z, wb4.w};
                const uint16_t* sb16 = reinterpret_cast<const uint16_t*>(st + 1024);
                const float sA = Half<DT>::to_f(sb16[(4 * g + 0) * 4 + tq]);
                const float sB = Half<DT>::to_f(sb16[(4 * g + 1) * 4 + tq]);
                const float bA = Half<DT>::to_f(sb16[(4 * g + 2) * 4 + tq]);
                const float bB = Half<DT>::to_f(sb16[(4 * g + 3) * 4 + tq]);

                // MMA #1 per token j: columns (lane group, digit 0|1).
                // MMA #2 per token pair i: columns (lane group, digit 2) of
                // token 2i (even) and 2i+1 (odd); the same 8 lanes carry B.
                constexpr int TP = (TMAX + 1) / 2;
                int slotdg[TMAX];
                int D[TMAX][4];
                int D2[TP][4];
#pragma unroll
                for (int j = 0; j < TMAX; ++j) {
                    const int slot = (j < T) ? s_uslot[ul * TMAX + j] : 0;
                    slotdg[j] = slot * nDG + dg;
                    D[j][0] = D[j][1] = D[j][2] = D[j][3] = 0;
                }
#pragma unroll
                for (int i = 0; i < TP; ++i) D2[i][0] = D2[i][1] = D2[i][2] = D2[i][3] = 0;
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    if (p) {
#pragma unroll
                        for (int j = 0; j < TMAX; ++j) {
                            D[j][0] <<= 2; D[j][1] <<= 2; D[j][2] <<= 2; D[j][3] <<= 2;
                        }
#pragma unroll
                        for (int i = 0; i < TP; ++i) {
                            D2[i][0] <<= 2; D2[i][1] <<= 2; D2[i][2] <<= 2; D2[i][3] <<= 2;
                        }
                    }
                    const uint32_t mask = 0x03030303u << (2 * p);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const uint32_t a0 = wa[2 * h] & mask, a1 = wb[2 * h] & mask;
                        const uint32_t a2 = wa[2 * h + 1] & mask, a3 = wb[2 * h + 1] & mask;
                        const int soff = 8 * (4 * h + p);
#pragma unroll
                        for (int j = 0; j < TMAX; ++j) {
                            if (j < T) {
                                uint2 bv = make_uint2(0u, 0u);
                                if (bActive)
                                    bv = lds64(s_dig + slotdg[j] * kDgStride + dsel * 64 + soff);
                                mma_u8s8(D[j], a0, a1, a2, a3, bv.x, bv.y);
                            }
                        }
#pragma unroll
                        for (int i = 0; i < TP; ++i) {
                            if (2 * i < T) {
                                const int jo = (2 * i + 1 < TMAX) ? 2 * i + 1 : 2 * i;
                                const int jj = 2 * i + dsel;
                                uint2 bv = make_uint2(0u, 0u);
                                if (bActive && jj < T)
                                    bv = lds64(s_dig + (dsel ? slotdg[jo] : slotdg[2 * i]) * kDgStride +
                                               128 + soff);
                                mma_u8s8(D2[i], a0, a1, a2, a3, bv.x, bv.y);
                            }
                        }
                    }
                }
                float* red = s_red + (size_t)((k - kb) * ptile + tl) * nK * TMAX * 16;
#pragma unroll
                for (int j = 0; j < TMAX; ++j) {
                    if (j < T) {
                        const float2 fsj = s_fs[slotdg[j]];
                        const int odd = j & 1;
                        const float va = fmaf((float)D[j][0], 65536.f,
                                              fmaf((float)D[j][1], 256.f, (float)D2[j >> 1][odd]));
                        const float vb = fmaf((float)D[j][2], 65536.f,
                                              fmaf((float)D[j][3], 256.f, (float)D2[j >> 1][2 + odd]));
                        float ra = fmaf(sA, va * fsj.x, bA * fsj.y);
                        float rb = fmaf(sB, vb * fsj.x, bB * fsj.y);
                        ra += __shfl_xor_sync(0xffffffffu, ra, 1);
                        rb += __shfl_xor_sync(0xffffffffu, rb, 1);
                        ra += __shfl_xor_sync(0xffffffffu, ra, 2);
                        rb += __shfl_xor_sync(0xffffffffu, rb, 2);
                        if (t == 0) {
                            red[(c * TMAX + j) * 16 + g] = ra;
                            red[(c * TMAX + j) * 16 + 8 + g] = rb;
                        }
                    }
                }
            }
            __syncwarp();
        }
        __syncthreads();
        // cross-chunk reduction and output for the tiles of this batch
        const int tfirst = kb * ptile, tlast = min(ntiles, kend * ptile);
        const int items = (tlast - tfirst) * TMAX * TR;
        for (int it = tid; it < items; it += blockDim.x) {
            const int tau = tfirst + it / (TMAX * TR);
            const int j = (it / TR) % TMAX, r = it % TR;
            const int4 tile = s_tiles[tau];
            if (j >= s_units[tile.x].z || r >= tile.z) continue;
            const float* red = s_red + (size_t)(tau - tfirst) * nK * TMAX * 16;
            const int pr = s_upair[tile.x * TMAX + j];
            if (MODE == kModeUpSwiglu) {
                float up = 0.f, gate = 0.f;
                for (int cc = 0; cc < nK; ++cc) {
                    up += red[(cc * TMAX + j) * 16 + r];
                    gate += red[(cc * TMAX + j) * 16 + 8 + r];
                }
                // the up||gate gather output is an activation-dtype array first
                float u = Half<DT>::to_f(Half<DT>::from_f(up));
                float gt = Half<DT>::to_f(Half<DT>::from_f(gate));
                gt = fminf(gt, a.clamp);
                u = fminf(fmaxf(u, -a.clamp), a.clamp);
                const float silu = gt / (1.f + expf(-gt));
                a.out[(size_t)pr * a.out_cols + tile.y + r] = Half<DT>::from_f(silu * u);
            } else {
                float acc = 0.f;
                for (int cc = 0; cc < nK; ++cc) acc += red[(cc * TMAX + j) * 16 + r];
                a.out[(size_t)pr * a.out_cols + tile.y + r] = Half<DT>::from_f(acc);
            }
        }
        __syncthreads();
    }
    cp_async_wait<0>();
    pdl_launch_dependents();
}

// Explicit instantiations: dtype x group size x mode x TMAX x stages.
#define MOMIJ_INST(DT, GS, MODE, TM, ST) \
    template __global__ void gemv_kernel<DT, GS, MODE, TM, ST>(const GemvArgs);
#define MOMIJ_INST_ST(DT, GS, MODE, TM) \
    MOMIJ_INST(DT, GS, MODE, TM, 4)     \
    MOMIJ_INST(DT, GS, MODE, TM, 8)
#define MOMIJ_INST_TM(DT, GS, MODE) \
    MOMIJ_INST_ST(DT, GS, MODE, 1)  \
    MOMIJ_INST_ST(DT, GS, MODE, 2)  \
    MOMIJ_INST_ST(DT, GS, MODE, 4)  \
    MOMIJ_INST_ST(DT, GS, MODE, 8)
#define MOMIJ_INST_MODE(DT, GS)          \
    MOMIJ_INST_TM(DT, GS, kModeRows)     \
    MOMIJ_INST_TM(DT, GS, kModeUpSwiglu)
MOMIJ_INST_MODE(MOMIJ_DTYPE_BF16, 64)
MOMIJ_INST_MODE(MOMIJ_DTYPE_BF16, 128)
MOMIJ_INST_MODE(MOMIJ_DTYPE_F16, 64)
MOMIJ_INST_MODE(MOMIJ_DTYPE_F16, 128)

}  // namespace momij
