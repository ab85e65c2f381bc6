// gemv.cu -- standalone 2-bit gather-GEMV kernel for the operator surface
// (momij_moe_gqmm2 / momij_moe_gqmm2_up_swiglu): reads the work plan written
// by plan_kernel, streams the planned rows with the engine of gemv_core.cuh
// and writes per-pair outputs (up||gate mode: the clamped SwiGLU of each row
// pair).  Each CTA owns a contiguous slice of the flattened (unit, row)
// space, so HBM work is balanced to one row.
#include "gemv_core.cuh"

namespace momij {

namespace {

template <int DT, int MODE, int TMAX>
struct StoreOut {  // one output of a finished tile -> out[pair, col]
    const int* upair;
    uint16_t* out;
    int out_cols;
    float clamp;
    __device__ void operator()(const int4& tile, int j, int r, float v, float v_gate) const {
        uint16_t* dst = out + (size_t)upair[tile.x * TMAX + j] * out_cols + tile.y + r;
        *dst = (MODE == kModeUpSwiglu) ? swiglu_staged<DT>(v, v_gate, clamp) : Half<DT>::from_f(v);
    }
};

}  // namespace

template <int DT, int GS, int MODE, int TMAX, int STAGES>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_kernel(const GemvArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ int s_ntiles, s_nvec, s_overflow;
    __shared__ __align__(8) uint64_t s_sbar;
    const int tid = threadIdx.x;
    constexpr int TR = GemvPhase<DT, GS, MODE, TMAX, STAGES>::TR;

    pdl_wait();
    const int U = a.plan[0];
    if (a.plan[1] != MOMIJ_OK || U <= 0) return;
    const int Ru = a.rows_per_unit;
    const long long Rtot = (long long)U * Ru;
    // slices of at most slice_rows rows (the shared-memory sizing bound),
    // at least one per CTA; CTA bx takes slices bx, bx + gridDim.x, ...
    const long long nsl = max((long long)gridDim.x, (Rtot + a.slice_rows - 1) / a.slice_rows);

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
    sb_init(&s_sbar);
    int sb_par = 0;  // phases of s_sbar completed by earlier slices
    bool ok = true;
    __syncthreads();

#pragma unroll 1
    for (long long sl = blockIdx.x; sl < nsl && ok; sl += gridDim.x) {
        const long long r0 = Rtot * sl / nsl, r1 = Rtot * (sl + 1) / nsl;
        if (r0 >= r1) continue;
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
        // and nothing more is written
        if (s_overflow) {
            if (tid == 0) atomicExch(a.plan + 2, MOMIJ_ERR_WORKSPACE);
            break;
        }

        PhaseTables tabs{s_tiles, s_units, s_uslot, s_ntiles};
        PhaseWeights wts{a.w, a.s, a.b, a.N, a.rows_per_unit, a.Kd};
        GemvPhase<DT, GS, MODE, TMAX, STAGES> ph(tabs, wts, s_stage, 0, a.nK,
                                                 reinterpret_cast<uint16_t*>(smem + a.off_sb), a.batch_tiles,
                                                 &s_sbar, true);
        ph.sb_par = sb_par;
        auto ahead = [&]() { ph.load_next(); };
        if (s_ntiles > 0) ph.issue_sb(0, min(s_ntiles, a.batch_tiles));
        ph.prefetch(ahead);
        // encode the activations while the first items land
        digitize<DT>(a.x, s_vecs, s_nvec, a.Kd, s_dig, s_fs, kConsumerThreads);
        bar_sync(kBarConsumers, kConsumerThreads);
        StoreOut<DT, MODE, TMAX> out{s_upair, a.out, a.out_cols, a.clamp};
        const bool done = ph.consume(s_dig, s_fs, s_red, true, out, ahead);
        ring_quiesce();
        sb_par = ph.sb_par;
        // this slice's tables, digits and ring are free again; a bounded wait
        // that gave up in any thread ends the loop in all of them
        ok = __syncthreads_and(done ? 1 : 0) != 0;
    }
    if (!ok && tid == 0) atomicExch(a.plan + 2, MOMIJ_ERR_TIMEOUT);
    pdl_launch_dependents();
}

// Explicit instantiations: dtype x group size x mode x TMAX x stages.
#define MOMIJ_INST(DT, GS, MODE, TM, ST) \
    template __global__ void gemv_kernel<DT, GS, MODE, TM, ST>(const GemvArgs);
#define MOMIJ_INST_ST(DT, GS, MODE, TM) \
    MOMIJ_INST(DT, GS, MODE, TM, 2)     \
    MOMIJ_INST(DT, GS, MODE, TM, 4)
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
