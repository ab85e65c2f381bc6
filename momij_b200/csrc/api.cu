// api.cu -- the extern "C" entry points of libmomij_moe.so (include/momij_moe.h).
//
// Host-side responsibilities: argument and shape validation (mirroring the
// reference's SeedlessError.unsupportedShape guards, SeedlessMetal.swift:
// 336-338, widened from K % 512 to K % 256), workspace carving, launch
// configuration of the gather-GEMV kernels, and programmatic dependent launch
// so that consecutive kernels of one MoE call overlap their prologues.
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "kernels.cuh"

using namespace momij;

namespace {

constexpr int kVersion = 100;

bool pdl_enabled() {
    static const bool on = [] {
        const char* v = std::getenv("MOMIJ_PDL");
        return !(v && v[0] == '0');
    }();
    return on;
}

int current_device_sm_count() {
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
        cache[dev] = n;
    }
    return cache[dev];
}

int max_dyn_smem() {
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    if (cache[dev] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        cache[dev] = n;
    }
    return cache[dev];
}

template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                   Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

int cuda_status(cudaError_t e) { return e == cudaSuccess ? MOMIJ_OK : MOMIJ_ERR_CUDA; }

// ---- per-kernel event timing (momij_profile_*) -----------------------------
// When enabled, every launch below is bracketed by a pair of CUDA events on
// its stream (recorded into a CUDA graph when the stream is capturing), the
// analogue of the reference's MOMIJ_PROFILE_MOE phase timers
// (MapleSeedlessMoE.swift:81-107) and GPU timestamps (SeedlessMetal.swift:
// 1050-1069).  Pairs are pooled and reused after momij_profile_collect.
struct ProfRec {
    cudaEvent_t a, b;
    int kid;
    bool used;
};
std::mutex g_prof_mu;
bool g_prof_on = false;
std::vector<ProfRec> g_prof;

// Inside a stream capture a plain cudaEventRecord only marks a dependency;
// the External flag makes it a real event-record node of the graph.
void record_event(cudaEvent_t ev, cudaStream_t st) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(st, &cs);
    if (cs == cudaStreamCaptureStatusActive)
        cudaEventRecordWithFlags(ev, st, cudaEventRecordExternal);
    else
        cudaEventRecord(ev, st);
}

int prof_begin(int kid, cudaStream_t st) {
    if (!g_prof_on) return -1;
    std::lock_guard<std::mutex> lk(g_prof_mu);
    size_t i = 0;
    while (i < g_prof.size() && g_prof[i].used) ++i;
    if (i == g_prof.size()) {
        if (g_prof.size() >= 65536) return -1;
        ProfRec r{};
        if (cudaEventCreate(&r.a) != cudaSuccess || cudaEventCreate(&r.b) != cudaSuccess) return -1;
        g_prof.push_back(r);
    }
    g_prof[i].used = true;
    g_prof[i].kid = kid;
    record_event(g_prof[i].a, st);
    return (int)i;
}
void prof_end(int slot, cudaStream_t st) {
    if (slot < 0) return;
    record_event(g_prof[slot].b, st);
}

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int pick_tmax(int per_unit_bound) {
    if (per_unit_bound <= 1) return 1;
    if (per_unit_bound <= 2) return 2;
    if (per_unit_bound <= 4) return 4;
    return 8;
}

// ---- workspace layout ------------------------------------------------------
struct Workspace {
    int32_t* plan;
    uint16_t* act;
    uint16_t* down;
    int32_t* inds;
    float* scores;
    size_t bytes;
};

size_t plan_bytes(int P) { return align_up(sizeof(int32_t) * (kPlanHeader + 5 * (size_t)P), 256); }

Workspace carve(void* ws, int M, int Ktop, int H, int I) {
    const size_t P = (size_t)M * Ktop;
    Workspace w{};
    unsigned char* p = static_cast<unsigned char*>(ws);
    size_t off = 0;
    w.plan = reinterpret_cast<int32_t*>(p + off);
    off += plan_bytes((int)P);
    w.act = reinterpret_cast<uint16_t*>(p + off);
    off += align_up(P * I * 2, 256);
    w.down = reinterpret_cast<uint16_t*>(p + off);
    off += align_up(P * H * 2, 256);
    w.inds = reinterpret_cast<int32_t*>(p + off);
    off += align_up(P * 4, 256);
    w.scores = reinterpret_cast<float*>(p + off);
    off += align_up(P * 4, 256);
    w.bytes = off;
    return w;
}

// ---- gather-GEMV dispatch --------------------------------------------------
using GemvFn = void (*)(const GemvArgs);

template <int DT, int GS, int MODE>
GemvFn pick_tm_st(int tmax, int stages) {
    const bool s8 = stages == 8;
    switch (tmax) {
        case 1: return s8 ? gemv_kernel<DT, GS, MODE, 1, 8> : gemv_kernel<DT, GS, MODE, 1, 4>;
        case 2: return s8 ? gemv_kernel<DT, GS, MODE, 2, 8> : gemv_kernel<DT, GS, MODE, 2, 4>;
        case 4: return s8 ? gemv_kernel<DT, GS, MODE, 4, 8> : gemv_kernel<DT, GS, MODE, 4, 4>;
        default: return s8 ? gemv_kernel<DT, GS, MODE, 8, 8> : gemv_kernel<DT, GS, MODE, 8, 4>;
    }
}
template <int DT, int GS>
GemvFn pick_mode(int mode, int tmax, int stages) {
    return mode == kModeUpSwiglu ? pick_tm_st<DT, GS, kModeUpSwiglu>(tmax, stages)
                                 : pick_tm_st<DT, GS, kModeRows>(tmax, stages);
}
GemvFn pick_gemv(int dtype, int gs, int mode, int tmax, int stages) {
    if (dtype == MOMIJ_DTYPE_BF16)
        return gs == 64 ? pick_mode<MOMIJ_DTYPE_BF16, 64>(mode, tmax, stages)
                        : pick_mode<MOMIJ_DTYPE_BF16, 128>(mode, tmax, stages);
    return gs == 64 ? pick_mode<MOMIJ_DTYPE_F16, 64>(mode, tmax, stages)
                    : pick_mode<MOMIJ_DTYPE_F16, 128>(mode, tmax, stages);
}

struct GemvLaunch {
    GemvArgs a;
    int grid, threads, stages;
    size_t smem;
};

// Worst-case shared-memory sizing from (P, shapes); returns false if the
// configuration cannot fit on the device.
bool configure_gemv(GemvLaunch& L, int mode, int tmax) {
    GemvArgs& a = L.a;
    const int nK = a.Kd / kChunk;
    int ptile = nK >= 16 ? 1 : 16 / nK;
    if (ptile > 4) ptile = 4;
    a.nK = nK;
    a.ptile = ptile;
    const int warps = nK * ptile;
    L.threads = 32 * warps;
    const int TR = mode == kModeUpSwiglu ? 8 : 16;
    const long long Ru = a.rows_per_unit;
    const long long Rmax = (long long)a.P * Ru;
    const int sms = current_device_sm_count();
    if (sms <= 0) return false;
    long long G = (Rmax + TR - 1) / TR;
    if (G > sms) G = sms;
    if (G < 1) G = 1;
    L.grid = (int)G;
    const long long rows_cta = (Rmax + G - 1) / G;
    a.max_units = (int)std::min<long long>(a.P, rows_cta / Ru + 2);
    a.max_tiles = (int)(rows_cta / TR + a.max_units + 1);
    a.max_vec = a.digit_all_tokens ? a.M : std::min(a.P, a.max_units * tmax);
    const int nDG = a.Kd / kDigitGroup;
    const int nrounds = (a.max_tiles + ptile - 1) / ptile;

    const size_t limit = (size_t)max_dyn_smem();
    for (int stages : {8, 4}) {
        for (int rounds = std::min(nrounds, 32); rounds >= 1; rounds = rounds > 1 ? rounds / 2 : 0) {
            size_t off = 0;
            a.off_tiles = (int)off; off += 16 * (size_t)a.max_tiles;
            a.off_units = (int)off; off += 16 * (size_t)a.max_units;
            a.off_upair = (int)off; off += 4 * (size_t)a.max_units * tmax;
            a.off_uslot = (int)off; off += 4 * (size_t)a.max_units * tmax;
            a.off_vecs = (int)off; off += 4 * (size_t)a.max_vec;
            off = align_up(off, 16);
            a.off_fs = (int)off; off += 8 * (size_t)a.max_vec * nDG;
            off = align_up(off, 16);
            a.off_dig = (int)off; off += (size_t)kDgStride * a.max_vec * nDG;
            off = align_up(off, 16);
            a.off_red = (int)off; off += 4 * (size_t)rounds * ptile * nK * tmax * 16;
            off = align_up(off, 128);
            a.off_stage = (int)off; off += (size_t)warps * stages * kStageBytes;
            if (off <= limit) {
                a.batch_rounds = rounds;
                L.stages = stages;
                L.smem = off;
                return true;
            }
            if (rounds == 1) break;
        }
    }
    return false;
}

int run_gemv(GemvLaunch& L, int mode, int tmax, int dtype, int gs, cudaStream_t st) {
    if (!configure_gemv(L, mode, tmax)) return MOMIJ_ERR_UNSUPPORTED_SHAPE;
    GemvFn fn = pick_gemv(dtype, gs, mode, tmax, L.stages);
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.smem);
    if (e != cudaSuccess) return MOMIJ_ERR_CUDA;
    const int slot = prof_begin(mode == kModeUpSwiglu ? MOMIJ_KERNEL_UP : MOMIJ_KERNEL_ROWS, st);
    const int rc = cuda_status(launch(fn, dim3(L.grid), dim3(L.threads), L.smem, st, L.a));
    prof_end(slot, st);
    return rc;
}

bool shape_ok(int Kdim, int gs) {
    return (gs == 64 || gs == 128) && Kdim >= kChunk && Kdim % kChunk == 0 && Kdim <= 16 * kChunk;
}

GemvLaunch make_launch(const void* x, int x_per_pair, const uint32_t* w, const void* s,
                       const void* b, int32_t* plan, void* out, int Kd, int N, int E, int M,
                       int Ktop, int rows_per_unit, int out_cols, float clamp) {
    GemvLaunch L{};
    GemvArgs& a = L.a;
    a.x = static_cast<const uint16_t*>(x);
    a.x_per_pair = x_per_pair;
    a.digit_all_tokens = (!x_per_pair && M <= 8) ? 1 : 0;
    a.w = w;
    a.s = static_cast<const uint16_t*>(s);
    a.b = static_cast<const uint16_t*>(b);
    a.plan = plan;
    a.out = static_cast<uint16_t*>(out);
    a.Kd = Kd;
    a.N = N;
    a.E = E;
    a.M = M;
    a.Ktop = Ktop;
    a.P = M * Ktop;
    a.rows_per_unit = rows_per_unit;
    a.out_cols = out_cols;
    a.clamp = clamp;
    return L;
}

// The bound on pairs sharing one expert that the plan/kernels must handle.
int tmax_for(int M, int Ktop, int lhs_per_expert) {
    (void)lhs_per_expert;
    // A token picks an expert at most once under the router; gqmm2 callers
    // may repeat an index inside a token, which the plan splits into more
    // units when it exceeds the bound.
    return pick_tmax(M < 1 ? 1 : (M > 8 ? 8 : M));
    (void)Ktop;
}

int launch_plan(const int32_t* inds, int P, int E, int tmax, int32_t* plan, cudaStream_t st) {
    const int slot = prof_begin(MOMIJ_KERNEL_PLAN, st);
    const int rc =
        cuda_status(launch(plan_kernel, dim3(1), dim3(1024), 0, st, inds, P, E, tmax, plan));
    prof_end(slot, st);
    return rc;
}

template <int DT>
int launch_combine(const uint16_t* down, const float* scores, uint16_t* y, int M, int Ktop, int H,
                   int resid, const int32_t* plan, cudaStream_t st) {
    const long long n = (long long)M * H;
    int blocks = (int)std::min<long long>((n + 255) / 256, 4096);
    if (blocks < 1) blocks = 1;
    const int slot = prof_begin(MOMIJ_KERNEL_COMBINE, st);
    int rc;
    if (resid)
        rc = cuda_status(launch(combine_kernel<DT, 1>, dim3(blocks), dim3(256), 0, st, down, scores,
                                y, M, Ktop, H, plan));
    else
        rc = cuda_status(launch(combine_kernel<DT, 0>, dim3(blocks), dim3(256), 0, st, down, scores,
                                y, M, Ktop, H, plan));
    prof_end(slot, st);
    return rc;
}

int launch_combine_dt(int dtype, const uint16_t* down, const float* scores, uint16_t* y, int M,
                      int Ktop, int H, int resid, const int32_t* plan, cudaStream_t st) {
    return dtype == MOMIJ_DTYPE_BF16
               ? launch_combine<MOMIJ_DTYPE_BF16>(down, scores, y, M, Ktop, H, resid, plan, st)
               : launch_combine<MOMIJ_DTYPE_F16>(down, scores, y, M, Ktop, H, resid, plan, st);
}

int check_device() {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return MOMIJ_ERR_NO_DEVICE;
    }
    return MOMIJ_OK;
}

// Shared body of expert_ffn and forward once inds/scores/plan are enqueued.
int ffn_after_plan(const void* x, const uint32_t* w_ug, const void* s_ug, const void* b_ug,
                   const uint32_t* w_dn, const void* s_dn, const void* b_dn, const float* scores,
                   void* y, void* resid_h, int M, int H, int I, int E, int Ktop, int gs,
                   float clamp, int dtype, int tmax, const Workspace& ws, cudaStream_t st) {
    GemvLaunch up = make_launch(x, 0, w_ug, s_ug, b_ug, ws.plan, ws.act, H, 2 * I, E, M, Ktop, I,
                                I, clamp);
    int rc = run_gemv(up, kModeUpSwiglu, tmax, dtype, gs, st);
    if (rc) return rc;
    GemvLaunch dn = make_launch(ws.act, 1, w_dn, s_dn, b_dn, ws.plan, ws.down, I, H, E, M, Ktop,
                                H, H, clamp);
    rc = run_gemv(dn, kModeRows, tmax, dtype, gs, st);
    if (rc) return rc;
    return launch_combine_dt(dtype, ws.down, scores, static_cast<uint16_t*>(resid_h ? resid_h : y),
                             M, Ktop, H, resid_h != nullptr, ws.plan, st);
}

}  // namespace

extern "C" {

const char* momij_status_string(int status) {
    switch (status) {
        case MOMIJ_OK: return "ok";
        case MOMIJ_ERR_UNSUPPORTED_SHAPE: return "unsupported shape";
        case MOMIJ_ERR_NOT_READY: return "not ready";
        case MOMIJ_ERR_NO_DEVICE: return "no CUDA device";
        case MOMIJ_ERR_INVALID_ARGUMENT: return "invalid argument";
        case MOMIJ_ERR_EXPERT_INDEX: return "expert index out of range";
        case MOMIJ_ERR_WORKSPACE: return "workspace too small";
        case MOMIJ_ERR_CUDA: return "CUDA runtime error";
        case MOMIJ_ERR_NCCL: return "NCCL error";
        case MOMIJ_ERR_TIMEOUT: return "device-side wait timed out";
        case MOMIJ_ERR_STOPPED: return "stopped";
        default: return "unknown status";
    }
}

int momij_version(void) { return kVersion; }

int momij_profile_enable(int on) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    g_prof_on = on != 0;
    return MOMIJ_OK;
}

int momij_profile_read(int kernel_id, double* total_ms, int* launches) {
    if (!total_ms || !launches) return MOMIJ_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> lk(g_prof_mu);
    double tot = 0.0;
    int n = 0;
    for (auto& r : g_prof) {
        if (!r.used || r.kid != kernel_id) continue;
        if (cudaEventSynchronize(r.b) != cudaSuccess) return MOMIJ_ERR_CUDA;
        float ms = 0.f;
        if (cudaEventElapsedTime(&ms, r.a, r.b) != cudaSuccess) return MOMIJ_ERR_CUDA;
        tot += ms;
        ++n;
    }
    *total_ms = tot;
    *launches = n;
    return MOMIJ_OK;
}

int momij_profile_reset(void) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    for (auto& r : g_prof) r.used = false;
    return MOMIJ_OK;
}

int momij_device_sm_count(void) { return current_device_sm_count(); }

int momij_moe_synchronize(momij_stream_t stream, const void* workspace) {
    if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess) return MOMIJ_ERR_CUDA;
    if (!workspace) return MOMIJ_OK;
    int32_t hdr[3] = {0, 0, 0};
    if (cudaMemcpy(hdr, workspace, sizeof(hdr), cudaMemcpyDeviceToHost) != cudaSuccess)
        return MOMIJ_ERR_CUDA;
    if (hdr[1] != MOMIJ_OK) return hdr[1];
    return hdr[2];
}

int momij_moe_route(const float* logits, int M, int E, int K, int32_t* inds, float* scores,
                    momij_stream_t stream) {
    if (int rc = check_device()) return rc;
    if (!logits || !inds || !scores || M < 0) return MOMIJ_ERR_INVALID_ARGUMENT;
    if (E < 1 || E > 1024 || K < 1 || K > 32 || K > E) return MOMIJ_ERR_UNSUPPORTED_SHAPE;
    if (M == 0) return MOMIJ_OK;
    const int warps = 8;
    int blocks = (M + warps - 1) / warps;
    return cuda_status(launch(route_kernel, dim3(blocks), dim3(32 * warps), 0,
                              static_cast<cudaStream_t>(stream), logits, M, E, K, inds, scores));
}

int momij_moe_permute(const int32_t* inds, const float* scores, int M, int K, int E,
                      int32_t* offsets, int32_t* pair, float* weight, momij_stream_t stream) {
    if (int rc = check_device()) return rc;
    if (!inds || !scores || !offsets || !pair || !weight || M < 0 || K < 1 || E < 1)
        return MOMIJ_ERR_INVALID_ARGUMENT;
    if (E > 8192) return MOMIJ_ERR_UNSUPPORTED_SHAPE;
    const size_t smem = sizeof(int) * (E + 1);
    return cuda_status(launch(permute_kernel, dim3(1), dim3(1024), smem,
                              static_cast<cudaStream_t>(stream), inds, scores, M * K, E, offsets,
                              pair, weight, static_cast<int32_t*>(nullptr)));
}

size_t momij_moe_workspace_size(int M, int Ktop, int H, int I) {
    if (M < 0 || Ktop < 1 || H < 0 || I < 0) return 0;
    return carve(nullptr, M, Ktop, H, I).bytes;
}

int momij_moe_gqmm2(const void* x, const uint32_t* w, const void* scales, const void* biases,
                    const int32_t* inds, void* out, int M, int Ktop, int Kdim, int N, int E, int gs,
                    int lhs_per_expert, int dtype, void* workspace, size_t workspace_bytes,
                    momij_stream_t stream) {
    if (int rc = check_device()) return rc;
    if (M < 0 || Ktop < 1 || E < 1 || N < 1 || (dtype != MOMIJ_DTYPE_BF16 && dtype != MOMIJ_DTYPE_F16))
        return MOMIJ_ERR_INVALID_ARGUMENT;
    if (!shape_ok(Kdim, gs)) return MOMIJ_ERR_UNSUPPORTED_SHAPE;
    if (M == 0) return MOMIJ_OK;
    if (!x || !w || !scales || !biases || !inds || !out || !workspace)
        return MOMIJ_ERR_INVALID_ARGUMENT;
    if (!shape_ok(Kdim, gs) || (long long)M * Ktop > MOMIJ_MAX_PAIRS)
        return MOMIJ_ERR_UNSUPPORTED_SHAPE;
    if (!aligned(x, 16) || !aligned(w, 16) || !aligned(scales, 8) || !aligned(biases, 8))
        return MOMIJ_ERR_INVALID_ARGUMENT;
    if (M == 0) return MOMIJ_OK;
    if (workspace_bytes < plan_bytes(M * Ktop)) return MOMIJ_ERR_WORKSPACE;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int32_t* plan = static_cast<int32_t*>(workspace);
    const int tmax = tmax_for(M, Ktop, lhs_per_expert);
    int rc = launch_plan(inds, M * Ktop, E, tmax, plan, st);
    if (rc) return rc;
    GemvLaunch L = make_launch(x, lhs_per_expert ? 1 : 0, w, scales, biases, plan, out, Kdim, N, E,
                               M, Ktop, N, N, 0.f);
    return run_gemv(L, kModeRows, tmax, dtype, gs, st);
}

int momij_moe_gqmm2_up_swiglu(const void* x, const uint32_t* w, const void* scales,
                              const void* biases, const int32_t* inds, void* act, int M, int Ktop,
                              int H, int I, int E, int gs, float clamp, int dtype, void* workspace,
                              size_t workspace_bytes, momij_stream_t stream) {
    if (int rc = check_device()) return rc;
    if (M < 0 || Ktop < 1 || E < 1 || I < 1 || (dtype != MOMIJ_DTYPE_BF16 && dtype != MOMIJ_DTYPE_F16))
        return MOMIJ_ERR_INVALID_ARGUMENT;
    if (!shape_ok(H, gs)) return MOMIJ_ERR_UNSUPPORTED_SHAPE;
    if (M == 0) return MOMIJ_OK;
    if (!x || !w || !scales || !biases || !inds || !act || !workspace)
        return MOMIJ_ERR_INVALID_ARGUMENT;
    if (!shape_ok(H, gs) || (long long)M * Ktop > MOMIJ_MAX_PAIRS)
        return MOMIJ_ERR_UNSUPPORTED_SHAPE;
    if (!aligned(x, 16) || !aligned(w, 16) || !aligned(scales, 8) || !aligned(biases, 8))
        return MOMIJ_ERR_INVALID_ARGUMENT;
    if (M == 0) return MOMIJ_OK;
    if (workspace_bytes < plan_bytes(M * Ktop)) return MOMIJ_ERR_WORKSPACE;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int32_t* plan = static_cast<int32_t*>(workspace);
    const int tmax = tmax_for(M, Ktop, 0);
    int rc = launch_plan(inds, M * Ktop, E, tmax, plan, st);
    if (rc) return rc;
    GemvLaunch L = make_launch(x, 0, w, scales, biases, plan, act, H, 2 * I, E, M, Ktop, I, I, clamp);
    return run_gemv(L, kModeUpSwiglu, tmax, dtype, gs, st);
}

int momij_moe_clamped_swiglu(const void* ug, void* act, int rows, int I, float clamp, int dtype,
                             momij_stream_t stream) {
    if (int rc = check_device()) return rc;
    if (!ug || !act || rows < 0 || I < 0) return MOMIJ_ERR_INVALID_ARGUMENT;
    const long long n = (long long)rows * I;
    if (n == 0) return MOMIJ_OK;
    int blocks = (int)std::min<long long>((n + 255) / 256, 4096);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    auto u = static_cast<const uint16_t*>(ug);
    auto o = static_cast<uint16_t*>(act);
    if (dtype == MOMIJ_DTYPE_BF16)
        return cuda_status(launch(swiglu_kernel<MOMIJ_DTYPE_BF16>, dim3(blocks), dim3(256), 0, st, u,
                                  o, rows, I, clamp));
    if (dtype == MOMIJ_DTYPE_F16)
        return cuda_status(launch(swiglu_kernel<MOMIJ_DTYPE_F16>, dim3(blocks), dim3(256), 0, st, u,
                                  o, rows, I, clamp));
    return MOMIJ_ERR_INVALID_ARGUMENT;
}

int momij_moe_score_reduce(const void* down, const float* scores, void* y, int M, int Ktop, int H,
                           int dtype, momij_stream_t stream) {
    if (int rc = check_device()) return rc;
    if (!down || !scores || !y || M < 0 || Ktop < 1 || H < 0 ||
        (dtype != MOMIJ_DTYPE_BF16 && dtype != MOMIJ_DTYPE_F16))
        return MOMIJ_ERR_INVALID_ARGUMENT;
    if ((long long)M * H == 0) return MOMIJ_OK;
    return launch_combine_dt(dtype, static_cast<const uint16_t*>(down), scores,
                             static_cast<uint16_t*>(y), M, Ktop, H, 0, nullptr,
                             static_cast<cudaStream_t>(stream));
}

int momij_moe_score_resid(const void* down, const float* scores, void* h, int M, int Ktop, int H,
                          int dtype, momij_stream_t stream) {
    if (int rc = check_device()) return rc;
    if (!down || !scores || !h || M < 0 || Ktop < 1 || H < 0 ||
        (dtype != MOMIJ_DTYPE_BF16 && dtype != MOMIJ_DTYPE_F16))
        return MOMIJ_ERR_INVALID_ARGUMENT;
    if ((long long)M * H == 0) return MOMIJ_OK;
    return launch_combine_dt(dtype, static_cast<const uint16_t*>(down), scores,
                             static_cast<uint16_t*>(h), M, Ktop, H, 1, nullptr,
                             static_cast<cudaStream_t>(stream));
}

static int validate_ffn(const void* x, const uint32_t* w_ug, const void* s_ug, const void* b_ug,
                        const uint32_t* w_dn, const void* s_dn, const void* b_dn, void* y,
                        void* resid_h, int M, int H, int I, int E, int Ktop, int gs, int dtype,
                        void* workspace, size_t workspace_bytes) {
    if (!x || !w_ug || !s_ug || !b_ug || !w_dn || !s_dn || !b_dn || (!y && !resid_h) ||
        !workspace || M < 0 || Ktop < 1 || E < 1 ||
        (dtype != MOMIJ_DTYPE_BF16 && dtype != MOMIJ_DTYPE_F16))
        return MOMIJ_ERR_INVALID_ARGUMENT;
    if (!shape_ok(H, gs) || !shape_ok(I, gs) || (long long)M * Ktop > MOMIJ_MAX_PAIRS)
        return MOMIJ_ERR_UNSUPPORTED_SHAPE;
    if (!aligned(x, 16) || !aligned(w_ug, 16) || !aligned(w_dn, 16) || !aligned(s_ug, 8) ||
        !aligned(b_ug, 8) || !aligned(s_dn, 8) || !aligned(b_dn, 8) || !aligned(workspace, 256))
        return MOMIJ_ERR_INVALID_ARGUMENT;
    if (workspace_bytes < momij_moe_workspace_size(M, Ktop, H, I)) return MOMIJ_ERR_WORKSPACE;
    return MOMIJ_OK;
}

int momij_moe_expert_ffn(const void* x, const uint32_t* w_ug, const void* s_ug, const void* b_ug,
                         const uint32_t* w_dn, const void* s_dn, const void* b_dn,
                         const int32_t* inds, const float* scores, void* y, void* resid_h, int M,
                         int H, int I, int E, int Ktop, int gs, float clamp, int dtype,
                         void* workspace, size_t workspace_bytes, momij_stream_t stream) {
    if (int rc = check_device()) return rc;
    if (M == 0 && Ktop >= 1) return MOMIJ_OK;
    if (!inds || !scores) return MOMIJ_ERR_INVALID_ARGUMENT;
    if (int rc = validate_ffn(x, w_ug, s_ug, b_ug, w_dn, s_dn, b_dn, y, resid_h, M, H, I, E, Ktop,
                              gs, dtype, workspace, workspace_bytes))
        return rc;
    if (M == 0) return MOMIJ_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    Workspace ws = carve(workspace, M, Ktop, H, I);
    const int tmax = tmax_for(M, Ktop, 0);
    int rc = launch_plan(inds, M * Ktop, E, tmax, ws.plan, st);
    if (rc) return rc;
    return ffn_after_plan(x, w_ug, s_ug, b_ug, w_dn, s_dn, b_dn, scores, y, resid_h, M, H, I, E,
                          Ktop, gs, clamp, dtype, tmax, ws, st);
}

int momij_moe_forward(const float* logits, const void* x, const uint32_t* w_ug, const void* s_ug,
                      const void* b_ug, const uint32_t* w_dn, const void* s_dn, const void* b_dn,
                      int32_t* inds, float* scores, void* y, void* resid_h, int M, int H, int I,
                      int E, int Ktop, int gs, float clamp, int dtype, void* workspace,
                      size_t workspace_bytes, momij_stream_t stream) {
    if (int rc = check_device()) return rc;
    if (M == 0 && Ktop >= 1) return MOMIJ_OK;
    if (!logits) return MOMIJ_ERR_INVALID_ARGUMENT;
    if (int rc = validate_ffn(x, w_ug, s_ug, b_ug, w_dn, s_dn, b_dn, y, resid_h, M, H, I, E, Ktop,
                              gs, dtype, workspace, workspace_bytes))
        return rc;
    if (E > 1024 || Ktop > 32 || Ktop > E) return MOMIJ_ERR_UNSUPPORTED_SHAPE;
    if (M == 0) return MOMIJ_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    Workspace ws = carve(workspace, M, Ktop, H, I);
    int32_t* ind_out = inds ? inds : ws.inds;
    float* sc_out = scores ? scores : ws.scores;
    const int tmax = tmax_for(M, Ktop, 0);
    const int slot = prof_begin(MOMIJ_KERNEL_PLAN, st);
    int rc = cuda_status(launch(route_plan_kernel, dim3(1), dim3(1024), 0, st, logits, M, E, Ktop,
                                tmax, ind_out, sc_out, ws.plan));
    prof_end(slot, st);
    if (rc) return rc;
    return ffn_after_plan(x, w_ug, s_ug, b_ug, w_dn, s_dn, b_dn, sc_out, y, resid_h, M, H, I, E,
                          Ktop, gs, clamp, dtype, tmax, ws, st);
}

int momij_synth_fill(void* dst, int64_t n, int kind, float a, float c, uint64_t seed,
                     uint64_t stream_id, int64_t start, int dtype, momij_stream_t stream) {
    if (int rc = check_device()) return rc;
    if (!dst || n < 0 || kind < 0 || kind > 3) return MOMIJ_ERR_INVALID_ARGUMENT;
    if (n == 0) return MOMIJ_OK;
    int blocks = (int)std::min<int64_t>((n + 255) / 256, 148 * 32);
    synth_fill_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(dst, n, kind, a, c,
                                                                             seed, stream_id, start,
                                                                             dtype);
    return cuda_status(cudaGetLastError());
}

}  // extern "C"
