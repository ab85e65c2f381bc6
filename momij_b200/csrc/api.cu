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
#include <atomic>
#include <cudaTypedefs.h>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "kernels.cuh"
#include "gemv_core.cuh"
#include "decode.cuh"
#include "layer.cuh"
#include "token.cuh"
#include "prefill.cuh"

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

// Dynamic shared memory a kernel of this library may request: the device's
// per-block opt-in limit less a reserve for the kernels' static shared
// memory (about 2 KB; the attribute call fails if the sum exceeds it).
constexpr int kStaticSmemReserve = 4096;
int max_dyn_smem() {
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    if (cache[dev] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        cache[dev] = n > kStaticSmemReserve ? n - kStaticSmemReserve : 0;
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
    unsigned* block_ctr;
    int32_t* grp;  // grouped path: offsets [1025], pair [P], weight [P] (float), block list (16-B aligned)
    int32_t* fix;  // grouped path: act outputs to recompute exactly (count, pad, then int2 entries)
    int fix_cap;
    size_t bytes;
};

// Grouped-path tables in the workspace (sized for up to kGrpMaxExperts experts).
constexpr int kGrpMaxExperts = 1024;
constexpr size_t kGrpOffsets = kGrpMaxExperts + 1;

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
    w.block_ctr = reinterpret_cast<unsigned*>(p + off);
    off += align_up((size_t)((H + 63) / 64) * 4, 256);
    w.grp = reinterpret_cast<int32_t*>(p + off);
    off += align_up(4 * (kGrpOffsets + 2 * P + 4 + block_list_ints((int)P, kGrpMaxExperts)), 256);
    // one entry per 8 (pair, row) outputs of up||gate: the fraction near a
    // rounding midpoint is ~1 % (bf16) to ~3 % (fp16)
    w.fix = reinterpret_cast<int32_t*>(p + off);
    w.fix_cap = (int)std::min<size_t>((P * (size_t)I + 7) / 8, (size_t)1 << 27);
    off += align_up(16 + 16 * (size_t)w.fix_cap, 256);
    w.bytes = off;
    return w;
}

// ---- fused decode layer (decode.cu) ------------------------------------------
constexpr int kNotApplicable = -1;

// Process-wide stop flag (the reference's stopFlag buffer, SeedlessMetal.swift:
// 60, 69-70) and the bound of the kernels' device-side waits.
std::atomic<const int32_t*> g_stop_flag{nullptr};
std::atomic<int> g_spin_limit{0};
constexpr int kDefaultSpinLimit = 1 << 22;
int spin_limit() {
    const int v = g_spin_limit.load();
    if (v != 0) return v > 0 ? v : 0;
    static const int env = [] {
        const char* e = std::getenv("MOMIJ_SPIN_LIMIT");
        const long n = e ? std::strtol(e, nullptr, 10) : 0;
        return n > 0 && n < (1L << 30) ? (int)n : kDefaultSpinLimit;
    }();
    return env;
}

// cuTensorMapEncodeTiled from the driver (the runtime is linked statically).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }();
    return fn;
}

// Tensor maps of weight tensors seen as bytes [rows, row_bytes]: packed codes
// with 128-byte swizzle and boxes 128 B wide, scales and biases without
// swizzle and boxes 16 B wide; box_rows rows.  halves > 0: a 3D view [E*2
// halves, half_rows, row_bytes] whose box takes box_rows rows of two
// consecutive halves (the up and the gate rows of one expert).  Cached per
// (device, address, shape, box).
struct MapKey {
    int dev;
    const void* ptr;
    long long rows;
    int row_bytes, box_rows, box_bytes, half_rows;
    bool operator==(const MapKey& o) const {
        return dev == o.dev && ptr == o.ptr && rows == o.rows && row_bytes == o.row_bytes && box_rows == o.box_rows &&
               box_bytes == o.box_bytes && half_rows == o.half_rows;
    }
};
struct MapKeyHash {
    size_t operator()(const MapKey& k) const {
        return std::hash<const void*>()(k.ptr) ^ (std::hash<long long>()(k.rows) * 31) ^
               ((size_t)k.row_bytes << 20) ^ ((size_t)k.box_rows << 8) ^ ((size_t)k.box_bytes << 40) ^
               ((size_t)k.half_rows << 44) ^ (size_t)k.dev;
    }
};
std::mutex g_map_mu;
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps;

bool weight_map(const void* ptr, long long rows, int row_bytes, int box_bytes, int box_rows, int half_rows,
                CUtensorMap* out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    const MapKey key{dev, ptr, rows, row_bytes, box_rows, box_bytes, half_rows};
    std::lock_guard<std::mutex> lk(g_map_mu);
    auto it = g_maps.find(key);
    if (it != g_maps.end()) {
        *out = it->second;
        return true;
    }
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    CUtensorMap m;
    const CUtensorMapSwizzle swz = box_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE;
    CUresult r;
    if (half_rows > 0) {
        cuuint64_t gdim[3] = {(cuuint64_t)row_bytes, (cuuint64_t)half_rows, (cuuint64_t)(rows / half_rows)};
        cuuint64_t gstride[2] = {(cuuint64_t)row_bytes, (cuuint64_t)row_bytes * (cuuint64_t)half_rows};
        cuuint32_t box[3] = {(cuuint32_t)box_bytes, (cuuint32_t)box_rows, 2};
        cuuint32_t estr[3] = {1, 1, 1};
        r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(ptr), gdim, gstride, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    } else {
        cuuint64_t gdim[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
        cuuint64_t gstride[1] = {(cuuint64_t)row_bytes};
        cuuint32_t box[2] = {(cuuint32_t)box_bytes, (cuuint32_t)box_rows};
        cuuint32_t estr[2] = {1, 1};
        r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), gdim, gstride, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    if (r != CUDA_SUCCESS) return false;
    if (g_maps.size() >= 8192) g_maps.clear();
    g_maps.emplace(key, m);
    *out = m;
    return true;
}

// The five maps of one weight tensor (decode.cuh: kDecMaps): 2D boxes of 64,
// 16, 8 and 128 rows, and (up||gate only) the 3D box of 64 rows x 2 halves.
bool weight_maps(const void* ptr, long long rows, int row_bytes, int box_bytes, int half_rows, CUtensorMap* maps) {
    const int heights[4] = {64, 16, 8, 128};
    for (int i = 0; i < 4; ++i)
        if (!weight_map(ptr, rows, row_bytes, box_bytes, heights[i], 0, &maps[i])) return false;
    if (half_rows > 0) return weight_map(ptr, rows, row_bytes, box_bytes, 64, half_rows, &maps[4]);
    return true;
}

struct LayerCall {
    const float* logits;
    const int32_t* inds_in;
    const float* scores_in;
    int32_t* inds_out;
    float* scores_out;
    const void* x;
    const uint32_t *w_ug, *w_dn;
    const void *s_ug, *b_ug, *s_dn, *b_dn;
    void* y;
    void* resid_h;
    int M, H, I, E, K;
    float clamp;
};

using DecodeFn = void (*)(const DecodeArgs);

template <int DT, int GS>
DecodeFn pick_decode_t(int T) {
    switch (T) {
        case 1: return moe_decode_kernel<DT, GS, 1>;
        case 2: return moe_decode_kernel<DT, GS, 2>;
        case 4: return moe_decode_kernel<DT, GS, 4>;
        default: return moe_decode_kernel<DT, GS, 8>;
    }
}
DecodeFn pick_decode(int dtype, int gs, int T) {
    if (dtype == MOMIJ_DTYPE_BF16)
        return gs == 64 ? pick_decode_t<MOMIJ_DTYPE_BF16, 64>(T) : pick_decode_t<MOMIJ_DTYPE_BF16, 128>(T);
    return gs == 64 ? pick_decode_t<MOMIJ_DTYPE_F16, 64>(T) : pick_decode_t<MOMIJ_DTYPE_F16, 128>(T);
}

// Phase tracing of fused-layer launches (momij_layer_trace).
std::mutex g_trace_mu;
long long* g_trace_buf = nullptr;
size_t g_trace_slots = 0, g_trace_next = 0;

long long* next_trace_slot(int G) {
    std::lock_guard<std::mutex> lk(g_trace_mu);
    if (!g_trace_buf || g_trace_slots == 0) return nullptr;
    long long* p = g_trace_buf + (g_trace_next % g_trace_slots) * (size_t)G * kTracePointsDec;
    ++g_trace_next;
    return p;
}

bool fused_enabled() {
    const char* v = std::getenv("MOMIJ_FUSED");
    return !(v && v[0] == '0');
}

// Static shared memory of the decode kernel (DecShared and the kernel's own).
constexpr int kDecStaticReserve = 8192;

// Launches the whole layer of a 2..8-token batch (or, with MOMIJ_DECODE_M1=tc,
// one token) as one cooperative tcgen05 kernel (decode.cu) when it fits;
// kNotApplicable lets the caller fall back.
int run_decode_layer(const LayerCall& c, int dtype, int gs, const Workspace& ws, cudaStream_t st) {
    const int P = c.M * c.K;
    if (!fused_enabled() || c.M > 8 || P > kDecMaxPairs || c.E > 256 || c.K > 32 || c.H % 512 || c.I % 512)
        return kNotApplicable;
    const int G = current_device_sm_count();
    if (G <= 0 || P > G) return kNotApplicable;  // a CTA's slice then spans at most two units
    const int T = pick_tmax(c.M);
    const int N = dec_mma_n(T);
    const int nG_up = c.H / 64, nG_dn = c.I / 64;
    // tiles per CTA: rows of the slice / tile height, + 1 for a unit boundary
    // CTA slices weigh a unit's rows c0 + its tokens; the longest slice is then
    // (c0 + T) / (c0 + 1) times the even one: c0 keeps it below one unit's
    // rows (a down slice then spans at most two units) and within the tables
    int c0 = 1;
    const double even = (double)P / G;  // units per CTA at most, in unit lengths
    while (c0 < 64 && (double)(c0 + T) / (c0 + 1) * even > 0.95) ++c0;
    const double ratio = (double)(c0 + T) / (c0 + 1);
    const long long rows_up = (long long)(((double)P * c.I / G) * ratio) + 8;
    const long long rows_dn = (long long)(((double)P * c.H / G) * ratio) + 8;
    if (rows_up / 64 + 2 > kDecMaxTiles || rows_dn / 128 + 2 > kDecMaxTiles ||
        rows_dn / 64 + 4 > kDecMaxLastBlocks || rows_dn > c.H)
        return kNotApplicable;

    // TMA row strides are multiples of 16 bytes: the scale rows (Kd / gs halves) too
    if ((c.H / gs * 2) % 16 || (c.I / gs * 2) % 16) return kNotApplicable;
    DecodeArgs a{};
    const long long wrows_ug = (long long)c.E * 2 * c.I, wrows_dn = (long long)c.E * c.H;
    if (!weight_maps(c.w_ug, wrows_ug, c.H / 4, 128, c.I, a.map_ug) ||
        !weight_maps(c.s_ug, wrows_ug, c.H / gs * 2, 16, c.I, a.map_sug) ||
        !weight_maps(c.b_ug, wrows_ug, c.H / gs * 2, 16, c.I, a.map_bug) ||
        !weight_maps(c.w_dn, wrows_dn, c.I / 4, 128, 0, a.map_dn) ||
        !weight_maps(c.s_dn, wrows_dn, c.I / gs * 2, 16, 0, a.map_sdn) ||
        !weight_maps(c.b_dn, wrows_dn, c.I / gs * 2, 16, 0, a.map_bdn))
        return kNotApplicable;
    a.logits = c.logits;
    a.inds_in = c.inds_in;
    a.scores_in = c.scores_in;
    a.inds_out = c.inds_out;
    a.scores_out = c.scores_out;
    a.x = static_cast<const uint16_t*>(c.x);
    a.act = ws.act;
    a.down = ws.down;
    a.y = c.resid_h ? nullptr : static_cast<uint16_t*>(c.y);
    a.h = static_cast<uint16_t*>(c.resid_h);
    a.ctrl = ws.plan;
    a.block_ctr = ws.block_ctr;
    a.stop = g_stop_flag.load();
    a.trace = next_trace_slot(G);
    a.M = c.M;
    a.H = c.H;
    a.I = c.I;
    a.E = c.E;
    a.K = c.K;
    a.gs = gs;
    a.spin_limit = spin_limit();
    a.slice_c0 = c0;
    a.clamp = c.clamp;

    // shared memory: ring of stages (codes + scales + biases) | B | per-group
    // factors | tile-end partials; the logits live in the ring (the producers
    // start only after the routing)
    const size_t b_bytes = (size_t)std::max(nG_up, 2 * nG_dn) * dec_b_group_bytes(N);
    const size_t fs_bytes = align_up(8 * (size_t)std::max(c.M * nG_up, 2 * T * nG_dn), 16);
    const size_t red_bytes = (size_t)4 * T * 128 * 4;  // one partial per MMA issuer
    const size_t lg_bytes = align_up(4 * (size_t)(c.logits ? c.M * c.E : 0), 16);
    const size_t fixed = align_up(b_bytes, 1024) + fs_bytes + red_bytes + 1024;
    int optin = 0, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    const long long room = (long long)optin - kDecStaticReserve - (long long)fixed;
    int stages = (int)std::min<long long>(kDecMaxStages, room / kDecStageBytes) & ~1;
    if (stages < 2 || (size_t)stages * kDecStageBytes < lg_bytes) return kNotApplicable;
    size_t off = 0;
    a.off_ring = (int)off; off += (size_t)stages * kDecStageBytes;
    a.off_b = (int)off; off += align_up(b_bytes, 1024);
    a.off_fs = (int)off; off += fs_bytes;
    a.off_red = (int)off; off += red_bytes;
    a.off_logits = a.off_ring;
    const size_t smem = off + 1024;  // + alignment of the base to 1024 B
    a.stages = stages;
    a.b_bytes = (int)b_bytes;

    DecodeFn fn = pick_decode(dtype, gs, T);
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return MOMIJ_ERR_CUDA;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kDecThreadsAll, smem) != cudaSuccess ||
        per_sm < 1)
        return kNotApplicable;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(G);
    cfg.blockDim = dim3(kDecThreadsAll);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    static bool pdl_with_coop = true;  // dropped if the driver refuses the pair
    cfg.numAttrs = (pdl_enabled() && pdl_with_coop) ? 2 : 1;
    const int slot = prof_begin(MOMIJ_KERNEL_LAYER, st);
    cudaError_t e = cudaLaunchKernelEx(&cfg, fn, a);
    if (e != cudaSuccess && cfg.numAttrs == 2) {
        cudaGetLastError();
        pdl_with_coop = false;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, fn, a);
    }
    prof_end(slot, st);
    return cuda_status(e);
}

// ---- single-token layer engine (layer.cu) ----------------------------------
using LayerFn = void (*)(const LayerArgs);

LayerFn pick_layer(int dtype, int gs) {
    if (dtype == MOMIJ_DTYPE_BF16)
        return gs == 64 ? moe_layer_kernel<MOMIJ_DTYPE_BF16, 64, 1, layer_stages(1)>
                        : moe_layer_kernel<MOMIJ_DTYPE_BF16, 128, 1, layer_stages(1)>;
    return gs == 64 ? moe_layer_kernel<MOMIJ_DTYPE_F16, 64, 1, layer_stages(1)>
                    : moe_layer_kernel<MOMIJ_DTYPE_F16, 128, 1, layer_stages(1)>;
}

// One token's whole layer as one cooperative kernel on the warp-level engine
// (the fastest single-token path measured); kNotApplicable when it does not fit.
int run_layer_engine(const LayerCall& c, int dtype, int gs, const Workspace& ws, cudaStream_t st) {
    const int P = c.M * c.K;
    if (c.M != 1 || P > kLayerMaxPairs || c.E > 1024 || c.K > 32) return kNotApplicable;
    const int tmax = 1, stages = layer_stages(tmax), rt = item_tiles(tmax);
    const int G = current_device_sm_count();
    if (G <= 0) return kNotApplicable;
    LayerArgs a{};
    a.logits = c.logits;
    a.inds_in = c.inds_in;
    a.scores_in = c.scores_in;
    a.inds_out = c.inds_out;
    a.scores_out = c.scores_out;
    a.x = static_cast<const uint16_t*>(c.x);
    a.w_ug = c.w_ug;
    a.s_ug = static_cast<const uint16_t*>(c.s_ug);
    a.b_ug = static_cast<const uint16_t*>(c.b_ug);
    a.w_dn = c.w_dn;
    a.s_dn = static_cast<const uint16_t*>(c.s_dn);
    a.b_dn = static_cast<const uint16_t*>(c.b_dn);
    a.y = c.resid_h ? nullptr : static_cast<uint16_t*>(c.y);
    a.h = static_cast<uint16_t*>(c.resid_h);
    a.M = c.M;
    a.H = c.H;
    a.I = c.I;
    a.E = c.E;
    a.K = c.K;
    a.clamp = c.clamp;
    a.stop = g_stop_flag.load();
    a.spin_limit = spin_limit();
    a.nK_up = a.H / kChunk;
    a.nK_dn = a.I / kChunk;
    const long long rows_up = ((long long)P * a.I + G - 1) / G;
    const long long rows_dn = ((long long)P * a.H + G - 1) / G;
    const int mu_up = (int)std::min<long long>(P, rows_up / a.I + 2);
    const int mu_dn = (int)std::min<long long>(P, rows_dn / a.H + 2);
    const int mt_up = (int)(rows_up / 8 + mu_up + 1);
    const int mt_dn = (int)(rows_dn / 16 + mu_dn + 1);
    if (rows_dn / 64 + 2 * mu_dn > kLayerMaxLastBlocks) return kNotApplicable;
    const int max_units = std::max(mu_up, mu_dn), max_tiles = std::max(mt_up, mt_dn);
    const int vec_dn = std::min(P, mu_dn * tmax);
    a.max_tiles = max_tiles;
    a.max_units = max_units;
    a.max_vec = vec_dn;
    const size_t ndg = std::max((size_t)a.M * (a.H / 64), (size_t)vec_dn * (a.I / 64));
    const size_t limit = (size_t)max_dyn_smem();
    size_t off = 0;
    a.off_logits = (int)off; off += a.logits ? 4 * (size_t)a.M * a.E : 0;
    off = align_up(off, 16);
    a.off_inds = (int)off; off += 4 * (size_t)P;
    a.off_scores = (int)off; off += 4 * (size_t)P;
    a.off_sorted = (int)off; off += 4 * (size_t)P;
    off = align_up(off, 16);
    a.off_pflag = (int)off; off += 16 * (size_t)P;  // per sorted pair: (expert, before, count)
    a.off_units = (int)off; off += 16 * (size_t)P;
    a.off_tiles_up = (int)off; off += 16 * (size_t)max_tiles;
    a.off_lunits_up = (int)off; off += 16 * (size_t)max_units;
    a.off_seg_up = (int)off; off += 16 * (size_t)max_units;
    a.off_tiles_dn = (int)off; off += 16 * (size_t)max_tiles;
    a.off_lunits_dn = (int)off; off += 16 * (size_t)max_units;
    a.off_seg_dn = (int)off; off += 16 * (size_t)max_units;
    a.off_upair_up = (int)off; off += 4 * (size_t)max_units * tmax;
    a.off_uslot_up = (int)off; off += 4 * (size_t)max_units * tmax;
    a.off_upair_dn = (int)off; off += 4 * (size_t)max_units * tmax;
    a.off_uslot_dn = (int)off; off += 4 * (size_t)max_units * tmax;
    a.off_xvecs = (int)off; off += 4 * (size_t)a.M;
    a.off_vecs_dn = (int)off; off += 4 * (size_t)vec_dn;
    off = align_up(off, 16);
    a.off_fs = (int)off; off += 8 * ndg;
    off = align_up(off, 16);
    a.off_dig = (int)off; off += (size_t)kDgStride * ndg;
    off = align_up(off, 16);
    // the red and scale/bias buffers take what the ring leaves, up to a whole
    // phase per batch; the phases share them
    const size_t ring = (size_t)kConsumerWarps * stages * slot_bytes(tmax);
    if (off + ring + 256 > limit) return kNotApplicable;
    const size_t avail = limit - off - ring - 256;
    const size_t rpt_up = 4 * (size_t)((a.nK_up + 1) / 2) * tmax * red_row(tmax),
                 rpt_dn = 4 * (size_t)((a.nK_dn + 1) / 2) * tmax * red_row(tmax);
    const size_t spt_up = sb_bytes_per_tile(a.H, gs, true), spt_dn = sb_bytes_per_tile(a.I, gs, true);
    size_t bu = (size_t)(mt_up + rt - 1) / rt * rt, bd = (size_t)(mt_dn + rt - 1) / rt * rt;
    auto need = [&]() { return std::max(bu * rpt_up, bd * rpt_dn) + std::max(bu * spt_up, bd * spt_dn) + 16; };
    while (need() > avail && (bu > (size_t)rt || bd > (size_t)rt)) {
        if (bu * (rpt_up + spt_up) >= bd * (rpt_dn + spt_dn) && bu > (size_t)rt)
            bu = std::max((size_t)rt, (bu / 2 + rt - 1) / rt * rt);
        else
            bd = std::max((size_t)rt, (bd / 2 + rt - 1) / rt * rt);
    }
    if (need() > avail) return kNotApplicable;
    a.batch_up = (int)bu;
    a.batch_dn = (int)bd;
    a.off_red = (int)off; off += std::max(bu * rpt_up, bd * rpt_dn);
    off = align_up(off, 16);
    a.off_sb = (int)off; off += std::max(bu * spt_up, bd * spt_dn);
    off = align_up(off, 128);
    a.off_stage = (int)off; off += ring;
    LayerFn fn = pick_layer(dtype, gs);
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)off) != cudaSuccess)
        return MOMIJ_ERR_CUDA;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kLayerThreads, off) != cudaSuccess || per_sm < 1)
        return kNotApplicable;
    a.trace = next_trace_slot(G);
    a.ctrl = ws.plan;
    a.block_ctr = ws.block_ctr;
    a.act = ws.act;
    a.down = ws.down;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(G);
    cfg.blockDim = dim3(kLayerThreads);
    cfg.dynamicSmemBytes = off;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    static bool pdl_with_coop = true;  // dropped if the driver refuses the pair
    cfg.numAttrs = (pdl_enabled() && pdl_with_coop) ? 2 : 1;
    const int slot = prof_begin(MOMIJ_KERNEL_LAYER, st);
    cudaError_t e = cudaLaunchKernelEx(&cfg, fn, a);
    if (e != cudaSuccess && cfg.numAttrs == 2) {
        cudaGetLastError();
        pdl_with_coop = false;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, fn, a);
    }
    prof_end(slot, st);
    return cuda_status(e);
}

// ---- single-token streaming layer (token.cu) ---------------------------------
using TokenFn = void (*)(const TokenArgs);

// The up||gate codes [2E halves][I rows][H/4 bytes] seen as the 4D tensor
// [128 B][I rows][H/512 column chunks][2E halves]: one box (128 B, 8 rows,
// every chunk, 2 halves) is a tile of 8 up rows and the matching 8 gate rows,
// laid out in shared memory as [half][chunk][row][128 B] (128-byte swizzle).
// Cached per (device, address, shape).
bool up_tile_map(const void* ptr, long long E, int I, int H, CUtensorMap* out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    const MapKey key{dev, ptr, E * 2 * I, H / 4, 8, 128, -I};  // negative half_rows: this 4D view
    std::lock_guard<std::mutex> lk(g_map_mu);
    auto it = g_maps.find(key);
    if (it != g_maps.end()) {
        *out = it->second;
        return true;
    }
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    const cuuint64_t rb = (cuuint64_t)H / 4;
    cuuint64_t gdim[4] = {128, (cuuint64_t)I, (cuuint64_t)H / 512, (cuuint64_t)(2 * E)};
    cuuint64_t gstride[3] = {rb, 128, rb * (cuuint64_t)I};
    cuuint32_t box[4] = {128, 8, (cuuint32_t)(H / 512), 2};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUtensorMap m;
    if (enc(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(ptr), gdim, gstride, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    if (g_maps.size() >= 8192) g_maps.clear();
    g_maps.emplace(key, m);
    *out = m;
    return true;
}

// One token's whole layer as one cooperative kernel that streams the expert
// weights by TMA (token.cu); kNotApplicable when the shapes, the alignment or
// the shared memory do not fit (gs 64, K <= 8, H <= 4096, H and I multiples
// of 512, E <= 512 when routing from logits).
int run_token_layer(const LayerCall& c, int dtype, int gs, const Workspace& ws, cudaStream_t st,
                    bool status_merge = false) {
    if (c.M < 1 || c.M > kTokMaxM || gs != 64 || c.K > kTokMaxK || c.K < 1 || (c.logits && c.E > kTokMaxE) ||
        c.H % 512 || c.I % 512 || c.H > 4096)
        return kNotApplicable;
    if (!aligned(c.w_ug, 16) || !aligned(c.w_dn, 16) || !aligned(c.s_ug, 16) || !aligned(c.b_ug, 16) ||
        !aligned(c.s_dn, 16) || !aligned(c.b_dn, 16) || !aligned(c.x, 16) || !aligned(ws.act, 16))
        return kNotApplicable;
    const int G = current_device_sm_count();
    if (G <= 0) return kNotApplicable;
    const long long T = (long long)c.K * c.I / 8;
    const int max_tiles = (int)((T + G - 1) / G);
    const int rpc = (c.H + G - 1) / G;
    if (max_tiles > kTokMaxTiles || rpc > kTokDnRows) return kNotApplicable;
    TokenArgs a{};
    const long long E = c.E;
    const int srb_up = c.H / 32, srb_dn = c.I / 32;  // scale bytes per row (gs 64)
    if (!up_tile_map(c.w_ug, E, c.I, c.H, &a.map[0]) ||
        !weight_map(c.s_ug, E * 2 * c.I, srb_up, srb_up, 8, c.I, &a.map[1]) ||
        !weight_map(c.b_ug, E * 2 * c.I, srb_up, srb_up, 8, c.I, &a.map[2]) ||
        !weight_map(c.w_dn, E * c.H, c.I / 4, 128, rpc, 0, &a.map[3]) ||
        !weight_map(c.s_dn, E * c.H, srb_dn, 16, rpc, 0, &a.map[4]) ||
        !weight_map(c.b_dn, E * c.H, srb_dn, 16, rpc, 0, &a.map[5]))
        return kNotApplicable;
    a.logits = c.logits;
    a.inds_in = c.inds_in;
    a.scores_in = c.scores_in;
    a.inds_out = c.inds_out;
    a.scores_out = c.scores_out;
    a.x = static_cast<const uint16_t*>(c.x);
    a.act = ws.act;
    a.y = c.resid_h ? nullptr : static_cast<uint16_t*>(c.y);
    a.h = static_cast<uint16_t*>(c.resid_h);
    a.ctrl = ws.plan;
    a.bar64 = reinterpret_cast<unsigned long long*>(ws.plan + kCtrlBar64);
    a.stop = g_stop_flag.load();
    a.H = c.H;
    a.I = c.I;
    a.E = c.E;
    a.K = c.K;
    a.M = c.M;
    a.spin_limit = spin_limit();
    a.status_merge = status_merge ? 1 : 0;
    a.rows_per_cta = rpc;
    a.clamp = c.clamp;
    // shared memory (from a 1024-aligned base): the stage ring, the logits,
    // then one region that the up phase (x digits, their group factors, up
    // partials) and the down phase (act digits, factors, down partials) use in turn
    size_t off = 0;
    a.off_ring = (int)off;
    off += (size_t)kTokStages * kTokStageBytes;
    a.off_logits = (int)off;
    off = align_up(off + 4 * std::max((size_t)kTokThreads, (size_t)c.M * c.E), 128);
    const size_t reg = off;
    a.off_xb = (int)off;
    off = align_up(off + tok_b_bytes(c.H), 16);
    a.off_xfs = (int)off;
    off = align_up(off + 8 * (size_t)(c.H / 64), 16);
    a.off_red_up = (int)off;
    off += 4 * (size_t)max_tiles * 16 * tok_red_stride(c.H / 512);
    const size_t end_up = off;
    off = reg;
    a.off_ab = (int)off;
    off = align_up(off + (size_t)c.K * tok_b_bytes(c.I), 16);
    a.off_afs = (int)off;
    off = align_up(off + 8 * (size_t)c.K * (c.I / 64), 16);
    a.off_red_dn = (int)off;
    off += 4 * (size_t)c.K * kTokDnRows * tok_red_stride(c.I / 512);
    off = std::max(off, end_up) + 1024;  // + the alignment slack of the base
    if (off > (size_t)max_dyn_smem()) return kNotApplicable;
    TokenFn fn = dtype == MOMIJ_DTYPE_BF16 ? moe_token_kernel<MOMIJ_DTYPE_BF16> : moe_token_kernel<MOMIJ_DTYPE_F16>;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)off) != cudaSuccess)
        return MOMIJ_ERR_CUDA;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kTokThreads, off) != cudaSuccess || per_sm < 1)
        return kNotApplicable;
    a.trace = next_trace_slot(G);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(G);
    cfg.blockDim = dim3(kTokThreads);
    cfg.dynamicSmemBytes = off;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    static bool pdl_with_coop = true;  // dropped if the driver refuses the pair
    cfg.numAttrs = (pdl_enabled() && pdl_with_coop) ? 2 : 1;
    const int slot = prof_begin(MOMIJ_KERNEL_LAYER, st);
    cudaError_t e = cudaLaunchKernelEx(&cfg, fn, a);
    if (e != cudaSuccess && cfg.numAttrs == 2) {
        cudaGetLastError();
        pdl_with_coop = false;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, fn, a);
    }
    prof_end(slot, st);
    return cuda_status(e);
}

// Engine of single-token layers: MOMIJ_DECODE_M1=warp selects the warp-level
// engine (layer.cu), =tc the tcgen05 kernel (decode.cu); the default is the
// TMA-streaming kernel (token.cu), with the warp-level engine for the shapes
// it does not take.
int m1_engine() {  // read per call: tests and benchmarks switch engines within a process
    const char* e = std::getenv("MOMIJ_DECODE_M1");
    if (e && std::strcmp(e, "tc") == 0) return 2;
    if (e && std::strcmp(e, "warp") == 0) return 1;
    return 0;
}

// Batches of 2..8 tokens: by default one launch of the streaming kernel that
// takes the tokens one after another (its producer streams the next token's
// weights during the current token's serial tail); MOMIJ_DECODE_MROW=seq
// launches it once per token, =tc takes the batched tcgen05 kernel.  Both
// streaming forms give the bits of M single-token calls; they beat the
// batched kernel at every size measured here (each token streams its own
// experts at the streaming rate, the batched kernel the distinct experts
// once at a lower rate).  Read per call, like m1_engine.
int mrow_mode() {
    const char* e = std::getenv("MOMIJ_DECODE_MROW");
    if (e && std::strcmp(e, "tc") == 0) return 2;
    if (e && std::strcmp(e, "seq") == 0) return 1;
    return 0;
}

// The tokens of a batch one by one through the streaming kernel: the same
// bits as M single-token calls.  kNotApplicable (before any launch) when the
// kernel does not take the shapes.
int run_token_batch(const LayerCall& c, int dtype, int gs, const Workspace& ws, cudaStream_t st) {
    const size_t esz = 2;  // bytes of a 16-bit activation
    for (int m = 0; m < c.M; ++m) {
        LayerCall t = c;
        t.M = 1;
        t.logits = c.logits ? c.logits + (size_t)m * c.E : nullptr;
        t.inds_in = c.inds_in ? c.inds_in + (size_t)m * c.K : nullptr;
        t.scores_in = c.scores_in ? c.scores_in + (size_t)m * c.K : nullptr;
        t.inds_out = c.inds_out ? c.inds_out + (size_t)m * c.K : nullptr;
        t.scores_out = c.scores_out ? c.scores_out + (size_t)m * c.K : nullptr;
        t.x = static_cast<const unsigned char*>(c.x) + (size_t)m * c.H * esz;
        t.y = c.y ? static_cast<unsigned char*>(c.y) + (size_t)m * c.H * esz : nullptr;
        t.resid_h = c.resid_h ? static_cast<unsigned char*>(c.resid_h) + (size_t)m * c.H * esz : nullptr;
        const int rc = run_token_layer(t, dtype, gs, ws, st, m > 0);
        if (rc != MOMIJ_OK) return rc;  // kNotApplicable only at m == 0: the shapes are the same for every token
    }
    return MOMIJ_OK;
}

// The fused layer: one token on the streaming kernel (or the engine the
// environment selects), 2..8 tokens token by token on the same kernel or on
// the batched tcgen05 kernel; kNotApplicable lets the caller fall back to the
// multi-kernel path.
int run_fused_layer(const LayerCall& c, int dtype, int gs, const Workspace& ws, cudaStream_t st) {
    if (!fused_enabled()) return kNotApplicable;
    if (c.M == 1 && m1_engine() == 0) {
        const int rc = run_token_layer(c, dtype, gs, ws, st);
        if (rc != kNotApplicable) return rc;
    }
    if (c.M > 1 && c.M <= kTokMaxM && m1_engine() == 0 && mrow_mode() != 2) {
        const int rc = mrow_mode() == 0 ? run_token_layer(c, dtype, gs, ws, st) : kNotApplicable;
        if (rc != kNotApplicable) return rc;
        const int rs = run_token_batch(c, dtype, gs, ws, st);
        if (rs != kNotApplicable) return rs;
    }
    if (c.M == 1 && m1_engine() != 2) {
        const int rc = run_layer_engine(c, dtype, gs, ws, st);
        if (rc != kNotApplicable) return rc;
    }
    return run_decode_layer(c, dtype, gs, ws, st);
}

// ---- gather-GEMV dispatch --------------------------------------------------
using GemvFn = void (*)(const GemvArgs);

template <int DT, int GS, int MODE>
GemvFn pick_tm_st(int tmax, int stages) {
    const bool s4 = stages == 4;
    switch (tmax) {
        case 1: return s4 ? gemv_kernel<DT, GS, MODE, 1, 4> : gemv_kernel<DT, GS, MODE, 1, 2>;
        case 2: return s4 ? gemv_kernel<DT, GS, MODE, 2, 4> : gemv_kernel<DT, GS, MODE, 2, 2>;
        case 4: return s4 ? gemv_kernel<DT, GS, MODE, 4, 4> : gemv_kernel<DT, GS, MODE, 4, 2>;
        default: return s4 ? gemv_kernel<DT, GS, MODE, 8, 4> : gemv_kernel<DT, GS, MODE, 8, 2>;
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
    int grid, threads, stages, tmax;
    size_t smem;
};
bool configure_gemv_smem(GemvLaunch& L, int nDG, size_t limit, size_t pt, int gs);

// Worst-case shared-memory sizing from (P, shapes); returns false if the
// configuration cannot fit on the device.
bool configure_gemv(GemvLaunch& L, int mode, int tmax, int gs) {
    GemvArgs& a = L.a;
    L.tmax = tmax;
    const int nK = a.Kd / kChunk;
    a.nK = nK;
    L.threads = kGemvThreads;
    const int TR = mode == kModeUpSwiglu ? 8 : 16;
    const long long Ru = a.rows_per_unit;
    const long long Rmax = (long long)a.P * Ru;
    const int sms = current_device_sm_count();
    if (sms <= 0) return false;
    long long G = (Rmax + TR - 1) / TR;
    if (G > sms) G = sms;
    if (G < 1) G = 1;
    L.grid = (int)G;
    const int nDG = a.Kd / kDigitGroup;
    const size_t limit = (size_t)max_dyn_smem();
    const size_t pt = 4 * (size_t)((nK + 1) / 2) * tmax * red_row(tmax);  // red_floats_per_tile
    // A CTA's slice starts as its share of the worst case; when the slice's
    // tables and token digits do not fit, slices shrink and each CTA loops
    // over several (large batches of few tokens per expert).
    for (long long rows_cta = (Rmax + G - 1) / G; rows_cta >= TR; rows_cta = (rows_cta + 1) / 2) {
        a.slice_rows = (int)std::min<long long>(rows_cta, 1LL << 30);
        a.max_units = (int)std::min<long long>(a.P, rows_cta / Ru + 2);
        a.max_tiles = (int)(rows_cta / TR + a.max_units + 1);
        a.max_vec = a.digit_all_tokens ? a.M : std::min(a.P, a.max_units * tmax);
        if (configure_gemv_smem(L, nDG, limit, pt, gs)) return true;
        if (rows_cta == TR) break;
    }
    return false;
}

// Shared-memory carve-up for the slice bounds in L.a (max_units, max_tiles,
// max_vec); false if even the smallest ring does not fit.
bool configure_gemv_smem(GemvLaunch& L, int nDG, size_t limit, size_t pt, int gs) {
    GemvArgs& a = L.a;
    const int tmax = L.tmax;
    const int rt = item_tiles(tmax);
    for (int stages : {4, 2}) {
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
        // the red and scale/bias buffers take what the ring leaves, up to
        // all tiles at once
        const size_t ring = (size_t)kConsumerWarps * stages * slot_bytes(tmax);
        if (off + ring + 256 > limit) continue;
        const size_t spt = sb_bytes_per_tile(a.Kd, gs, true);
        const size_t bt = std::min((size_t)(a.max_tiles + rt - 1) / rt * rt,
                                   (limit - off - ring - 256) / (pt + spt) / rt * rt);
        if (bt < (size_t)rt) continue;
        a.batch_tiles = (int)bt;
        a.off_red = (int)off;
        off += bt * pt;
        off = align_up(off, 16);
        a.off_sb = (int)off;
        off += bt * spt;
        off = align_up(off, 128);
        a.off_stage = (int)off; off += ring;
        L.stages = stages;
        L.smem = off;
        return true;
    }
    return false;
}

int run_gemv(GemvLaunch& L, int mode, int tmax, int dtype, int gs, cudaStream_t st) {
    if (!configure_gemv(L, mode, tmax, gs)) return MOMIJ_ERR_UNSUPPORTED_SHAPE;
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
    // Batches beyond 8 tokens cut units at 4 pairs: the digits of a slice's
    // two units (8 vectors) then fit in shared memory at H = 4096.
    return pick_tmax(M < 1 ? 1 : (M > 8 ? 4 : M));
    (void)Ktop;
}

int launch_plan(const int32_t* inds, int P, int E, int tmax, int32_t* plan, cudaStream_t st,
                int allow_pad = 0) {
    const int slot = prof_begin(MOMIJ_KERNEL_PLAN, st);
    const int rc = cuda_status(
        launch(plan_kernel, dim3(1), dim3(1024), 0, st, inds, P, E, tmax, plan, allow_pad));
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

// ---- grouped (prefill) path: permute + tcgen05 grouped GEMMs + combine ------
bool grouped_enabled(int M, int Ktop, int E) {
    const char* v = std::getenv("MOMIJ_GROUPED");
    if (v && v[0] == '0') return (long long)M * Ktop > MOMIJ_MAX_PAIRS;  // forced off unless required
    if (v && v[0] == '1') return M > 8;
    // tokens per expert large enough for the weights to be re-used across tokens
    return M > 8 && ((long long)M * Ktop >= 32LL * E || (long long)M * Ktop > MOMIJ_MAX_PAIRS);
}

using GroupedFn = void (*)(const GroupedArgs);
using FixupFn = void (*)(const FixupArgs);
FixupFn pick_fixup(int dtype, int gs) {
    if (dtype == MOMIJ_DTYPE_BF16)
        return gs == 64 ? act_fixup_kernel<MOMIJ_DTYPE_BF16, 64> : act_fixup_kernel<MOMIJ_DTYPE_BF16, 128>;
    return gs == 64 ? act_fixup_kernel<MOMIJ_DTYPE_F16, 64> : act_fixup_kernel<MOMIJ_DTYPE_F16, 128>;
}
template <int DT, int GS>
GroupedFn pick_grouped_dt(int mode) {
    return mode == kModeUpSwiglu ? grouped_gemm_kernel<DT, GS, kModeUpSwiglu> : grouped_gemm_kernel<DT, GS, kModeRows>;
}
GroupedFn pick_grouped(int dtype, int gs, int mode) {
    if (dtype == MOMIJ_DTYPE_BF16)
        return gs == 64 ? pick_grouped_dt<MOMIJ_DTYPE_BF16, 64>(mode) : pick_grouped_dt<MOMIJ_DTYPE_BF16, 128>(mode);
    return gs == 64 ? pick_grouped_dt<MOMIJ_DTYPE_F16, 64>(mode) : pick_grouped_dt<MOMIJ_DTYPE_F16, 128>(mode);
}

int run_grouped(const void* x, const uint32_t* w_ug, const void* s_ug, const void* b_ug,
                const uint32_t* w_dn, const void* s_dn, const void* b_dn, const int32_t* inds,
                const float* scores, void* y, void* resid_h, int M, int H, int I, int E, int Ktop,
                int gs, float clamp, int dtype, const Workspace& ws, cudaStream_t st) {
    if (E > kGrpMaxExperts || I % 64 || H % 128) return MOMIJ_ERR_UNSUPPORTED_SHAPE;
    const int P = M * Ktop;
    // status words: the work-plan header ([1] routing status, [2] sticky error
    // word), as for the other paths (combine_kernel, momij_moe_synchronize)
    int32_t* hdr = ws.plan;
    int32_t* offsets = ws.grp;
    int32_t* pair = offsets + kGrpOffsets;
    float* weight = reinterpret_cast<float*>(pair + P);
    // the block list is read as int4 entries: 16-byte aligned (the region has 4 ints of slack)
    int32_t* blocks = reinterpret_cast<int32_t*>(align_up(reinterpret_cast<uintptr_t>(weight + P), 16));
    if (cudaMemsetAsync(hdr + 1, 0, sizeof(int32_t), st) != cudaSuccess ||
        cudaMemsetAsync(ws.fix, 0, sizeof(int32_t), st) != cudaSuccess)
        return MOMIJ_ERR_CUDA;
    const int G = current_device_sm_count();
    if (G <= 0) return MOMIJ_ERR_CUDA;
    int slot = prof_begin(MOMIJ_KERNEL_PLAN, st);
    int rc = cuda_status(launch(permute_kernel, dim3(std::min(E, 2 * G)), dim3(kPermuteThreads),
                                sizeof(int) * (E + 1), st, inds, scores, P, E, offsets, pair, weight, hdr + 1));
    if (!rc) rc = cuda_status(launch(block_list_kernel, dim3(1), dim3(32), 0, st,
                                     static_cast<const int32_t*>(offsets), E, blocks,
                                     static_cast<const int32_t*>(hdr + 1)));
    prof_end(slot, st);
    if (rc) return rc;
    const size_t smem = grouped_smem_bytes();
    // The GEMMs run along K in class order (the dequantised weight tiles'
    // order): the tokens are reordered into the down buffer (free until the
    // down GEMM, M <= P rows) and the up GEMM writes act in that order.
    {
        const long long blocks16 = (long long)M * H / 16;
        const int nb = (int)std::min<long long>((blocks16 + 255) / 256, 4L * G);
        rc = cuda_status(launch(class_order_kernel, dim3(nb > 0 ? nb : 1), dim3(256), 0, st,
                                static_cast<const uint4*>(x), reinterpret_cast<uint4*>(ws.down), blocks16));
        if (rc) return rc;
    }
    for (int mode : {kModeUpSwiglu, kModeRows}) {
        GroupedArgs a{};
        a.x = static_cast<const uint16_t*>(mode == kModeUpSwiglu ? ws.down : ws.act);
        a.x_per_pair = mode == kModeUpSwiglu ? 0 : 1;
        a.w = mode == kModeUpSwiglu ? w_ug : w_dn;
        a.s = static_cast<const uint16_t*>(mode == kModeUpSwiglu ? s_ug : s_dn);
        a.b = static_cast<const uint16_t*>(mode == kModeUpSwiglu ? b_ug : b_dn);
        a.blocks = blocks;
        a.pairs = pair;
        a.status = hdr;
        a.out = mode == kModeUpSwiglu ? ws.act : ws.down;
        a.Kd = mode == kModeUpSwiglu ? H : I;
        a.N = mode == kModeUpSwiglu ? 2 * I : H;
        a.Ru = mode == kModeUpSwiglu ? I : 0;
        a.Ktop = Ktop;
        a.clamp = clamp;
        a.E = E;
        a.P = P;
        a.fix = mode == kModeUpSwiglu ? ws.fix : nullptr;
        a.fix_cap = ws.fix_cap;
        a.fix_ulps = fix_ulps_for(H);
        GroupedFn fn = pick_grouped(dtype, gs, mode);
        if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return MOMIJ_ERR_CUDA;
        slot = prof_begin(mode == kModeUpSwiglu ? MOMIJ_KERNEL_UP : MOMIJ_KERNEL_ROWS, st);
        rc = cuda_status(launch(fn, dim3(G), dim3(kGroupedThreads), smem, st, a));
        if (!rc && mode == kModeUpSwiglu) {  // the listed act values, exactly
            FixupArgs f{};
            f.x = static_cast<const uint16_t*>(x);
            f.w = w_ug;
            f.s = static_cast<const uint16_t*>(s_ug);
            f.b = static_cast<const uint16_t*>(b_ug);
            f.inds = inds;
            f.fix = ws.fix;
            f.status = hdr;
            f.act = ws.act;
            f.Kd = H;
            f.I = I;
            f.Ktop = Ktop;
            f.fix_cap = ws.fix_cap;
            f.clamp = clamp;
            rc = cuda_status(launch(pick_fixup(dtype, gs), dim3(4 * G), dim3(256), 0, st, f));
        }
        prof_end(slot, st);
        if (rc) return rc;
    }
    return launch_combine_dt(dtype, ws.down, scores, static_cast<uint16_t*>(resid_h ? resid_h : y), M,
                             Ktop, H, resid_h != nullptr, hdr, st);
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

int momij_layer_trace(void* device_buffer, size_t bytes) {
    std::lock_guard<std::mutex> lk(g_trace_mu);
    const int G = current_device_sm_count();
    if (!device_buffer || bytes == 0 || G <= 0) {
        g_trace_buf = nullptr;
        g_trace_slots = 0;
        return device_buffer ? MOMIJ_ERR_INVALID_ARGUMENT : MOMIJ_OK;
    }
    g_trace_buf = static_cast<long long*>(device_buffer);
    g_trace_slots = bytes / ((size_t)G * kTracePointsDec * sizeof(long long));
    g_trace_next = 0;
    return g_trace_slots ? MOMIJ_OK : MOMIJ_ERR_WORKSPACE;
}

int momij_profile_reset(void) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    for (auto& r : g_prof) r.used = false;
    return MOMIJ_OK;
}

int momij_device_sm_count(void) { return current_device_sm_count(); }

int momij_set_stop_flag(const int32_t* device_flag) {
    g_stop_flag.store(device_flag);
    return MOMIJ_OK;
}

int momij_set_spin_limit(int polls) {
    if (polls < -1) return MOMIJ_ERR_INVALID_ARGUMENT;
    g_spin_limit.store(polls);
    return MOMIJ_OK;
}

int momij_moe_synchronize(momij_stream_t stream, const void* workspace) {
    if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess) return MOMIJ_ERR_CUDA;
    if (!workspace) return MOMIJ_OK;
    int32_t hdr[3] = {0, 0, 0};
    if (cudaMemcpy(hdr, workspace, sizeof(hdr), cudaMemcpyDeviceToHost) != cudaSuccess)
        return MOMIJ_ERR_CUDA;
    if (hdr[1] != MOMIJ_OK) return hdr[1];
    if (hdr[2] != MOMIJ_OK) {
        // the error word is sticky on the device; report it once
        int32_t* err = static_cast<int32_t*>(const_cast<void*>(workspace)) + 2;
        if (cudaMemset(err, 0, sizeof(int32_t)) != cudaSuccess) return MOMIJ_ERR_CUDA;
    }
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
    const int G = current_device_sm_count();
    if (G <= 0) return MOMIJ_ERR_CUDA;
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(permute_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return MOMIJ_ERR_CUDA;
    return cuda_status(launch(permute_kernel, dim3(std::min(E, 2 * G)), dim3(kPermuteThreads), smem,
                              static_cast<cudaStream_t>(stream), inds, scores, M * K, E, offsets,
                              pair, weight, static_cast<int32_t*>(nullptr)));
}

namespace {
using GateFn = void (*)(const uint16_t*, const uint16_t*, float*, int, int, int);
using RouterFn = void (*)(const uint16_t*, const uint16_t*, unsigned*, float*, int32_t*, float*, int, int, int,
                          int);
GateFn pick_gate(int xt, int wt) {
    if (xt == MOMIJ_DTYPE_BF16)
        return wt == MOMIJ_DTYPE_BF16 ? gate_gemv_kernel<MOMIJ_DTYPE_BF16, MOMIJ_DTYPE_BF16>
                                      : gate_gemv_kernel<MOMIJ_DTYPE_BF16, MOMIJ_DTYPE_F16>;
    return wt == MOMIJ_DTYPE_BF16 ? gate_gemv_kernel<MOMIJ_DTYPE_F16, MOMIJ_DTYPE_BF16>
                                  : gate_gemv_kernel<MOMIJ_DTYPE_F16, MOMIJ_DTYPE_F16>;
}
RouterFn pick_router(int xt, int wt) {
    if (xt == MOMIJ_DTYPE_BF16)
        return wt == MOMIJ_DTYPE_BF16 ? fused_router_kernel<MOMIJ_DTYPE_BF16, MOMIJ_DTYPE_BF16>
                                      : fused_router_kernel<MOMIJ_DTYPE_BF16, MOMIJ_DTYPE_F16>;
    return wt == MOMIJ_DTYPE_BF16 ? fused_router_kernel<MOMIJ_DTYPE_F16, MOMIJ_DTYPE_BF16>
                                  : fused_router_kernel<MOMIJ_DTYPE_F16, MOMIJ_DTYPE_F16>;
}
bool dtype_ok(int dt) { return dt == MOMIJ_DTYPE_BF16 || dt == MOMIJ_DTYPE_F16; }
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int launch_gate(const void* x, const void* w, float* logits, int M, int H, int E, int xt, int wt,
                cudaStream_t st) {
    const int warps = 8;
    return cuda_status(launch(pick_gate(xt, wt), dim3((E + warps - 1) / warps, (M + 7) / 8), dim3(32 * warps), 0,
                              st, static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(w), logits, M, H,
                              E));
}
}  // namespace

int momij_moe_router_logits(const void* x, const void* w_gate, float* logits, int M, int H, int E,
                            int x_dtype, int w_dtype, momij_stream_t stream) {
    if (int rc = check_device()) return rc;
    if (!x || !w_gate || !logits || M < 0 || H < 1 || E < 1 || !dtype_ok(x_dtype) || !dtype_ok(w_dtype))
        return MOMIJ_ERR_INVALID_ARGUMENT;
    if (H % 256 || !aligned16(x) || !aligned16(w_gate)) return MOMIJ_ERR_UNSUPPORTED_SHAPE;
    if (M == 0) return MOMIJ_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int slot = prof_begin(MOMIJ_KERNEL_PLAN, st);
    const int rc = launch_gate(x, w_gate, logits, M, H, E, x_dtype, w_dtype, st);
    prof_end(slot, st);
    return rc;
}

int momij_moe_fused_router(const void* x, const void* w_gate, uint32_t* counter, float* logits,
                           int32_t* inds, float* scores, int M, int H, int E, int K, int x_dtype,
                           int w_dtype, momij_stream_t stream) {
    if (int rc = check_device()) return rc;
    if (!x || !w_gate || !counter || !logits || !inds || !scores || M < 0 || H < 1 || E < 1 || K < 1 ||
        !dtype_ok(x_dtype) || !dtype_ok(w_dtype))
        return MOMIJ_ERR_INVALID_ARGUMENT;
    if (H % 256 || E % 8 || K > 32 || K > E || M > 64 || E > 8192 || !aligned16(x) || !aligned16(w_gate))
        return MOMIJ_ERR_UNSUPPORTED_SHAPE;
    if (M == 0) return MOMIJ_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    RouterFn fn = pick_router(x_dtype, w_dtype);
    const size_t smem = sizeof(float) * (size_t)E;
    if (smem > 48 * 1024 && cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
                                cudaSuccess)
        return MOMIJ_ERR_CUDA;
    const int slot = prof_begin(MOMIJ_KERNEL_PLAN, st);
    const int rc = cuda_status(launch(fn, dim3(E / 8), dim3(256), smem, st, static_cast<const uint16_t*>(x),
                                      static_cast<const uint16_t*>(w_gate), reinterpret_cast<unsigned*>(counter),
                                      logits, inds, scores, M, H, E, K));
    prof_end(slot, st);
    return rc;
}

int momij_rms_norm(const void* x, const void* w, void* out, int M, int H, float eps, int dtype,
                   momij_stream_t stream) {
    if (int rc = check_device()) return rc;
    if (!x || !w || !out || M < 0 || H < 1 || !dtype_ok(dtype)) return MOMIJ_ERR_INVALID_ARGUMENT;
    if (M == 0) return MOMIJ_OK;
    auto fn = dtype == MOMIJ_DTYPE_BF16 ? rms_norm_kernel<MOMIJ_DTYPE_BF16> : rms_norm_kernel<MOMIJ_DTYPE_F16>;
    return cuda_status(launch(fn, dim3(M), dim3(256), 0, static_cast<cudaStream_t>(stream),
                              static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(w),
                              static_cast<uint16_t*>(out), H, eps));
}

size_t momij_moe_block_workspace_size(int M, int Ktop, int H, int I, int E) {
    if (M < 0 || Ktop < 1 || H < 0 || I < 0 || E < 1) return 0;
    return carve(nullptr, M, Ktop, H, I).bytes + align_up((size_t)M * H * 2, 256) + align_up((size_t)M * E * 4, 256);
}

int momij_moe_block(void* h, const void* norm_w, float eps, const void* w_gate, int gate_dtype,
                    const uint32_t* w_ug, const void* s_ug, const void* b_ug, const uint32_t* w_dn,
                    const void* s_dn, const void* b_dn, int32_t* inds, float* scores, int M, int H,
                    int I, int E, int Ktop, int gs, float clamp, int dtype, void* workspace,
                    size_t workspace_bytes, momij_stream_t stream) {
    if (int rc = check_device()) return rc;
    if (!h || !norm_w || !w_gate || !workspace || M < 0 || !dtype_ok(gate_dtype) || !dtype_ok(dtype))
        return MOMIJ_ERR_INVALID_ARGUMENT;
    if (M == 0) return MOMIJ_OK;
    if (workspace_bytes < momij_moe_block_workspace_size(M, Ktop, H, I, E)) return MOMIJ_ERR_WORKSPACE;
    if (H % 256 || !aligned16(h) || !aligned16(w_gate)) return MOMIJ_ERR_UNSUPPORTED_SHAPE;
    const size_t base = carve(nullptr, M, Ktop, H, I).bytes;
    unsigned char* tail = static_cast<unsigned char*>(workspace) + base;
    void* xn = tail;
    float* logits = reinterpret_cast<float*>(tail + align_up((size_t)M * H * 2, 256));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (int rc = momij_rms_norm(h, norm_w, xn, M, H, eps, dtype, stream)) return rc;
    int rc;
    {
        const int slot = prof_begin(MOMIJ_KERNEL_PLAN, st);
        rc = launch_gate(xn, w_gate, logits, M, H, E, dtype, gate_dtype, st);
        prof_end(slot, st);
    }
    if (rc) return rc;
    return momij_moe_forward(logits, xn, w_ug, s_ug, b_ug, w_dn, s_dn, b_dn, inds, scores, nullptr, h, M, H, I, E,
                             Ktop, gs, clamp, dtype, workspace, base, stream);
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
    int rc = launch_plan(inds, M * Ktop, E, tmax, plan, st, /*allow_pad=*/1);
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
    int rc = launch_plan(inds, M * Ktop, E, tmax, plan, st, /*allow_pad=*/1);
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
    if (!shape_ok(H, gs) || !shape_ok(I, gs) || (long long)M * Ktop > MOMIJ_MAX_GROUPED_PAIRS)
        return MOMIJ_ERR_UNSUPPORTED_SHAPE;
    if ((long long)M * Ktop > MOMIJ_MAX_PAIRS && (E > kGrpMaxExperts || I % 64 || H % 128))
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
    if (grouped_enabled(M, Ktop, E))
        return run_grouped(x, w_ug, s_ug, b_ug, w_dn, s_dn, b_dn, inds, scores, y, resid_h, M, H, I, E,
                           Ktop, gs, clamp, dtype, ws, st);
    const LayerCall lc{nullptr, inds, scores, nullptr, nullptr, x, w_ug, w_dn, s_ug, b_ug, s_dn, b_dn,
                       y, resid_h, M, H, I, E, Ktop, clamp};
    const int frc = run_fused_layer(lc, dtype, gs, ws, st);
    if (frc != kNotApplicable) return frc;
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
    if (grouped_enabled(M, Ktop, E)) {
        const int slot = prof_begin(MOMIJ_KERNEL_PLAN, st);
        const int warps = 8;
        int rc = cuda_status(launch(route_kernel, dim3((M + warps - 1) / warps), dim3(32 * warps), 0, st,
                                    logits, M, E, Ktop, ind_out, sc_out));
        prof_end(slot, st);
        if (rc) return rc;
        return run_grouped(x, w_ug, s_ug, b_ug, w_dn, s_dn, b_dn, ind_out, sc_out, y, resid_h, M, H, I,
                           E, Ktop, gs, clamp, dtype, ws, st);
    }
    const LayerCall lc{logits, nullptr, nullptr, ind_out, sc_out, x, w_ug, w_dn, s_ug, b_ug, s_dn, b_dn,
                       y, resid_h, M, H, I, E, Ktop, clamp};
    const int frc = run_fused_layer(lc, dtype, gs, ws, st);
    if (frc != kNotApplicable) return frc;
    const int tmax = tmax_for(M, Ktop, 0);
    const int slot = prof_begin(MOMIJ_KERNEL_PLAN, st);
    int rc;
    if (M <= 32) {  // one block routes every token (a warp each) and plans
        rc = cuda_status(launch(route_plan_kernel, dim3(1), dim3(1024), 0, st, logits, M, E, Ktop, tmax,
                                ind_out, sc_out, ws.plan));
    } else {  // many tokens: route on as many blocks as needed, then plan
        const int warps = 8;
        rc = cuda_status(launch(route_kernel, dim3((M + warps - 1) / warps), dim3(32 * warps), 0, st, logits, M,
                                E, Ktop, ind_out, sc_out));
        if (!rc)
            rc = cuda_status(launch(plan_kernel, dim3(1), dim3(1024), 0, st, static_cast<const int32_t*>(ind_out),
                                    M * Ktop, E, tmax, ws.plan, 0));
    }
    prof_end(slot, st);
    if (rc) return rc;
    return ffn_after_plan(x, w_ug, s_ug, b_ug, w_dn, s_dn, b_dn, sc_out, y, resid_h, M, H, I, E,
                          Ktop, gs, clamp, dtype, tmax, ws, st);
}

int momij_moe_ep_dispatch(const int32_t* inds, const void* x, int M, int K, int E, int world,
                          int capacity, int H, void* send_x, int32_t* send_meta, int32_t* slot_map,
                          int32_t* status, momij_stream_t stream) {
    if (int rc = check_device()) return rc;
    if (M < 0 || K < 1 || E < 1 || world < 1 || capacity < 0 || H < 8) return MOMIJ_ERR_INVALID_ARGUMENT;
    if (E % world || (long long)M * K > MOMIJ_MAX_PAIRS || (long long)M * K > capacity || H % 8)
        return MOMIJ_ERR_UNSUPPORTED_SHAPE;
    if (M == 0) return MOMIJ_OK;
    if (!inds || !x || !send_x || !send_meta || !slot_map || !status || !aligned(x, 16) ||
        !aligned(send_x, 16))
        return MOMIJ_ERR_INVALID_ARGUMENT;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int P = M * K;
    if (cudaMemsetAsync(status, 0, sizeof(int32_t), st) != cudaSuccess) return MOMIJ_ERR_CUDA;
    int rc = cuda_status(launch(ep_slots_kernel, dim3(1), dim3(1024), 0, st, inds, P, E, world, capacity,
                                send_meta, slot_map, status));
    if (rc) return rc;
    const int row16 = H / 8;
    const int blocks = (int)std::min<long long>(((long long)P * row16 + 255) / 256, 2048);
    return cuda_status(launch(ep_gather_kernel, dim3(blocks), dim3(256), 0, st,
                              static_cast<const uint4*>(x), static_cast<const int32_t*>(slot_map), P, K,
                              row16, static_cast<uint4*>(send_x)));
}

int momij_moe_ep_combine(const void* back, const float* scores, const int32_t* slot_map, void* y,
                         void* resid_h, int M, int K, int H, int dtype, const int32_t* status,
                         momij_stream_t stream) {
    if (int rc = check_device()) return rc;
    if (M < 0 || K < 1 || H < 1 || (dtype != MOMIJ_DTYPE_BF16 && dtype != MOMIJ_DTYPE_F16))
        return MOMIJ_ERR_INVALID_ARGUMENT;
    if (M == 0) return MOMIJ_OK;
    if (!back || !scores || !slot_map || !status || (!y && !resid_h)) return MOMIJ_ERR_INVALID_ARGUMENT;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const long long n = (long long)M * H;
    const int blocks = (int)std::min<long long>((n + 255) / 256, 4096);
    auto b = static_cast<const uint16_t*>(back);
    auto o = static_cast<uint16_t*>(resid_h ? resid_h : y);
    const bool r = resid_h != nullptr;
    if (dtype == MOMIJ_DTYPE_BF16)
        return cuda_status(r ? launch(ep_combine_kernel<MOMIJ_DTYPE_BF16, 1>, dim3(blocks), dim3(256), 0, st, b,
                                      scores, slot_map, o, M, K, H, status)
                             : launch(ep_combine_kernel<MOMIJ_DTYPE_BF16, 0>, dim3(blocks), dim3(256), 0, st, b,
                                      scores, slot_map, o, M, K, H, status));
    return cuda_status(r ? launch(ep_combine_kernel<MOMIJ_DTYPE_F16, 1>, dim3(blocks), dim3(256), 0, st, b,
                                  scores, slot_map, o, M, K, H, status)
                         : launch(ep_combine_kernel<MOMIJ_DTYPE_F16, 0>, dim3(blocks), dim3(256), 0, st, b,
                                  scores, slot_map, o, M, K, H, status));
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
