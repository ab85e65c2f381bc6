// noalloc.cu -- momij_moe_gqmm2_noalloc: the gather-GEMV for callers that
// cannot allocate device memory.
//
// Who needs it: a caller that owns only its inputs and outputs and has no
// device allocator to hand -- e.g. a foreign-language binding that receives
// already-resident buffers, or a serving engine that reserves all device
// memory at start-up and forbids allocation inside its token loop (a
// cudaMalloc there can synchronize the device and stall the pipeline).
// momij_moe_gqmm2 needs a caller-provided workspace for its work plan; this
// variant keeps that plan in a fixed array compiled into the library instead,
// so the call performs no cudaMalloc, cudaFree or other allocation.
//
// Costs and rules of the fixed array:
//   * it is g_noalloc_plan below, sized for MOMIJ_NOALLOC_MAX_PAIRS pairs
//     (20,736 bytes); every GPU that loads the library holds it until the
//     process exits;
//   * every call shares it and it keeps the last call's contents; the plan
//     kernel rewrites every field the GEMV reads at the start of each call, so
//     nothing has to be cleared between calls, but calls whose execution
//     overlaps on the GPU (different streams, or devices sharing the same
//     context) race on it -- serialise them;
//   * the device address of the array is looked up once per device, on that
//     device's first call, with cudaGetSymbolAddress; make that first call
//     before any stream capture on that device.
#include <mutex>

#include "kernels.cuh"

namespace {

// Bytes of a work plan for MOMIJ_NOALLOC_MAX_PAIRS pairs: header + 4 ints per
// unit + 1 int per pair, rounded up to 256 (the layout the plan kernel writes).
constexpr size_t kNoAllocPlanBytes =
    ((sizeof(int32_t) * (momij::kPlanHeader + 5 * (size_t)MOMIJ_NOALLOC_MAX_PAIRS) + 255) / 256) * 256;

static __device__ __align__(256) int32_t g_noalloc_plan[kNoAllocPlanBytes / sizeof(int32_t)];

std::mutex g_noalloc_mu;
void* g_noalloc_addr[64] = {};

// The host-side name g_noalloc_plan is only a stand-in for the symbol; the
// kernels get the device address, fetched here for the current device.
int noalloc_plan_address(void** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MOMIJ_ERR_CUDA;
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_plan) != cudaSuccess || !p) {
            cudaGetLastError();
            return MOMIJ_ERR_CUDA;
        }
        g_noalloc_addr[dev] = p;
    }
    *out = g_noalloc_addr[dev];
    return MOMIJ_OK;
}

}  // namespace

extern "C" int momij_moe_gqmm2_noalloc(const void* x, const uint32_t* w, const void* scales,
                                       const void* biases, const int32_t* inds, void* out, int M,
                                       int Ktop, int Kdim, int N, int E, int gs, int lhs_per_expert,
                                       int dtype, momij_stream_t stream) {
    if (M < 0 || Ktop < 1) return MOMIJ_ERR_INVALID_ARGUMENT;
    if ((long long)M * Ktop > MOMIJ_NOALLOC_MAX_PAIRS) return MOMIJ_ERR_WORKSPACE;
    if (M == 0) return MOMIJ_OK;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        return MOMIJ_ERR_NO_DEVICE;
    }
    void* plan = nullptr;
    if (int rc = noalloc_plan_address(&plan)) return rc;
    return momij_moe_gqmm2(x, w, scales, biases, inds, out, M, Ktop, Kdim, N, E, gs,
                           lhs_per_expert, dtype, plan, kNoAllocPlanBytes, stream);
}
