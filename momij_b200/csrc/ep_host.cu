// ep_host.cu -- the expert-parallel layer behind the C ABI (momij_moe_ep_*):
// one object per rank holds the communicator and the exchange buffers, and
// momij_moe_ep_forward enqueues a whole layer on the caller's stream:
//
//   route (or the caller's inds/scores) -> momij_moe_ep_dispatch (fixed
//   capacity rows per destination; the destination's local expert indices in
//   one extra row of its segment) -> grouped ncclSend/ncclRecv of the
//   segments -> the rank's experts over the received rows (gqmm2_up_swiglu +
//   gqmm2 with Ktop = 1; empty rows carry expert -1 and are skipped) ->
//   grouped send/recv of the outputs -> momij_moe_ep_combine into y or the
//   residual stream.
//
// No counts travel to the host, so a layer needs no device-to-host
// synchronisation and can be captured in a CUDA graph.  NCCL is resolved at
// run time (dlopen of libnccl.so.2, preferring the copy the process already
// loaded, e.g. PyTorch's), so the library itself does not link NCCL.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "momij_moe.h"

struct momij_ep {
    ncclComm_t comm = nullptr;
    bool own_comm = false;
    int rank = 0, world = 1, E = 0, H = 0, I = 0, K = 0, max_tokens = 0, gs = 64, dtype = 0;
    float clamp = 7.0f;
    int cap = 0, seg = 0, rows = 0;  // pair rows per destination, + the index row, all rows
    int32_t *inds = nullptr, *slot_map = nullptr, *status = nullptr, *send_meta = nullptr, *recv_meta = nullptr;
    float* scores = nullptr;
    uint16_t *send_x = nullptr, *recv_x = nullptr, *act = nullptr, *down = nullptr, *back = nullptr;
    void* ws = nullptr;
    size_t ws_bytes = 0;
};

namespace {

struct Nccl {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    bool ok = false;
};

const Nccl& nccl() {
    static Nccl n;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        n.GetUniqueId = reinterpret_cast<decltype(n.GetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
        n.CommInitRank = reinterpret_cast<decltype(n.CommInitRank)>(dlsym(h, "ncclCommInitRank"));
        n.CommDestroy = reinterpret_cast<decltype(n.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
        n.GroupStart = reinterpret_cast<decltype(n.GroupStart)>(dlsym(h, "ncclGroupStart"));
        n.GroupEnd = reinterpret_cast<decltype(n.GroupEnd)>(dlsym(h, "ncclGroupEnd"));
        n.Send = reinterpret_cast<decltype(n.Send)>(dlsym(h, "ncclSend"));
        n.Recv = reinterpret_cast<decltype(n.Recv)>(dlsym(h, "ncclRecv"));
        n.ok = n.GetUniqueId && n.CommInitRank && n.CommDestroy && n.GroupStart && n.GroupEnd && n.Send && n.Recv;
    });
    return n;
}

template <typename T>
bool dev_alloc(T** p, size_t n) {
    return cudaMalloc(reinterpret_cast<void**>(p), n * sizeof(T) > 0 ? n * sizeof(T) : 16) == cudaSuccess;
}

void release(momij_ep* ep) {
    void* bufs[] = {ep->inds, ep->slot_map, ep->status, ep->send_meta, ep->recv_meta, ep->scores, ep->send_x,
                    ep->act, ep->down, ep->ws};
    for (void* b : bufs)
        if (b) cudaFree(b);
    if (ep->world > 1) {
        if (ep->recv_x) cudaFree(ep->recv_x);
        if (ep->back) cudaFree(ep->back);
    }
    if (ep->own_comm && ep->comm) nccl().CommDestroy(ep->comm);
    delete ep;
}

// Segment exchange: rank r sends segment d of `send` to rank d and receives
// rank d's segment r into segment d of `recv` (seg_bytes each).
int exchange(const momij_ep* ep, const void* send, void* recv, size_t seg_bytes, cudaStream_t st) {
    const Nccl& n = nccl();
    if (n.GroupStart() != ncclSuccess) return MOMIJ_ERR_NCCL;
    for (int d = 0; d < ep->world; ++d) {
        const char* s = static_cast<const char*>(send) + (size_t)d * seg_bytes;
        char* r = static_cast<char*>(recv) + (size_t)d * seg_bytes;
        if (n.Send(s, seg_bytes, ncclUint8, d, ep->comm, st) != ncclSuccess ||
            n.Recv(r, seg_bytes, ncclUint8, d, ep->comm, st) != ncclSuccess) {
            n.GroupEnd();
            return MOMIJ_ERR_NCCL;
        }
    }
    return n.GroupEnd() == ncclSuccess ? MOMIJ_OK : MOMIJ_ERR_NCCL;
}

}  // namespace

extern "C" {

int momij_nccl_unique_id(void* out) {
    if (!out) return MOMIJ_ERR_INVALID_ARGUMENT;
    const Nccl& n = nccl();
    if (!n.ok) return MOMIJ_ERR_NCCL;
    ncclUniqueId id;
    if (n.GetUniqueId(&id) != ncclSuccess) return MOMIJ_ERR_NCCL;
    std::memcpy(out, &id, sizeof(id));
    return MOMIJ_OK;
}

int momij_moe_ep_init(void* nccl_comm, const void* unique_id, int rank, int world, int E, int H, int I, int K,
                      int max_tokens, int gs, float clamp, int dtype, momij_ep_t** out) {
    if (!out || world < 1 || rank < 0 || rank >= world || E < 1 || H < 1 || I < 1 || K < 1 || max_tokens < 1 ||
        (dtype != MOMIJ_DTYPE_BF16 && dtype != MOMIJ_DTYPE_F16) || (!nccl_comm && !unique_id && world > 1))
        return MOMIJ_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    int dev_count = 0;
    if (cudaGetDeviceCount(&dev_count) != cudaSuccess || dev_count == 0) return MOMIJ_ERR_NO_DEVICE;
    // experts split evenly; the index row holds a segment's expert indices as
    // 32-bit words (seg <= H / 2); the experts step runs on world * seg rows
    // with one slot each (<= MOMIJ_MAX_PAIRS)
    const int cap = max_tokens * K, seg = cap + 1;
    if (E % world || seg > H / 2 || (long long)world * seg > MOMIJ_MAX_PAIRS) return MOMIJ_ERR_UNSUPPORTED_SHAPE;
    momij_ep* ep = new momij_ep();
    ep->rank = rank;
    ep->world = world;
    ep->E = E;
    ep->H = H;
    ep->I = I;
    ep->K = K;
    ep->max_tokens = max_tokens;
    ep->gs = gs;
    ep->clamp = clamp;
    ep->dtype = dtype;
    ep->cap = cap;
    ep->seg = seg;
    ep->rows = world * seg;
    if (nccl_comm) {
        ep->comm = *static_cast<ncclComm_t*>(nccl_comm);
    } else if (world > 1 || unique_id) {
        const Nccl& n = nccl();
        if (!n.ok) {
            delete ep;
            return MOMIJ_ERR_NCCL;
        }
        ncclUniqueId id;
        std::memcpy(&id, unique_id, sizeof(id));
        if (n.CommInitRank(&ep->comm, world, id, rank) != ncclSuccess) {
            delete ep;
            return MOMIJ_ERR_NCCL;
        }
        ep->own_comm = true;
    }
    const size_t rows = ep->rows;
    bool ok = dev_alloc(&ep->inds, (size_t)cap) && dev_alloc(&ep->scores, (size_t)cap) &&
              dev_alloc(&ep->slot_map, (size_t)cap) && dev_alloc(&ep->status, 1) &&
              dev_alloc(&ep->send_meta, rows) && dev_alloc(&ep->recv_meta, rows) &&
              dev_alloc(&ep->send_x, rows * H) && dev_alloc(&ep->act, rows * I) && dev_alloc(&ep->down, rows * H);
    if (ok && world > 1) ok = dev_alloc(&ep->recv_x, rows * H) && dev_alloc(&ep->back, rows * H);
    if (ok && world == 1) {  // nothing to exchange: the receive side is the send side
        ep->recv_x = ep->send_x;
        ep->back = ep->down;
    }
    ep->ws_bytes = momij_moe_workspace_size((int)rows, 1, 0, 0);
    ok = ok && cudaMalloc(&ep->ws, ep->ws_bytes) == cudaSuccess && cudaMemset(ep->ws, 0, ep->ws_bytes) == cudaSuccess &&
         cudaMemset(ep->status, 0, 4) == cudaSuccess && cudaMemset(ep->send_x, 0, rows * H * 2) == cudaSuccess &&
         cudaMemset(ep->act, 0, rows * I * 2) == cudaSuccess && cudaMemset(ep->down, 0, rows * H * 2) == cudaSuccess;
    if (!ok) {
        release(ep);
        return MOMIJ_ERR_CUDA;
    }
    *out = ep;
    return MOMIJ_OK;
}

int momij_moe_ep_forward(momij_ep_t* ep, const float* logits, const int32_t* inds, const float* scores,
                         const void* x, const uint32_t* w_ug, const void* s_ug, const void* b_ug,
                         const uint32_t* w_dn, const void* s_dn, const void* b_dn, void* y, void* resid_h, int M,
                         momij_stream_t stream) {
    if (!ep || !x || !w_ug || !s_ug || !b_ug || !w_dn || !s_dn || !b_dn || (!y && !resid_h) || M < 0 ||
        (!logits && (!inds || !scores)))
        return MOMIJ_ERR_INVALID_ARGUMENT;
    if (M > ep->max_tokens) return MOMIJ_ERR_UNSUPPORTED_SHAPE;
    if (M == 0) return MOMIJ_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int K = ep->K, H = ep->H, I = ep->I, E = ep->E, w = ep->world, seg = ep->seg, cap = ep->cap;
    int rc;
    const int32_t* ind = inds;
    const float* sc = scores;
    if (logits) {
        if ((rc = momij_moe_route(logits, M, E, K, ep->inds, ep->scores, stream))) return rc;
        ind = ep->inds;
        sc = ep->scores;
    }
    if ((rc = momij_moe_ep_dispatch(ind, x, M, K, E, w, seg, H, ep->send_x, ep->send_meta, ep->slot_map,
                                    ep->status, stream)))
        return rc;
    const size_t row_bytes = (size_t)H * 2, seg_bytes = (size_t)seg * row_bytes;
    if (w > 1) {
        // the segment's expert indices ride in its last row (slot cap, always empty)
        if (cudaMemcpy2DAsync(reinterpret_cast<char*>(ep->send_x) + (size_t)cap * row_bytes, seg_bytes, ep->send_meta,
                              (size_t)seg * 4, (size_t)seg * 4, w, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
            return MOMIJ_ERR_CUDA;
        if ((rc = exchange(ep, ep->send_x, ep->recv_x, seg_bytes, st))) return rc;
        if (cudaMemcpy2DAsync(ep->recv_meta, (size_t)seg * 4,
                              reinterpret_cast<const char*>(ep->recv_x) + (size_t)cap * row_bytes, seg_bytes,
                              (size_t)seg * 4, w, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
            return MOMIJ_ERR_CUDA;
    }
    const int32_t* meta = w > 1 ? ep->recv_meta : ep->send_meta;
    const int El = E / w;
    if ((rc = momij_moe_gqmm2_up_swiglu(ep->recv_x, w_ug, s_ug, b_ug, meta, ep->act, ep->rows, 1, H, I, El, ep->gs,
                                        ep->clamp, ep->dtype, ep->ws, ep->ws_bytes, stream)))
        return rc;
    if ((rc = momij_moe_gqmm2(ep->act, w_dn, s_dn, b_dn, meta, ep->down, ep->rows, 1, I, H, El, ep->gs, 0,
                              ep->dtype, ep->ws, ep->ws_bytes, stream)))
        return rc;
    if (w > 1 && (rc = exchange(ep, ep->down, ep->back, seg_bytes, st))) return rc;
    return momij_moe_ep_combine(ep->back, sc, ep->slot_map, y, resid_h, M, K, H, ep->dtype, ep->status, stream);
}

int momij_moe_ep_status(momij_ep_t* ep, momij_stream_t stream) {
    if (!ep) return MOMIJ_ERR_INVALID_ARGUMENT;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cudaStreamSynchronize(st) != cudaSuccess) return MOMIJ_ERR_CUDA;
    int32_t s = 0;
    if (cudaMemcpy(&s, ep->status, 4, cudaMemcpyDeviceToHost) != cudaSuccess) return MOMIJ_ERR_CUDA;
    if (s != MOMIJ_OK) return s;
    return momij_moe_synchronize(stream, ep->ws);
}

int momij_moe_ep_destroy(momij_ep_t* ep) {
    if (!ep) return MOMIJ_ERR_INVALID_ARGUMENT;
    cudaDeviceSynchronize();
    release(ep);
    return MOMIJ_OK;
}

}  // extern "C"
