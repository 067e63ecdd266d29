// peer_merge.cu -- cross-GPU merge of split-KV partials over peer memory (NVLink P2P).
//
// Long-context decode splits each layer's keys across ranks; every rank holds a
// normalised partial (O_r, LSE_r) for the 16 x n_q query rows of a layer.  Instead of
// an all-gather followed by a merge (two steps, a collective library in between), the
// ranks push their partials into each other's peer buffers with tagged 8-byte stores
// and merge as soon as every peer's words carry the expected tag (peer.cuh has the
// buffer layout and the protocol; the decode entry point sqmix_fa_decode_peers runs
// the same exchange inside its split merge).  Here the partials come from the caller
// (o_local, lse_local): out = sum_r O_r e^{LSE_r - L} * sigmoid(gate).
// No TMA, no multicast: plain stores to peer memory, loads of local memory, bounded
// spins.
#include <cuda_runtime.h>
#include <math.h>

#include <cstring>

#include "common.cuh"
#include "peer.cuh"
#include "sqmix.h"

namespace sqmix {
namespace {

struct PeerMergeParams {
    PeerExchange px;
    const float *o_local;  // [rows][256]
    const float *lse_local;
    const float *gate;     // nullable [rows][256] f32
    float *out;            // [rows][256]
    float *lse_out;        // nullable [rows]
};

// grid (rows, kPeerSlices), 256 threads: the first warp holds dims slice * 32 + lane
__global__ void __launch_bounds__(256) peer_merge_kernel(PeerMergeParams p) {
    const int row = blockIdx.x, sl = blockIdx.y, t = threadIdx.x;
    // programmatic dependent launch: the partial comes from the kernel before this one
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" :::);
    float y_loc = 0.f, lse_loc = 0.f;
    if (t < 32) {
        y_loc = p.o_local[row * 256 + sl * 32 + t];
        lse_loc = p.lse_local[row];
    }
    float y = 0.f, lse = 0.f;
    if (!peer_exchange(p.px, row, sl, y_loc, lse_loc, kWaitLimitNs, y, lse)) return;
    if (t < 32) {
        const int col = sl * 32 + t;
        if (p.gate) y *= 1.f / (1.f + __expf(-p.gate[row * 256 + col]));
        p.out[row * 256 + col] = y;
        if (p.lse_out && sl == 0 && t == 0) p.lse_out[row] = lse;
    }
}

}  // namespace
}  // namespace sqmix

using namespace sqmix;

extern "C" size_t sqmix_peer_buffer_bytes(int32_t n_slots) {
    if (n_slots < 1) return 0;
    return peer_layout(n_slots).total;
}

extern "C" int sqmix_peer_buffer_reset(void *dev_ptr, int32_t n_slots, sqmix_stream_t stream) {
    SQMIX_CHECK_ARG(dev_ptr && n_slots >= 1 && n_slots <= 4096, "peer_buffer_reset: bad arguments (n_slots=%d)",
                    n_slots);
    return cuda_status(cudaMemsetAsync(dev_ptr, 0, peer_layout(n_slots).total, reinterpret_cast<cudaStream_t>(stream)),
                       "peer_buffer_reset");
}

extern "C" int sqmix_peer_buffer_create(int32_t n_slots, void **dev_ptr, void *ipc_handle) {
    SQMIX_CHECK_ARG(dev_ptr && ipc_handle && n_slots >= 1 && n_slots <= 4096,
                    "peer_buffer_create: bad arguments (n_slots=%d)", n_slots);
    static_assert(sizeof(cudaIpcMemHandle_t) <= SQMIX_IPC_HANDLE_BYTES, "IPC handle size");
    const size_t bytes = peer_layout(n_slots).total;
    void *p = nullptr;
    int rc = cuda_status(cudaMalloc(&p, bytes), "peer_buffer_create: cudaMalloc");
    if (rc == SQMIX_OK) rc = cuda_status(cudaMemset(p, 0, bytes), "peer_buffer_create: memset");
    cudaIpcMemHandle_t h;
    if (rc == SQMIX_OK) rc = cuda_status(cudaIpcGetMemHandle(&h, p), "peer_buffer_create: cudaIpcGetMemHandle");
    if (rc != SQMIX_OK) {
        if (p) cudaFree(p);
        return rc;
    }
    memset(ipc_handle, 0, SQMIX_IPC_HANDLE_BYTES);
    memcpy(ipc_handle, &h, sizeof(h));
    *dev_ptr = p;
    return SQMIX_OK;
}

extern "C" int sqmix_peer_buffer_open(const void *ipc_handle, void **peer_ptr) {
    SQMIX_CHECK_ARG(ipc_handle && peer_ptr, "peer_buffer_open: null argument");
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof(h));
    void *p = nullptr;
    const int rc = cuda_status(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess),
                               "peer_buffer_open: cudaIpcOpenMemHandle");
    if (rc == SQMIX_OK) *peer_ptr = p;
    return rc;
}

extern "C" int sqmix_peer_buffer_close(void *peer_ptr) {
    SQMIX_CHECK_ARG(peer_ptr, "peer_buffer_close: null pointer");
    return cuda_status(cudaIpcCloseMemHandle(peer_ptr), "peer_buffer_close");
}

extern "C" int sqmix_peer_buffer_destroy(void *dev_ptr) {
    SQMIX_CHECK_ARG(dev_ptr, "peer_buffer_destroy: null pointer");
    return cuda_status(cudaFree(dev_ptr), "peer_buffer_destroy");
}

extern "C" int sqmix_attn_merge_peers(const sqmix_peer_merge_args *a, sqmix_stream_t stream) {
    SQMIX_CHECK_ARG(a != nullptr, "attn_merge_peers: null args");
    SQMIX_CHECK_ARG(a->n_ranks >= 1 && a->n_ranks <= kPeerMaxRanks && a->rank >= 0 && a->rank < a->n_ranks,
                    "attn_merge_peers: rank %d of %d (at most %d ranks)", a->rank, a->n_ranks, kPeerMaxRanks);
    SQMIX_CHECK_ARG(a->rows >= 1 && a->rows <= kPeerMaxRows, "attn_merge_peers: rows=%d (1..%d)", a->rows,
                    kPeerMaxRows);
    SQMIX_CHECK_ARG(a->n_slots >= 1 && a->n_slots <= 4096 && a->slot >= 0 && a->slot < a->n_slots,
                    "attn_merge_peers: slot %d of %d", a->slot, a->n_slots);
    SQMIX_CHECK_ARG(a->buffers && a->o_local && a->lse_local && a->out, "attn_merge_peers: null pointer argument");
    PeerMergeParams p;
    p.px.n_ranks = a->n_ranks;
    p.px.rank = a->rank;
    p.px.slot = a->slot;
    p.px.n_slots = a->n_slots;
    p.px.bufs = const_cast<uint8_t *const *>(reinterpret_cast<const uint8_t *const *>(a->buffers));
    p.px.status = static_cast<uint32_t *>(a->status);
    p.o_local = a->o_local;
    p.lse_local = a->lse_local;
    p.gate = a->gate;
    p.out = a->out;
    p.lse_out = a->lse_out;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a->rows, kPeerSlices);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = reinterpret_cast<cudaStream_t>(stream);
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_status(cudaLaunchKernelEx(&cfg, peer_merge_kernel, p), "attn_merge_peers launch");
}
