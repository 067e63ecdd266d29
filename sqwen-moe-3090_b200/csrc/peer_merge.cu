// peer_merge.cu -- cross-GPU merge of split-KV partials over peer memory (NVLink P2P).
//
// Long-context decode splits each layer's keys across ranks; every rank holds a
// normalised partial (O_r, LSE_r) for the 16 x n_q query rows of a layer.  Instead of
// an all-gather followed by a merge (two steps, a collective library in between), one
// kernel per rank publishes its partial into its own peer-visible buffer, raises a
// flag, waits (bounded) for the same flag of every peer and reads the peers' partials
// directly with P2P loads, merging as it goes (out = sum_r O_r e^{LSE_r - L} * gate).
//
// Buffer of a rank (cudaMalloc'ed here, exported with cudaIpcGetMemHandle, mapped by
// the other ranks with cudaIpcOpenMemHandle):
//   [slot][parity 2][rows][257 f32]   published partials (O row, then LSE)
//   [slot][kMaxCtas]  u32             publish flags (count of publications)
//   [slot][kMaxCtas]  u32             local counters (never read by peers)
// A CTA handles one (row, 64-column slice) and owns flag [slot][cta]: publication c
// of a slot goes to parity c & 1 and sets the flag to c; readers wait for flag >= c.
// Double buffering by parity makes reuse safe: a rank publishes c + 2 only after it
// consumed every peer's c + 1, which each peer publishes after it finished reading c.
// No TMA, no multicast: plain stores and loads of peer memory, bounded spins.
#include <cuda_runtime.h>
#include <math.h>

#include <cstring>

#include "common.cuh"
#include "sqmix.h"

namespace sqmix {
namespace {

constexpr int kRowF = 257;      // floats per published row: 256 O + LSE
constexpr int kSlices = 4;      // 64-column slices per row
constexpr int kMaxCtas = 32 * kSlices;  // rows <= 32 (n_q <= 2)

struct PeerLayout {
    size_t data_bytes_per_slot;
    size_t data_bytes, flags_off, counters_off, total;
};
__host__ __device__ inline PeerLayout peer_layout(int n_slots) {
    PeerLayout L;
    L.data_bytes_per_slot = static_cast<size_t>(2) * 32 * kRowF * sizeof(float);
    L.data_bytes = L.data_bytes_per_slot * n_slots;
    L.flags_off = (L.data_bytes + 255) / 256 * 256;
    L.counters_off = L.flags_off + static_cast<size_t>(n_slots) * kMaxCtas * sizeof(uint32_t);
    L.total = L.counters_off + static_cast<size_t>(n_slots) * kMaxCtas * sizeof(uint32_t);
    return L;
}

struct PeerMergeParams {
    int n_ranks, rank, slot, n_slots, rows;
    uint8_t *const *bufs;  // device array [n_ranks]: every rank's buffer as mapped here
    const float *o_local;  // [rows][256]
    const float *lse_local;
    const float *gate;     // nullable [rows][256] f32
    float *out;            // [rows][256]
    float *lse_out;        // nullable [rows]
    uint32_t *err;         // nullable status word
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// grid (rows, kSlices), 64 threads: thread = column of the slice
__global__ void __launch_bounds__(64) peer_merge_kernel(PeerMergeParams p) {
    const int row = blockIdx.x, sl = blockIdx.y, t = threadIdx.x;
    const int cta = row * kSlices + sl;
    const int col = sl * 64 + t;
    const PeerLayout L = peer_layout(p.n_slots);
    uint8_t *own = p.bufs[p.rank];
    uint32_t *flag = reinterpret_cast<uint32_t *>(own + L.flags_off) + p.slot * kMaxCtas + cta;
    uint32_t *count = reinterpret_cast<uint32_t *>(own + L.counters_off) + p.slot * kMaxCtas + cta;
    __shared__ uint32_t s_c;
    __shared__ int s_ok;
    // programmatic dependent launch: the partial comes from the kernel before this one
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" :::);
    if (t == 0) s_c = *count + 1;
    __syncthreads();
    const uint32_t c = s_c;
    const size_t data_off = p.slot * L.data_bytes_per_slot +
                            (static_cast<size_t>(c & 1) * 32 + row) * kRowF * sizeof(float);
    // publish this CTA's slice of the local partial (and the row's LSE from slice 0)
    float *mine = reinterpret_cast<float *>(own + data_off);
    const float o_me = p.o_local[row * 256 + col];
    const float l_me = p.lse_local[row];
    mine[col] = o_me;
    if (sl == 0 && t == 0) mine[256] = l_me;
    // the CTA barrier orders every thread's stores before thread 0's release of the
    // flag at system scope (cumulativity), so peers that acquire the flag see the data
    __syncthreads();
    if (t == 0) {
        st_release_sys(flag, c);
        *count = c;
    }
    // wait for every peer's publication c of this slice (bounded), one thread per peer
    if (t == 0) s_ok = 1;
    __syncthreads();
    if (t < p.n_ranks && t != p.rank) {
        const uint32_t *pf = reinterpret_cast<const uint32_t *>(p.bufs[t] + L.flags_off) + p.slot * kMaxCtas + cta;
        bool ok = ld_acquire_sys(pf) >= c;
        if (!ok) {
            const uint64_t t0 = globaltimer_ns();
            while (!(ok = ld_acquire_sys(pf) >= c)) {
                if (globaltimer_ns() - t0 > kWaitLimitNs) break;
            }
        }
        if (!ok) {
            s_ok = 0;
            if (p.err) atomicOr(p.err, 1u);
        }
    }
    __syncthreads();
    if (!s_ok) return;
    // merge: every peer's LSE and column are loaded at once (one NVLink round trip)
    float lse_r[8], o_r[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
        if (r < p.n_ranks) {
            const float *pr = reinterpret_cast<const float *>(p.bufs[r] + data_off);
            lse_r[r] = r == p.rank ? l_me : __ldcv(pr + 256);
            o_r[r] = r == p.rank ? o_me : __ldcv(pr + col);
        } else {
            lse_r[r] = -INFINITY;
            o_r[r] = 0.f;
        }
    }
    float M = -INFINITY;
#pragma unroll
    for (int r = 0; r < 8; ++r) M = fmaxf(M, lse_r[r]);
    float acc = 0.f, Ls = 0.f;
    if (M > -INFINITY) {
#pragma unroll
        for (int r = 0; r < 8; ++r) {
            if (lse_r[r] == -INFINITY) continue;
            const float w = __expf(lse_r[r] - M);
            acc = fmaf(o_r[r], w, acc);
            Ls += w;
        }
    }
    float y = Ls > 0.f ? acc / Ls : 0.f;
    if (p.gate) y *= 1.f / (1.f + __expf(-p.gate[row * 256 + col]));
    p.out[row * 256 + col] = y;
    if (p.lse_out && sl == 0 && t == 0) p.lse_out[row] = Ls > 0.f ? M + logf(Ls) : -INFINITY;
}

}  // namespace
}  // namespace sqmix

using namespace sqmix;

extern "C" size_t sqmix_peer_buffer_bytes(int32_t n_slots) {
    if (n_slots < 1) return 0;
    return peer_layout(n_slots).total;
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
    SQMIX_CHECK_ARG(a->n_ranks >= 1 && a->n_ranks <= 8 && a->rank >= 0 && a->rank < a->n_ranks,
                    "attn_merge_peers: rank %d of %d (at most 8 ranks)", a->rank, a->n_ranks);
    SQMIX_CHECK_ARG(a->rows >= 1 && a->rows <= 32, "attn_merge_peers: rows=%d (1..32)", a->rows);
    SQMIX_CHECK_ARG(a->n_slots >= 1 && a->slot >= 0 && a->slot < a->n_slots, "attn_merge_peers: slot %d of %d",
                    a->slot, a->n_slots);
    SQMIX_CHECK_ARG(a->buffers && a->o_local && a->lse_local && a->out, "attn_merge_peers: null pointer argument");
    PeerMergeParams p;
    p.n_ranks = a->n_ranks;
    p.rank = a->rank;
    p.slot = a->slot;
    p.n_slots = a->n_slots;
    p.rows = a->rows;
    p.bufs = const_cast<uint8_t *const *>(reinterpret_cast<const uint8_t *const *>(a->buffers));
    p.o_local = a->o_local;
    p.lse_local = a->lse_local;
    p.gate = a->gate;
    p.out = a->out;
    p.lse_out = a->lse_out;
    p.err = static_cast<uint32_t *>(a->status);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a->rows, kSlices);
    cfg.blockDim = dim3(64);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = reinterpret_cast<cudaStream_t>(stream);
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_status(cudaLaunchKernelEx(&cfg, peer_merge_kernel, p), "attn_merge_peers launch");
}
