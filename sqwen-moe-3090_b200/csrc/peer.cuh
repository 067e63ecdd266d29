// peer.cuh -- layout of the peer buffers through which split-KV ranks exchange their
// (O, LSE) partials (sqmix_attn_merge_peers, sqmix_fa_decode_peers).
//
// Every rank owns one buffer (cudaMalloc'ed, exported by IPC handle, mapped by the
// other ranks).  Ranks PUSH: a rank writes its partial into every other rank's buffer
// with plain 8-byte stores over NVLink and each receiver waits on its own local memory.
// Each 8-byte word carries a 32-bit value and a 32-bit publication tag, written by one
// single-copy-atomic store, so a receiver that sees the expected tag in a word also
// sees that word's value: no flag, no fence, no remote polling (the low-latency
// protocol of collective libraries).
//
//   data     [slot][parity 2][src rank 8][row 32][slice 8][33] u64
//            word j < 32: dim slice*32 + j of row `row` of src's normalised O;
//            word 32: the row's LSE (natural log); high 32 bits: the tag
//   counters [slot][row 32 * slice 8] u32, read and written only by the owning rank
//
// Publication c (1, 2, ...) of a slot goes to parity c & 1 with tag c.  A rank writes
// publication c + 2 of a slot only after it has read every peer's publication c + 1 of
// that slot, which each peer writes after it has finished reading publication c: so a
// parity buffer is never overwritten while its previous publication is being read.
// A zeroed buffer holds no publication (tags start at 1).
#pragma once

#include <stddef.h>
#include <stdint.h>

namespace sqmix {

constexpr int kPeerMaxRanks = 8;
constexpr int kPeerMaxRows = 32;   // 16 heads x n_q <= 2
constexpr int kPeerSlices = 8;     // 32-dim slices per 256-dim row
constexpr int kPeerWords = 33;     // 32 dims + LSE per (row, slice)

struct PeerLayout {
    size_t slot_words;   // u64 words of one slot (both parities)
    size_t data_bytes;
    size_t counters_off;
    size_t total;
};

__host__ __device__ inline PeerLayout peer_layout(int n_slots) {
    PeerLayout L;
    L.slot_words = static_cast<size_t>(2) * kPeerMaxRanks * kPeerMaxRows * kPeerSlices * kPeerWords;
    L.data_bytes = L.slot_words * sizeof(uint64_t) * static_cast<size_t>(n_slots);
    L.counters_off = (L.data_bytes + 255) / 256 * 256;
    L.total = L.counters_off + static_cast<size_t>(n_slots) * kPeerMaxRows * kPeerSlices * sizeof(uint32_t);
    return L;
}

// Word index of (slot, parity, src, row, slice, j) in the data area.
__host__ __device__ inline size_t peer_word(const PeerLayout &L, int slot, uint32_t parity, int src, int row,
                                            int slice, int j) {
    return static_cast<size_t>(slot) * L.slot_words +
           ((((static_cast<size_t>(parity) * kPeerMaxRanks + src) * kPeerMaxRows + row) * kPeerSlices + slice) *
                kPeerWords +
            j);
}

#ifdef __CUDACC__
// One 8-byte store of {value, tag}: single-copy atomic, visible to the receiver whole.
__device__ __forceinline__ void peer_put(uint64_t *w, float v, uint32_t tag) {
    asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(w), "r"(__float_as_uint(v)), "r"(tag)
                 : "memory");
}
__device__ __forceinline__ uint2 peer_get(const uint64_t *w) {
    uint2 r;
    asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(w) : "memory");
    return r;
}
#endif

}  // namespace sqmix

#ifdef __CUDACC__
namespace sqmix {

struct PeerExchange {
    int n_ranks, rank, slot, n_slots;
    uint8_t *const *bufs;  // device array [n_ranks]: every rank's buffer as mapped here
    uint32_t *status;      // nullable: bit 1 set when a wait for a peer gave up
};

__device__ __forceinline__ uint64_t peer_globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// The exchange of one (row, 32-dim slice) of the split-KV result, by a CTA of two or
// more warps.  Warp 0's lanes hold this rank's normalised partial for dims slice*32 +
// lane in y_loc and the row's LSE in lse_loc.  Pushes them into every other rank's
// buffer, waits (bounded by wait_ns; warps 1.. poll the peers' words in turn, in this
// rank's own memory) for every peer's publication of the same slot, and merges: y = sum_r O_r e^{lse_r - L},
// lse = L = log sum_r e^{lse_r} (natural log).  Returns, in warp 0, whether every peer
// arrived; on a timeout it sets bit 1 of *status and the caller writes nothing.
// Every rank calls this once per slot per step, for the same (row, slice) grid.
__device__ inline bool peer_exchange(const PeerExchange &px, int row, int slice, float y_loc, float lse_loc,
                                     uint64_t wait_ns, float &y, float &lse) {
    __shared__ float s_val[kPeerMaxRanks][kPeerWords];
    __shared__ uint32_t s_c;
    __shared__ int s_ok;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const PeerLayout L = peer_layout(px.n_slots);
    uint32_t *count = reinterpret_cast<uint32_t *>(px.bufs[px.rank] + L.counters_off) +
                      (static_cast<size_t>(px.slot) * kPeerMaxRows + row) * kPeerSlices + slice;
    if (tid == 0) {
        s_c = *count + 1;
        s_ok = 1;
    }
    __syncthreads();
    const uint32_t c = s_c;
    const uint32_t par = c & 1u;
    if (warp == 0) {
        for (int r = 0; r < px.n_ranks; ++r) {
            if (r == px.rank) continue;
            uint64_t *w = reinterpret_cast<uint64_t *>(px.bufs[r]) + peer_word(L, px.slot, par, px.rank, row, slice, 0);
            peer_put(w + lane, y_loc, c);
            if (lane == 0) peer_put(w + 32, lse_loc, c);
        }
        s_val[px.rank][lane] = y_loc;
        if (lane == 0) s_val[px.rank][32] = lse_loc;
    } else {
        // warps 1.. poll the peers in turn (warp w: peers w - 1, w - 1 + (warps - 1), ...;
        // one peer each when the CTA has n_ranks warps or more)
        const int n_warps = blockDim.x >> 5;
        for (int k = warp - 1; k < px.n_ranks - 1; k += n_warps - 1) {
            const int src = k < px.rank ? k : k + 1;
            const uint64_t *w = reinterpret_cast<const uint64_t *>(px.bufs[px.rank]) +
                                peer_word(L, px.slot, par, src, row, slice, 0);
            bool ok = true;
            for (int j = lane; j < kPeerWords && ok; j += 32) {
                uint2 v = peer_get(w + j);
                if (v.y != c) {
                    const uint64_t t0 = peer_globaltimer();
                    while ((v = peer_get(w + j)).y != c) {
                        if (peer_globaltimer() - t0 > wait_ns) {
                            ok = false;
                            break;
                        }
                    }
                }
                s_val[src][j] = __uint_as_float(v.x);
            }
            if (!__all_sync(0xffffffffu, ok)) {
                if (lane == 0) {
                    s_ok = 0;
                    if (px.status) atomicOr(px.status, 1u);
                }
                break;
            }
        }
    }
    __syncthreads();
    if (tid == 0) *count = c;
    if (!s_ok) return false;
    if (warp == 0) {
        float M = -INFINITY;
        for (int r = 0; r < px.n_ranks; ++r) M = fmaxf(M, s_val[r][32]);
        float acc = 0.f, Ls = 0.f;
        if (M > -INFINITY) {
            for (int r = 0; r < px.n_ranks; ++r) {
                const float lr = s_val[r][32];
                if (lr == -INFINITY) continue;
                const float wgt = __expf(lr - M);
                acc = fmaf(s_val[r][lane], wgt, acc);
                Ls += wgt;
            }
        }
        y = Ls > 0.f ? acc / Ls : 0.f;
        lse = Ls > 0.f ? M + logf(Ls) : -INFINITY;
    }
    return true;
}

}  // namespace sqmix
#endif
