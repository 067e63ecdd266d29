// FlashAttention prefill over the tiled q4_0 cache on the sm_100a tensor cores
// (tcgen05 / TMEM, CTA pairs).  Replaces ggml_flash_attn_ext for T >= 1 query tokens
// (src/model/attn.rs:238-249) with the causal mask of src/model/graph.rs:553-559
// (query t sees keys j <= q_pos0 + t, j < n_kv), GQA 16 / 2 heads, head_dim 256,
// the partial RoPE of attn.rs:183-204 on Q and the sigmoid output gate of
// attn.rs:282-283.
//
// Work decomposition.  An M-tile is 32 query tokens x the 8 query heads of one KV
// head (256 rows, row r = 8 * token + head), computed by a CTA pair (a cluster of
// two): the even CTA holds rows 0-127 (tokens 0-15), the odd one rows 128-255, and
// the even CTA's MMA thread issues cta_group::2 MMAs with M = 256.  Each CTA
// dequantises only half of every K/V tile (its 32 keys of K, its 128 head dimensions
// of V): the pair shares the operand, so the per-SM shared-memory traffic for K/V
// (dequantised stores + tensor-core reads) is half that of one CTA doing M = 128.
// The key tiles of all M-tiles, concatenated, are cut into one equal segment per
// pair of the persistent grid (one pair per two SMs); a segment is one to a few items
// (the part of one M-tile inside the segment).  Each item leaves (m, l, O) partials per
// row; fa_prefill_merge_kernel combines the items of an M-tile, applies the gate and
// writes the output.  pf_prep_kernel builds the item table from the device scalars
// n_kv and q_pos0 (CUDA-graph friendly) and writes Q once per call in the operand
// layout; the main and merge kernels are its programmatic dependents (each waits for
// its predecessor with griddepcontrol.wait after a prologue that overlaps it).
//
// One CTA (13 warps):
//   warp 0      TMEM allocation (pair form, both CTAs); in the even CTA lane 0 issues
//               the MMAs: S = Q K^T (M 256, N 128, K 256; Q and K from shared memory)
//               into one of two 128-column TMEM S buffers, then O += P V (M 256,
//               N 256, K 128; P read from tensor memory) into the TMEM O accumulator,
//               in the order S(0) S(1) PV(0) S(2) PV(1) ... so that the tensor cores
//               compute the next S while the softmax warps work on the current one;
//   warps 1-4   softmax: thread = row; reads S from TMEM in two passes (row maximum,
//               then exponentials), online softmax in the log2 domain with lazy
//               rescaling (O is rescaled only when the row maximum grows by more than
//               2^8), writes P (f16, two keys per column) over the first half of the S
//               buffer, and at the end of an item reads O and writes the partials;
//   warps 5-12  producers: bring the item's Q image (prepared once per call by
//               pf_prep_kernel: RoPE, f16, contraction order, swizzled) into shared
//               memory with one bulk copy, and dequantise this CTA's half of each K and
//               V tile from q4_0 into 128-byte-swizzled shared memory (two-buffer K and
//               V rings; the raw q4_0 of the next tile is loaded while the current one
//               is converted).
// Barriers that gate an MMA live in the even CTA; the odd CTA's warps arrive on them
// remotely (one elected lane per warp, default release semantics, which do not wait for
// the producers' prefetch loads in flight).  MMA completions are committed to the
// barrier at the same offset in both CTAs.  The per-item broadcast (item slot written
// into the peer) uses release / acquire at cluster scope.
// The contraction order of the head dimension is permuted so that each 16-byte
// chunk of the tiled cache dequantises into one 16-byte shared-memory chunk; Q uses
// the same permutation (K side) and the merge undoes the V-side one.
#include <math.h>

#include "common.cuh"
#include "sqmix.h"
#include "tc.cuh"

namespace sqmix {
namespace {

constexpr int kPfRows = 128;    // rows of one CTA (16 tokens x 8 heads)
constexpr int kPairRows = 256;  // rows of an M-tile (the pair)
constexpr int kPfTok = 16;
constexpr int kPairTok = 32;
constexpr int kPfKeys = 128;  // keys per tile
constexpr int kPfThreads = 13 * 32;
constexpr int kProdWarp0 = 5;
constexpr int kProdThreads = 256;
constexpr int kProdWarps = kProdThreads / 32;
constexpr int kSoftWarps = 4;
constexpr int kMaxMtiles = 512;  // setup block size; T <= 4096 gives <= 256 M-tiles

// shared memory (offsets from a 1024-byte aligned base; identical in both CTAs), all
// operands 128-byte swizzled:
//   Q      K-major, 4 regions (64 contraction positions) x 128 rows x 128 B
//   K ring 2 buffers: this CTA's 64 keys of a tile, K-major, 4 regions x 64 keys x 128 B
//   V ring 2 buffers: 128 keys x this CTA's 128 output columns, MN-major, 2 blocks of
//          64 columns x 128 keys x 128 B
constexpr uint32_t kQOff = 0;
constexpr uint32_t kQBytes = 65536;
constexpr uint32_t kQRegion = 16384;
constexpr uint32_t kKOff = kQBytes;
constexpr uint32_t kKBuf = 32768;
constexpr uint32_t kKRegion = 8192;
constexpr uint32_t kVOff = kKOff + 2 * kKBuf;
constexpr uint32_t kVBuf = 32768;
constexpr uint32_t kVBlock = 16384;
constexpr uint32_t kBarOff = kVOff + 2 * kVBuf;
constexpr uint32_t kSmemBytes = kBarOff + 256 + 1024;

// TMEM columns
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kOCol = 0;    // O: 256 columns f32
constexpr uint32_t kSCol = 256;  // S buffers: 2 x 128 columns (P, f16 pairs, over the first 64)

constexpr float kRescaleLog2 = 8.0f;

// workspace layout
constexpr int kMaxPairs = 2048;
constexpr size_t kWsHeader = 256;  // [0] u32 err, [12] u32 n_items, [16] u32 tiles per segment
constexpr size_t kWsMtab = kWsHeader;                         // int4 per M-tile
constexpr size_t kWsSegs = kWsMtab + kMaxMtiles * 16;         // int per pair + 1: first item of each segment
constexpr size_t kWsItems = kWsSegs + (kMaxPairs + 64) * 4;   // int4 per item

__host__ __device__ inline size_t align256(size_t x) { return (x + 255) / 256 * 256; }
// every segment boundary inside an M-tile adds one item
__host__ __device__ inline int pf_items_max(int n_pairs, int n_mtiles) { return n_pairs + n_mtiles + 1; }
// Q image: per M-tile and CTA the 64 KB shared-memory image of Q (f16, RoPE applied,
// contraction order, K-major 128-byte swizzle), copied in by one bulk copy per item
constexpr size_t kQImgBytes = kQBytes;
__host__ __device__ inline void pf_ws_layout(int n_pairs, int n_mtiles, size_t *ml, size_t *o, size_t *qimg,
                                             size_t *total) {
    const size_t items = static_cast<size_t>(pf_items_max(n_pairs, n_mtiles));
    *ml = align256(kWsItems + items * 16);
    *o = align256(*ml + items * kPairRows * 2 * sizeof(float));
    *qimg = align256(*o + items * kPairRows * 256 * sizeof(float));
    *total = *qimg + static_cast<size_t>(n_mtiles) * 2 * kQImgBytes;
}
__host__ __device__ inline int pf_n_mtiles(int T) { return 2 * ((T + kPairTok - 1) / kPairTok); }

struct PfParams {
    const void *q;
    int q_dtype;
    int64_t q_st, q_sh;
    const uint8_t *k_cache, *v_cache;
    const int64_t *n_kv, *q_pos0;
    int64_t capacity;
    int T;
    int n_mtiles;
    float c;  // scale * log2(e)
    int rope_n_rot;
    float rope_theta_scale;
    int64_t rope_pos_offset;
    uint8_t *ws;
    int items_max;
    size_t qimg_off;  // workspace offset of the Q image
};

__device__ __forceinline__ uint32_t *ws_err(uint8_t *ws) { return reinterpret_cast<uint32_t *>(ws); }
__device__ __forceinline__ uint32_t *ws_nitems(uint8_t *ws) { return reinterpret_cast<uint32_t *>(ws + 12); }

__device__ __forceinline__ int64_t clamp_nkv(const PfParams &p, uint8_t *ws, bool report) {
    int64_t n_kv = *p.n_kv;
    if (n_kv > p.capacity) {
        if (report) atomicOr(ws_err(ws), 8u);
        n_kv = p.capacity;
    }
    return n_kv < 0 ? 0 : n_kv;
}

// ---- item table ------------------------------------------------------------------
// The M-tiles' key tiles, concatenated in M-tile order (W tiles in all), are cut into
// n_pairs segments of ceil(W / n_pairs) tiles; pair q processes segment q.  An item is
// the part of one M-tile inside one segment: (m, first tile, end tile, 0).  Items are
// numbered in (M-tile, segment) order, which keeps each segment's items contiguous:
// segs[q] .. segs[q + 1] - 1.  mtab[m] = (first item, item count, -1, tiles).
__device__ __forceinline__ void block_scan_excl(int *buf, int m, int v, int &excl, int &total) {
    buf[m] = v;
    __syncthreads();
    for (int off = 1; off < kMaxMtiles; off <<= 1) {
        const int a = m >= off ? buf[m - off] : 0;
        __syncthreads();
        buf[m] += a;
        __syncthreads();
    }
    excl = buf[m] - v;
    total = buf[kMaxMtiles - 1];
    __syncthreads();
}

__device__ void pf_setup_block(const PfParams &p, int n_pairs) {
    __shared__ int scan[kMaxMtiles];
    const int m = threadIdx.x;
    const int64_t n_kv = clamp_nkv(p, p.ws, m == 0);
    const int64_t q_pos0 = *p.q_pos0;
    int len = 0;  // key tiles (kPfKeys keys each) the M-tile sees
    if (m < p.n_mtiles) {
        int t_last = kPairTok * (m >> 1) + kPairTok - 1;
        if (t_last > p.T - 1) t_last = p.T - 1;
        int64_t lim = q_pos0 + t_last + 1;
        if (lim > n_kv) lim = n_kv;
        if (lim < 0) lim = 0;
        len = static_cast<int>((lim + kPfKeys - 1) / kPfKeys);
    }
    int off, W;
    block_scan_excl(scan, m, len, off, W);
    const int seg = W > 0 ? (W + n_pairs - 1) / n_pairs : 1;
    const int q0 = off / seg;
    const int n_it = len > 0 ? (off + len - 1) / seg - q0 + 1 : 0;
    int ibase, total;
    block_scan_excl(scan, m, n_it, ibase, total);
    int4 *mtab = reinterpret_cast<int4 *>(p.ws + kWsMtab);
    int *segs = reinterpret_cast<int *>(p.ws + kWsSegs);
    int4 *items = reinterpret_cast<int4 *>(p.ws + kWsItems);
    if (total > p.items_max) {  // cannot happen (at most n_mtiles + n_pairs items); guarded anyway
        if (m == 0) {
            atomicOr(ws_err(p.ws), 32u);
            *ws_nitems(p.ws) = 0;
        }
        for (int q = m; q <= n_pairs; q += blockDim.x) segs[q] = 0;
        if (m < p.n_mtiles) mtab[m] = make_int4(0, 0, -1, 0);
        return;
    }
    if (m < p.n_mtiles) {
        mtab[m] = make_int4(ibase, n_it, -1, len);
        for (int k = 0; k < n_it; ++k) {
            const int q = q0 + k;
            const int lo = max(off, q * seg) - off, hi = min(off + len, (q + 1) * seg) - off;
            items[ibase + k] = make_int4(m, lo, hi, 0);
            if (q * seg >= off) segs[q] = ibase + k;  // segment q starts in this M-tile
        }
    }
    // segments past the end of the work are empty
    const int q_used = (W + seg - 1) / seg;
    for (int q = q_used + m; q <= n_pairs; q += blockDim.x) segs[q] = total;
    if (m == 0) {
        *ws_nitems(p.ws) = static_cast<uint32_t>(total);
        reinterpret_cast<uint32_t *>(p.ws)[4] = static_cast<uint32_t>(seg);
    }
}

// ---- Q image ---------------------------------------------------------------------
// real head dimension of contraction (K-side) position p, 0..255
__device__ __forceinline__ int k_real_dim(int p) {
    const int i1 = p >> 7, c = (p >> 5) & 3, w = (p >> 3) & 3, e = p & 7;
    const int b = 4 * i1 + w;
    return 32 * b + 4 * c + (e & 3) + 16 * (e >> 2);
}


// One block per query token (padded to whole M-tiles), 8 f16 pairs per thread, all
// loads issued before the RoPE table is needed: RoPE (the table of rope_cos_sin for the
// position, as ggml builds its cache), f16, contraction permutation; pair w of a row
// holds positions 2w, 2w+1, which are the adjacent head dimensions k_real_dim(2w),
// k_real_dim(2w) + 1.  Rows of padding tokens are zero.  Q rows must be aligned to two
// elements (the host checks it).
template <int DT>
__device__ __forceinline__ float2 load_pair_t(const void *src, int64_t i) {
    if (DT == SQMIX_F32) return *reinterpret_cast<const float2 *>(static_cast<const float *>(src) + i);
    if (DT == SQMIX_BF16)
        return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(static_cast<const __nv_bfloat16 *>(src) + i));
    return __half22float2(*reinterpret_cast<const __half2 *>(static_cast<const __half *>(src) + i));
}

// Thread tid (0..255) of token t writes pair w = tid % 128 of the rows of heads
// 2k + tid / 128, k = 0..7: everything but the head is the same for the eight pairs.
template <int DT>
__device__ void pf_qprep_token(const PfParams &p, int t, int tid, float2 *rope_tab) {
    const int half = p.rope_n_rot >> 1;
    const bool live = t < p.T;
    const int w = tid & 127, hsel = tid >> 7;
    const int dim = k_real_dim(2 * w);  // even; dim + 1 is position 2w + 1
    const bool rot = dim < p.rope_n_rot, lo = dim < half;
    const int pdim = lo ? dim + half : dim - half;  // RoPE partner
    const int ri = lo ? dim : dim - half;
    float2 x[8], y[8];
    const int64_t row0 = t * p.q_st + hsel * p.q_sh;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        x[k] = y[k] = make_float2(0.f, 0.f);
        if (live) {
            const int64_t rbase = row0 + 2 * k * p.q_sh;
            x[k] = load_pair_t<DT>(p.q, rbase + dim);
            if (rot) y[k] = load_pair_t<DT>(p.q, rbase + pdim);
        }
    }
    if (tid < 32) {
        const int i = tid;
        rope_tab[i] = (i < half && live) ? rope_cos_sin(*p.q_pos0 + t + p.rope_pos_offset, p.rope_theta_scale, i)
                                         : make_float2(1.f, 0.f);
    }
    __syncthreads();
    float2 c0 = make_float2(1.f, 0.f), c1 = c0;
    if (rot) {
        c0 = rope_tab[ri];
        c1 = rope_tab[ri + 1];
    }
    // image address: M-tile m = (t / 32) * 2 + head / 8, pair row prr = (t % 32) * 8 + head % 8
    // (its CTA = prr / 128 is the same for all eight heads), positions 2w, 2w+1 -> region,
    // 16-byte chunk swizzled with row % 8 = (2k) % 8 + hsel
    const int prr0 = (t % kPairTok) * 8;
    const int cta = prr0 >> 7;
    const int el = (2 * w) & 63, chunk = el >> 3;
    uint8_t *img = p.ws + p.qimg_off + ((2 * w) >> 6) * kQRegion + (el & 7) * 2;
    const size_t m0 = static_cast<size_t>(t / kPairTok) * 2;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        uint32_t v = 0u;
        if (live) {
            float2 z = x[k];
            if (rot)
                z = lo ? make_float2(__fsub_rn(__fmul_rn(x[k].x, c0.x), __fmul_rn(y[k].x, c0.y)),
                                     __fsub_rn(__fmul_rn(x[k].y, c1.x), __fmul_rn(y[k].y, c1.y)))
                       : make_float2(__fadd_rn(__fmul_rn(y[k].x, c0.y), __fmul_rn(x[k].x, c0.x)),
                                     __fadd_rn(__fmul_rn(y[k].y, c1.y), __fmul_rn(x[k].y, c1.x)));
            v = pack_half2(z.x, z.y);
        }
        const int r7 = ((2 * k) & 7) + hsel;
        const int rr = (prr0 & 127) + r7;
        const size_t byte = ((m0 + (k >> 2)) * 2 + cta) * kQImgBytes + rr * 128 + (((chunk ^ r7) & 7) << 4);
        *reinterpret_cast<uint32_t *>(img + byte) = v;
    }
}

// One launch before the main kernel: block 0 builds the item table (first in grid
// order, so that its scan overlaps the Q blocks instead of trailing them), blocks
// 1 .. T_pad/2 prepare Q for two tokens each (256 threads per token).  The main kernel,
// launched as its programmatic dependent, runs its prologue meanwhile.
constexpr int kPrepThreads = kMaxMtiles;  // 512
__global__ void __launch_bounds__(kPrepThreads) pf_prep_kernel(PfParams p, int n_pairs) {
    asm volatile("griddepcontrol.launch_dependents;" :::);
    if (blockIdx.x == 0) {
        pf_setup_block(p, n_pairs);
        return;
    }
    __shared__ float2 rope_tab[2][32];
    const int half_id = threadIdx.x >> 8;
    const int t = 2 * (blockIdx.x - 1) + half_id, tid = threadIdx.x & 255;
    if (p.q_dtype == SQMIX_F32)
        pf_qprep_token<SQMIX_F32>(p, t, tid, rope_tab[half_id]);
    else if (p.q_dtype == SQMIX_BF16)
        pf_qprep_token<SQMIX_BF16>(p, t, tid, rope_tab[half_id]);
    else
        pf_qprep_token<SQMIX_F16>(p, t, tid, rope_tab[half_id]);
}

// ---- helpers -----------------------------------------------------------------------
__device__ __forceinline__ uint32_t swz(uint32_t row, uint32_t chunk) {
    return row * 128u + (((chunk ^ (row & 7u)) & 7u) << 4);
}
__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}
// two nibbles (already isolated in bits 0-3 of bytes bl, bh of x) -> f16 pair (n - 8) * d
__device__ __forceinline__ uint32_t nib_pair(uint32_t x, uint32_t sel, __half2 d2) {
    uint32_t h;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(h) : "r"(x), "r"(0x64u), "r"(sel));
    const __half2 v = __hsub2(u32_as_h2(h), __float2half2_rn(1032.0f));
    return h2_as_u32(__hmul2(v, d2));
}
// Bounded wait whose outcome is the same in every lane of the warp: all lanes wait,
// then vote, so that a warp never splits on a timeout.  Every lane of the warp must
// call it.
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag, uint32_t *err,
                                          uint32_t bit) {
    bool ok = false;
    if (!*abort_flag) {
        ok = mbar_wait(bar, parity);
        if (!ok) {
            atomicOr(err, bit);
            *abort_flag = 1;
        }
    }
    return __all_sync(0xffffffffu, ok);
}
// single-thread form (the MMA thread, the item ring); `cl`: acquire at cluster scope
__device__ __forceinline__ bool wait_or_abort(uint64_t *bar, uint32_t parity, volatile int *abort_flag,
                                              uint32_t *err, uint32_t bit, bool cl = false) {
    if (*abort_flag) return false;
    if (cl ? mbar_wait_cl(bar, parity) : mbar_wait(bar, parity)) return true;
    atomicOr(err, bit);
    *abort_flag = 1;
    return false;
}

// real head dimension of output (V-side) column v, 0..255
__device__ __forceinline__ int v_real_dim(int v) {
    const int i = v >> 6, g = (v >> 3) & 7, w = (v >> 1) & 3, hi = v & 1;
    const int b = 2 * i + (w >> 1), m = w & 1;
    return 32 * b + 8 * m + g + 16 * hi;
}

struct SmemCtl {
    uint64_t k_full[2];     // even CTA: producer warps of both CTAs (K buffer filled)
    uint64_t v_full[2];     // even CTA: producer warps of both CTAs (V buffer filled)
    uint64_t s_full[2];     // both: S MMA complete (S ready; its K buffer free)
    uint64_t pv_done[2];    // both: PV MMA complete (O updated; its V buffer free)
    uint64_t p_full[2];     // even CTA: softmax warps of both CTAs (P written)
    uint64_t q_load;        // local: bulk copy of Q
    uint64_t q_full;        // even CTA: one arrival per CTA (Q in shared memory)
    uint64_t q_free;        // both: MMA completion of an item's last S (Q reusable)
    uint64_t o_free;        // even CTA: softmax warps of both CTAs (partials read)
    uint64_t item_full[2];  // both: the fetcher
    uint64_t item_empty[2]; // even CTA: every consumer thread of both CTAs
    uint64_t final_bar;     // both: MMA completion
    int4 item[2];
    uint32_t tmem_base;
    int abort_flag;
};
static_assert(sizeof(SmemCtl) <= 256, "control block");

// Raw q4_0 of this CTA's part of one 128-key tile for one producer thread (2 K + 2 V jobs).
struct RawTile {
    uint4 kn[2], vn[2], vs[2];
    uint2 ks[2];
};

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPfThreads, 1) fa_prefill_kernel(PfParams p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base_s = (raw + 1023u) & ~1023u;  // shared address of the aligned base
    uint8_t *base = smem_raw + (base_s - raw);
    SmemCtl *ctl = reinterpret_cast<SmemCtl *>(base + kBarOff);
    volatile int *abort_flag = &ctl->abort_flag;
    uint32_t *err = ws_err(p.ws);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();  // 0: issues the MMAs; 1: its peer
    // shared::cluster address of a barrier of the even CTA / of the peer CTA
    auto lead = [&](uint64_t *bar) -> uint32_t { return mapa_shared(smem_u32(bar), 0); };
    auto peer = [&](const void *x) -> uint32_t { return mapa_shared(smem_u32(x), rank ^ 1u); };
    if (threadIdx.x == 0) {
        for (int s = 0; s < 2; ++s) {
            mbar_init(&ctl->k_full[s], 2 * kProdWarps);
            mbar_init(&ctl->v_full[s], 2 * kProdWarps);
            mbar_init(&ctl->s_full[s], 1);
            mbar_init(&ctl->pv_done[s], 1);
            mbar_init(&ctl->p_full[s], 2 * kSoftWarps);
            mbar_init(&ctl->item_full[s], 1);
            // even CTA: MMA lane + softmax + producers; odd CTA: softmax + producers
            mbar_init(&ctl->item_empty[s], (kPfThreads - 31) + (kPfThreads - 32));
        }
        mbar_init(&ctl->q_load, 1);
        mbar_init(&ctl->q_full, 2);
        mbar_init(&ctl->q_free, 1);
        mbar_init(&ctl->o_free, 2 * kSoftWarps);
        mbar_init(&ctl->final_bar, 1);
        ctl->abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tc::tmem_alloc_pair(&ctl->tmem_base, kTmemCols);
        tc::tmem_relinquish_pair();
    }
    tc::fence_before();
    __syncthreads();
    cluster_sync_all();  // both CTAs' barriers are initialised before any remote arrival
    tc::fence_after();
    const uint32_t tmem = ctl->tmem_base;
    // launched as the programmatic dependent of pf_prep_kernel: the prologue above
    // overlapped it; the item table and the Q image are read only after it completes
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" :::);

    const int64_t n_kv = clamp_nkv(p, p.ws, false);
    const int64_t q_pos0 = *p.q_pos0;
    const int4 *items = reinterpret_cast<const int4 *>(p.ws + kWsItems);
    // this pair's segment of the item list
    const int *segs = reinterpret_cast<const int *>(p.ws + kWsSegs);
    const int pair = static_cast<int>(blockIdx.x >> 1);
    const int seg_lo = segs[pair], seg_hi = segs[pair + 1];
    const size_t ml_off = align256(kWsItems + static_cast<size_t>(p.items_max) * 16);
    const size_t o_off = align256(ml_off + static_cast<size_t>(p.items_max) * kPairRows * 2 * sizeof(float));
    float *part_ml = reinterpret_cast<float *>(p.ws + ml_off);
    float *part_o = reinterpret_cast<float *>(p.ws + o_off);

    // item ring: the even CTA's first producer fetches and writes the item into both
    // CTAs; every consumer thread of both CTAs copies it and releases the slot
    auto get_item = [&](int iter, int4 &it, bool fetcher) -> bool {
        const int slot = iter & 1;
        if (fetcher) {
            int4 e = make_int4(-1, 0, 0, -1);
            if (iter < 2 ||
                wait_or_abort(&ctl->item_empty[slot], ((iter - 2) >> 1) & 1, abort_flag, err, 64u, true)) {
                const int q = seg_lo + iter;
                e = q < seg_hi ? items[q] : make_int4(-1, 0, 0, 0);
                e.w = q;
            }
            ctl->item[slot] = e;
            st_cluster_v4(peer(&ctl->item[slot]), e);
            mbar_arrive_cl(lead(&ctl->item_full[slot]));
            mbar_arrive_cl(peer(&ctl->item_full[slot]));
        }
        if (!wait_or_abort(&ctl->item_full[slot], (iter >> 1) & 1, abort_flag, err, 64u, true)) return false;
        it = ctl->item[slot];
        mbar_arrive_cl(lead(&ctl->item_empty[slot]));
        return it.x >= 0;
    };
    // parity of tile jj's completion on a barrier of a two-buffer ring (tiles b, b+2, ...)
    auto ring_parity = [](int jj) -> uint32_t { return static_cast<uint32_t>(jj >> 1) & 1u; };

    const uint32_t idesc_s = tc::idesc_f16_f32(2 * 128, kPfKeys, 0, 0);
    const uint32_t idesc_pv = tc::idesc_f16_f32(2 * 128, 256, 0, 1);

    if (warp == 0) {
        // =========================== MMA issuer (even CTA) ===========================
        if (rank == 0 && lane == 0) {
            int j = 0;
            bool ok = true;
            // completion of the MMAs issued so far -> barrier `bar` in both CTAs
            auto commit_both = [&](uint64_t *bar) {
                tc::commit_pair(lead(bar));
                tc::commit_pair(peer(bar));
            };
            auto issue_s = [&](int jj, bool last_of_item) -> bool {
                const int sb = jj & 1;
                if (!wait_or_abort(&ctl->k_full[sb], ring_parity(jj), abort_flag, err, 1u)) return false;
                tc::fence_after();
#pragma unroll
                for (int ks = 0; ks < 16; ++ks) {
                    // A = Q (this CTA's 128 rows), B = this CTA's 64 keys; both K-major
                    const uint64_t a = tc::desc_sw128(base_s + kQOff + (ks >> 2) * kQRegion + (ks & 3) * 32, 16, 1024);
                    const uint64_t b = tc::desc_sw128(
                        base_s + kKOff + sb * kKBuf + (ks >> 2) * kKRegion + (ks & 3) * 32, 16, 1024);
                    tc::mma_ss_pair(tmem + kSCol + sb * kPfKeys, a, b, idesc_s, ks > 0 ? 1u : 0u);
                }
                commit_both(&ctl->s_full[sb]);
                if (last_of_item) commit_both(&ctl->q_free);
                return true;
            };
            auto issue_pv = [&](int jj, bool first) -> bool {
                const int bb = jj & 1;
                if (!wait_or_abort(&ctl->p_full[bb], ring_parity(jj), abort_flag, err, 1u)) return false;
                if (!wait_or_abort(&ctl->v_full[bb], ring_parity(jj), abort_flag, err, 1u)) return false;
                tc::fence_after();
#pragma unroll
                for (int ks = 0; ks < kPfKeys / 16; ++ks) {
                    // A = P (f16, two keys per column) in the first 64 columns of S buffer bb;
                    // B = this CTA's 128 output columns (MN-major, 2 blocks of 64)
                    const uint64_t b = tc::desc_sw128(base_s + kVOff + bb * kVBuf + ks * 2048, kVBlock, 1024);
                    tc::mma_ts_pair(tmem + kOCol, tmem + kSCol + bb * kPfKeys + ks * 8, b, idesc_pv,
                                    (!first || ks > 0) ? 1u : 0u);
                }
                commit_both(&ctl->pv_done[bb]);
                return true;
            };
            for (int iter = 0; ok; ++iter) {
                int4 it;
                if (!get_item(iter, it, false)) break;
                const int n = it.z - it.y;
                if (!wait_or_abort(&ctl->q_full, iter & 1, abort_flag, err, 1u)) break;
                tc::fence_after();
                const int jf = j;
                // S(jj) goes into the S buffer whose P was read by PV(jj - 2), issued earlier
                if (!issue_s(jf, n == 1)) break;
                for (int t = 0; t < n; ++t) {
                    if (t + 1 < n && !issue_s(jf + t + 1, t + 2 == n)) { ok = false; break; }
                    // the item's first PV overwrites O: the previous item's partials are read
                    // (its S MMAs may run during that epilogue)
                    if (t == 0 && iter > 0) {
                        if (!wait_or_abort(&ctl->o_free, (iter - 1) & 1, abort_flag, err, 1u)) { ok = false; break; }
                        tc::fence_after();
                    }
                    if (!issue_pv(jf + t, t == 0)) { ok = false; break; }
                }
                j = jf + n;
            }
            // drain: every MMA issued so far completes before either CTA releases TMEM
            commit_both(&ctl->final_bar);
            if (!mbar_wait(&ctl->final_bar, 0)) atomicOr(err, 128u);
        }
    } else if (warp < kProdWarp0) {
        // =========================== softmax ===========================
        const int r = 32 * (warp & 3) + lane;  // TMEM lane == row
        const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;
        auto wwait = [&](uint64_t *bar, uint32_t parity) -> bool {
            return warp_wait(bar, parity, abort_flag, err, 2u);
        };
        // one elected arrival per warp on a barrier of the even CTA (after every lane's
        // tcgen05 accesses are complete and fenced)
        auto warp_arrive = [&](uint64_t *bar) {
            tc::fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(lead(bar));
        };
        int j = 0;
        for (int iter = 0;; ++iter) {
            int4 it;
            const bool got = get_item(iter, it, false);
            if (!__all_sync(0xffffffffu, got)) break;
            const int m = it.x, kt0 = it.y, kt1 = it.z, item = it.w;
            const int token = kPairTok * (m >> 1) + kPfTok * static_cast<int>(rank) + (r >> 3);
            int64_t lim = q_pos0 + token;
            if (lim > n_kv - 1) lim = n_kv - 1;
            if (token >= p.T) lim = -1;
            float m_run = -INFINITY, l_run = 0.f;
            bool ok = true;
            for (int kt = kt0; kt < kt1; ++kt, ++j) {
                const int b = j & 1;
                const uint32_t sbuf = tmem + lane_base + kSCol + b * kPfKeys;
                if (!wwait(&ctl->s_full[b], ring_parity(j))) { ok = false; break; }
                tc::fence_after();
                const int64_t key0 = static_cast<int64_t>(kt) * kPfKeys;
                // keys key0 + k with k <= vis_last are visible (clamped to -1 .. kPfKeys - 1)
                int64_t vl = lim - key0;
                vl = vl < -1 ? -1 : (vl > kPfKeys - 1 ? kPfKeys - 1 : vl);
                const int vis_last = static_cast<int>(vl);
                const bool any_masked = __any_sync(0xffffffffu, vis_last < kPfKeys - 1);
                // pass 1: row maximum of the raw scores over the 128 keys
                float mx[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) mx[i] = -INFINITY;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    uint32_t sr[64];
                    tc::ld64(sbuf + 64 * h, sr);
                    if (any_masked) {
#pragma unroll
                        for (int i = 0; i < 64; ++i)
                            mx[i & 7] = fmaxf(mx[i & 7], 64 * h + i <= vis_last ? __uint_as_float(sr[i]) : -INFINITY);
                    } else {
#pragma unroll
                        for (int i = 0; i < 64; ++i) mx[i & 7] = fmaxf(mx[i & 7], __uint_as_float(sr[i]));
                    }
                }
                const float mt = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                                       fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))) *
                                 p.c;
                const bool grow = mt > m_run + kRescaleLog2 || (m_run == -INFINITY && mt > -INFINITY);
                const float m_new = grow ? mt : m_run;
                const bool first = kt == kt0;
                const bool need = grow && m_run > -INFINITY && !first;
                const float alpha = need ? ex2(m_run - m_new) : 1.f;
                if (__any_sync(0xffffffffu, need)) {
                    // O holds the PV of the previous tile once it completes
                    const int jp = j - 1;
                    if (!wwait(&ctl->pv_done[jp & 1], ring_parity(jp))) {
                        ok = false;
                        break;
                    }
                    tc::fence_after();
#pragma unroll 1
                    for (int ch = 0; ch < 8; ++ch) {
                        uint32_t o[32];
                        tc::ld32(tmem + lane_base + kOCol + ch * 32, o);
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                        tc::st32(tmem + lane_base + kOCol + ch * 32, o);
                    }
                    tc::wait_st();
                }
                l_run *= alpha;
                m_run = m_new;
                // pass 2: p = 2^(c s - m), masked entries 2^-inf = 0 (a row with nothing
                // visible yet subtracts 0 instead of -inf); P (f16 pairs) replaces S in the
                // first 64 columns of the buffer, half h over columns already read
                const float msub = m_run == -INFINITY ? 0.f : m_run;
                float lsum[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) lsum[i] = 0.f;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    uint32_t sr[64];
                    tc::ld64(sbuf + 64 * h, sr);
                    if (any_masked) {
#pragma unroll
                        for (int i = 0; i < 64; ++i)
                            if (64 * h + i > vis_last) sr[i] = 0xff800000u;  // -inf
                    }
                    uint32_t ph[32];
#pragma unroll
                    for (int i = 0; i < 64; i += 2) {
                        const float p0 = ex2(fmaf(__uint_as_float(sr[i]), p.c, -msub));
                        const float p1 = ex2(fmaf(__uint_as_float(sr[i + 1]), p.c, -msub));
                        lsum[(i >> 1) & 7] += p0 + p1;
                        ph[i >> 1] = pack_half2(p0, p1);
                    }
                    tc::st32(sbuf + 32 * h, ph);
                }
                l_run += ((lsum[0] + lsum[1]) + (lsum[2] + lsum[3])) + ((lsum[4] + lsum[5]) + (lsum[6] + lsum[7]));
                tc::wait_st();
                warp_arrive(&ctl->p_full[b]);
            }
            if (!ok) break;
            // ---- item epilogue: partial (m, l, O) of every row ----
            const int jl = j - 1;
            if (!wwait(&ctl->pv_done[jl & 1], ring_parity(jl))) break;
            tc::fence_after();
            // O partials column-chunk-major ([item][column / 4][row][4]): a warp's stores
            // of one chunk cover 512 contiguous bytes
            const int rowp = static_cast<int>(rank) * kPfRows + r;
            float4 *ob = reinterpret_cast<float4 *>(part_o) + static_cast<size_t>(item) * 64 * kPairRows + rowp;
#pragma unroll 1
            for (int ch = 0; ch < 8; ++ch) {
                uint32_t o[32];
                tc::ld32(tmem + lane_base + kOCol + ch * 32, o);
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    ob[(ch * 8 + i) * kPairRows] = make_float4(__uint_as_float(o[4 * i]), __uint_as_float(o[4 * i + 1]),
                                                               __uint_as_float(o[4 * i + 2]),
                                                               __uint_as_float(o[4 * i + 3]));
            }
            warp_arrive(&ctl->o_free);
            *reinterpret_cast<float2 *>(part_ml + (static_cast<size_t>(item) * kPairRows + rowp) * 2) =
                make_float2(m_run, l_run);
        }
    } else {
        // =========================== producers ===========================
        const int pt = threadIdx.x - kProdWarp0 * 32;  // 0..255
        const bool fetcher = rank == 0 && pt == 0;
        auto pwait = [&](uint64_t *bar, uint32_t parity) -> bool {
            return warp_wait(bar, parity, abort_flag, err, 4u);
        };
        auto warp_arrive = [&](uint64_t *bar) {
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(lead(bar));
        };
        int j = 0;
        // K job u: 16 B of nibbles of one of this CTA's 64 keys of the tile (16-key groups
        // 4 rank .. 4 rank + 3); V job u: 16 B of nibbles of one of the 128 keys, this
        // CTA's segments 2 rank, 2 rank + 1
        auto load_raw = [&](int kt, int kvh, RawTile &rw) {
            const int64_t g0 = static_cast<int64_t>(kt) * (kPfKeys / kGroupTokens);
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int job = pt + kProdThreads * u;
                {
                    const int gl = job >> 7, ch = job & 127;
                    const int i = ch >> 5, g = (ch >> 2) & 7, c = ch & 3;
                    const int64_t ku = ((g0 + 4 * rank + gl) * kHeadsKV + kvh) * kUnitBytes;
                    rw.kn[u] = __ldg(reinterpret_cast<const uint4 *>(p.k_cache + ku + i * 512 + (4 * g + c) * 16));
                    rw.ks[u] = __ldg(reinterpret_cast<const uint2 *>(p.k_cache + ku + kUnitQsBytes + g * 32 +
                                                                     (i >> 1) * 16 + 8 * (i & 1)));
                }
                {
                    const int gi = job >> 6, rest = job & 63;
                    const int i = 2 * static_cast<int>(rank) + (rest >> 5), g = (rest >> 2) & 7, c = rest & 3;
                    const int64_t vu = ((g0 + gi) * kHeadsKV + kvh) * kUnitBytes;
                    rw.vn[u] = __ldg(reinterpret_cast<const uint4 *>(p.v_cache + vu + i * 512 + (4 * g + c) * 16));
                    rw.vs[u] = __ldg(reinterpret_cast<const uint4 *>(p.v_cache + vu + kUnitQsBytes + c * 64 + 16 * i));
                }
            }
        };
        for (int iter = 0;; ++iter) {
            int4 it;
            const bool got = get_item(iter, it, fetcher);
            if (!__all_sync(0xffffffffu, got)) break;
            const int m = it.x, kt0 = it.y, kt1 = it.z;
            const int kvh = m & 1;
            if (warp == kProdWarp0) {
                // ---- Q: the item's prepared 64 KB image by one bulk copy, once the previous
                // item's S MMAs (its readers) are complete ----
                if (iter > 0 && !pwait(&ctl->q_free, (iter - 1) & 1)) break;
                if (lane == 0) {
                    mbar_arrive_expect_tx(&ctl->q_load, static_cast<uint32_t>(kQImgBytes));
                    bulk_g2s(base + kQOff, p.ws + p.qimg_off + (static_cast<size_t>(m) * 2 + rank) * kQImgBytes,
                             static_cast<uint32_t>(kQImgBytes), &ctl->q_load);
                }
                if (!pwait(&ctl->q_load, iter & 1)) break;
                if (lane == 0) mbar_arrive_remote(lead(&ctl->q_full));
            }
            RawTile cur;
            load_raw(kt0, kvh, cur);
            bool ok = true;
            // ---- K / V tiles: the raw q4_0 of tile kt+1 is loaded while tile kt is converted ----
            for (int kt = kt0; kt < kt1; ++kt, ++j) {
                const int b = j & 1;
                RawTile nxt;
                if (kt + 1 < kt1) load_raw(kt + 1, kvh, nxt);
                const int64_t key0 = static_cast<int64_t>(kt) * kPfKeys;
                // K buffer b: free once S(j - 2) is complete
                if (j >= 2 && !pwait(&ctl->s_full[b], ring_parity(j - 2))) { ok = false; break; }
                const uint32_t kst = base_s + kKOff + b * kKBuf;
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    // key row gl*16 + g + 8*(i>>1) of this CTA's 64; blocks 4*(i&1) + w ->
                    // region (i&1)*2 + (c>>1), chunks (c&1)*4 + w.  Lanes c and c+2 write the
                    // same chunks of different regions (same banks): they take w in the order w ^ 2.
                    const int job = pt + kProdThreads * u;
                    const int gl = job >> 7, ch = job & 127;
                    const int i = ch >> 5, g = (ch >> 2) & 7, c = ch & 3;
                    const int row = gl * 16 + g + 8 * (i >> 1);
                    const bool live = key0 + 64 * static_cast<int>(rank) + row < n_kv;
                    // slot s holds word w = s ^ (rot ? 2 : 0) and its scale d[w >> 1]
                    const bool rot = (c & 2) != 0;
                    const uint32_t w4[4] = {rot ? cur.kn[u].z : cur.kn[u].x, rot ? cur.kn[u].w : cur.kn[u].y,
                                            rot ? cur.kn[u].x : cur.kn[u].z, rot ? cur.kn[u].y : cur.kn[u].w};
                    const uint32_t d4[2] = {rot ? cur.ks[u].y : cur.ks[u].x, rot ? cur.ks[u].x : cur.ks[u].y};
                    const uint32_t rb = kst + ((i & 1) * 2 + (c >> 1)) * kKRegion;
#pragma unroll
                    for (int s4 = 0; s4 < 4; ++s4) {
                        uint4 o = make_uint4(0u, 0u, 0u, 0u);
                        if (live) {
                            const __half2 dd = u32_as_h2(d4[s4 >> 1]);
                            const __half d1 = (s4 & 1) ? __high2half(dd) : __low2half(dd);
                            const __half2 d2 = __half2half2(d1);
                            const uint32_t lo = w4[s4] & 0x0F0F0F0Fu;
                            const uint32_t hi = (w4[s4] >> 4) & 0x0F0F0F0Fu;
                            o = make_uint4(nib_pair(lo, 0x4140u, d2), nib_pair(lo, 0x4342u, d2),
                                           nib_pair(hi, 0x4140u, d2), nib_pair(hi, 0x4342u, d2));
                        }
                        sts128(rb + swz(row, (c & 1) * 4 + (rot ? (s4 ^ 2) : s4)), o);
                    }
                }
                tc::fence_proxy_async_smem();
                warp_arrive(&ctl->k_full[b]);
                // V buffer b: free once PV(j - 2) is complete
                if (j >= 2 && !pwait(&ctl->pv_done[b], ring_parity(j - 2))) { ok = false; break; }
                const uint32_t vst = base_s + kVOff + b * kVBuf;
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    // tokens {2c, 2c+8, 2c+1, 2c+9} (byte positions 0..3) of group gi;
                    // blocks 2i + (w>>1); block il, chunk g
                    const int job = pt + kProdThreads * u;
                    const int gi = job >> 6, rest = job & 63;
                    const int il = rest >> 5, g = (rest >> 2) & 7, c = rest & 3;
                    const uint32_t w4[4] = {cur.vn[u].x, cur.vn[u].y, cur.vn[u].z, cur.vn[u].w};
                    const uint32_t d4[4] = {cur.vs[u].x, cur.vs[u].y, cur.vs[u].z, cur.vs[u].w};
                    const uint32_t rb = vst + il * kVBlock;
                    // lo/hi nibbles of the 4 tokens, token-interleaved: [l0 h0 l1 h1], [l2 h2 l3 h3]
                    uint32_t xy[4][2];
#pragma unroll
                    for (int w = 0; w < 4; ++w) {
                        const uint32_t lo = w4[w] & 0x0F0F0F0Fu;
                        const uint32_t hi = (w4[w] >> 4) & 0x0F0F0F0Fu;
                        asm("prmt.b32 %0, %1, %2, 0x5140;" : "=r"(xy[w][0]) : "r"(lo), "r"(hi));
                        asm("prmt.b32 %0, %1, %2, 0x7362;" : "=r"(xy[w][1]) : "r"(lo), "r"(hi));
                    }
#pragma unroll
                    for (int pos = 0; pos < 4; ++pos) {
                        const int tt = (pos & 1) * 8 + 2 * c + (pos >> 1);
                        const int row = gi * 16 + tt;
                        const int jj = (pos >> 1) + 2 * (pos & 1);  // scale slot of this token
                        uint4 outv = make_uint4(0u, 0u, 0u, 0u);
                        if (key0 + row < n_kv) {
                            uint32_t o4[4];
#pragma unroll
                            for (int w = 0; w < 4; ++w) {
                                // scales: [b=2i: jj0..3][b=2i+1: jj0..3] as 8 halves
                                const int hidx = (w >> 1) * 4 + jj;
                                const __half2 dd = u32_as_h2(d4[hidx >> 1]);
                                const __half d1 = (hidx & 1) ? __high2half(dd) : __low2half(dd);
                                o4[w] = nib_pair(xy[w][pos >> 1], (pos & 1) ? 0x4342u : 0x4140u,
                                                 __half2half2(d1));
                            }
                            outv = make_uint4(o4[0], o4[1], o4[2], o4[3]);
                        }
                        sts128(rb + swz(row, g), outv);
                    }
                }
                tc::fence_proxy_async_smem();
                warp_arrive(&ctl->v_full[b]);
                if (kt + 1 < kt1) cur = nxt;
            }
            if (!ok) break;
        }
    }

    // Neither CTA releases TMEM or exits while the pair's MMAs or remote arrivals may
    // still touch its memory: past the cluster barrier the even CTA has seen its drain
    // complete, and the odd CTA then takes the drain's arrival on its own barrier.
    tc::fence_before();
    __syncthreads();
    cluster_sync_all();
    if (rank == 1 && threadIdx.x == 0 && !mbar_wait(&ctl->final_bar, 0)) atomicOr(err, 128u);
    __syncthreads();
    tc::fence_after();
    if (warp == 0) {
        __syncwarp();
        tc::tmem_dealloc_pair(tmem, kTmemCols);
    }
}

// ---- merge of the items of each M-tile, gate, output ------------------------------
struct PfMergeParams {
    const uint8_t *ws;
    int items_max;
    int T;
    const void *gate;
    int gate_dtype;
    int64_t g_st, g_sh;
    float *out;
    float *lse;
};

// grid (T, 2 KV heads), 256 threads: one block merges the 8 rows (heads) of one token.
// Thread i reads the 16-byte partial chunks (column chunk i / 8 and i / 8 + 32, row
// i % 8), so that a warp's loads cover 128 contiguous bytes per chunk, and folds the
// items in one online pass; the rows are then written through shared memory in head-
// dimension order (1 KB contiguous per row).
__global__ void __launch_bounds__(256) fa_prefill_merge_kernel(PfMergeParams p) {
    __shared__ float orow[8][256];
    __shared__ float lse_s[8];
    const int t = blockIdx.x, kvh = blockIdx.y, i = threadIdx.x;
    const int hq = i & 7, c4a = i >> 3;  // chunks c4a and c4a + 32
    const int m = (t / kPairTok) * 2 + kvh;
    // The item table (prep kernel) and the gate (written before the call) are complete
    // when this grid starts (its predecessor, the main kernel, waited for them before
    // triggering it); only the partials need the grid-dependency wait.
    const int4 mt = reinterpret_cast<const int4 *>(p.ws + kWsMtab)[m];
    float gs[8];
#pragma unroll
    for (int h = 0; h < 8; ++h)
        gs[h] = p.gate ? load_act(p.gate, t * p.g_st + (kvh * 8 + h) * p.g_sh + i, p.gate_dtype) : 0.f;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const size_t ml_off = align256(kWsItems + static_cast<size_t>(p.items_max) * 16);
    const size_t o_off = align256(ml_off + static_cast<size_t>(p.items_max) * kPairRows * 2 * sizeof(float));
    const float2 *part_ml = reinterpret_cast<const float2 *>(p.ws + ml_off);
    const float4 *part_o = reinterpret_cast<const float4 *>(p.ws + o_off);
    const int n_parts = mt.y + (mt.z >= 0 ? 1 : 0);
    const int r = (t % kPairTok) * 8 + hq;  // row of the M-tile (odd CTA's rows from 128)
    auto item_of = [&](int k) { return static_cast<size_t>(k < mt.y ? mt.x + k : mt.z); };
    // the partials of up to kBatch items are loaded at once (one round trip), then folded
    constexpr int kBatch = 4;
    float M = -INFINITY, L = 0.f;
    float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
    for (int k0 = 0; k0 < n_parts; k0 += kBatch) {
        float2 ml[kBatch];
        float4 o0[kBatch], o1[kBatch];
#pragma unroll
        for (int k = 0; k < kBatch; ++k) {
            ml[k] = make_float2(-INFINITY, 0.f);
            if (k0 + k < n_parts) {
                const size_t item = item_of(k0 + k);
                ml[k] = __ldcg(&part_ml[item * kPairRows + r]);
                o0[k] = __ldcg(&part_o[(item * 64 + c4a) * kPairRows + r]);
                o1[k] = __ldcg(&part_o[(item * 64 + c4a + 32) * kPairRows + r]);
            }
        }
        float mn = M;
#pragma unroll
        for (int k = 0; k < kBatch; ++k) mn = fmaxf(mn, ml[k].x);
        if (mn == -INFINITY) continue;  // nothing visible so far (l = 0, O = 0)
        const float sa = ex2(M - mn);   // 2^-inf = 0 before the first visible item
        M = mn;
        L *= sa;
        a0 = make_float4(a0.x * sa, a0.y * sa, a0.z * sa, a0.w * sa);
        a1 = make_float4(a1.x * sa, a1.y * sa, a1.z * sa, a1.w * sa);
#pragma unroll
        for (int k = 0; k < kBatch; ++k) {
            if (ml[k].x == -INFINITY) continue;  // absent, or nothing visible in that item
            const float w = ex2(ml[k].x - M);
            L = fmaf(ml[k].y, w, L);
            a0 = make_float4(fmaf(o0[k].x, w, a0.x), fmaf(o0[k].y, w, a0.y), fmaf(o0[k].z, w, a0.z),
                             fmaf(o0[k].w, w, a0.w));
            a1 = make_float4(fmaf(o1[k].x, w, a1.x), fmaf(o1[k].y, w, a1.y), fmaf(o1[k].z, w, a1.z),
                             fmaf(o1[k].w, w, a1.w));
        }
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    const float4 src[2] = {a0, a1};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int v0 = 4 * (c4a + 32 * h);
        orow[hq][v_real_dim(v0)] = src[h].x * inv;
        orow[hq][v_real_dim(v0 + 1)] = src[h].y * inv;
        orow[hq][v_real_dim(v0 + 2)] = src[h].z * inv;
        orow[hq][v_real_dim(v0 + 3)] = src[h].w * inv;
    }
    if (c4a == 0) lse_s[hq] = L > 0.f ? (M + log2f(L)) * 0.6931471805599453f : -INFINITY;
    __syncthreads();
#pragma unroll
    for (int h = 0; h < 8; ++h) {
        float o = orow[h][i];
        if (p.gate) o *= 1.f / (1.f + expf(-gs[h]));
        p.out[(static_cast<size_t>(t) * 16 + kvh * 8 + h) * 256 + i] = o;
    }
    if (p.lse && i < 8) p.lse[t * 16 + kvh * 8 + i] = lse_s[i];
}

// CTA pairs of the persistent grid for a request of n_ctas CTAs (0 = as many pairs as
// can be resident at once, at most one CTA per SM).
int pf_pairs(int n_ctas) {
    if (n_ctas > 0) return n_ctas >= 2 ? n_ctas / 2 : 1;
    static int resident = 0;
    if (resident == 0) {
        int pairs = sqmix_device_sm_count(-1) / 2;
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.gridDim = dim3(2 * pairs);
        cfg.blockDim = dim3(kPfThreads);
        cfg.dynamicSmemBytes = kSmemBytes;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaFuncSetAttribute(fa_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kSmemBytes)) == cudaSuccess &&
            cudaOccupancyMaxActiveClusters(&n, fa_prefill_kernel, &cfg) == cudaSuccess && n > 0 && n < pairs)
            pairs = n;
        cudaGetLastError();
        resident = pairs < 1 ? 1 : pairs;
    }
    return resident;
}

}  // namespace
}  // namespace sqmix

using namespace sqmix;

extern "C" size_t sqmix_fa_prefill_workspace_bytes(int32_t n_q, int32_t n_ctas) {
    const int n_pairs = pf_pairs(n_ctas);
    if (n_q < 1) n_q = 1;
    size_t a, b, c, total;
    pf_ws_layout(n_pairs, pf_n_mtiles(n_q), &a, &b, &c, &total);
    return total;
}

extern "C" int sqmix_fa_prefill(const sqmix_fa_args *a, sqmix_stream_t stream) {
    SQMIX_CHECK_ARG(a != nullptr, "fa_prefill: null args");
    SQMIX_CHECK_ARG(!a->q_norm && !a->k_norm,
                    "fa_prefill: q_norm / k_norm are decode-only; normalise with sqmix_head_norm first");
    SQMIX_CHECK_ARG(a->q && a->k_cache && a->v_cache && a->n_kv && a->q_pos0 && a->out && a->workspace,
                    "fa_prefill: null pointer argument");
    SQMIX_CHECK_ARG(a->n_q >= 1 && a->n_q <= 4096, "fa_prefill: n_q=%d (1..4096)", a->n_q);
    SQMIX_CHECK_ARG(a->q_dtype == SQMIX_F32 || a->q_dtype == SQMIX_F16 || a->q_dtype == SQMIX_BF16,
                    "fa_prefill: q dtype %d", a->q_dtype);
    SQMIX_CHECK_ARG(!a->gate || a->gate_dtype == SQMIX_F32 || a->gate_dtype == SQMIX_F16 ||
                        a->gate_dtype == SQMIX_BF16,
                    "fa_prefill: gate dtype %d", a->gate_dtype);
    SQMIX_CHECK_ARG(a->capacity > 0 && a->capacity % SQMIX_KV_PAD == 0, "fa_prefill: capacity");
    SQMIX_CHECK_ARG((reinterpret_cast<uintptr_t>(a->k_cache) & 15) == 0 &&
                        (reinterpret_cast<uintptr_t>(a->v_cache) & 15) == 0 &&
                        (reinterpret_cast<uintptr_t>(a->workspace) & 255) == 0,
                    "fa_prefill: caches must be 16-byte and the workspace 256-byte aligned");
    {
        const size_t esz = a->q_dtype == SQMIX_F32 ? 4 : 2;
        SQMIX_CHECK_ARG(reinterpret_cast<uintptr_t>(a->q) % (2 * esz) == 0 && a->q_stride_tok % 2 == 0 &&
                            a->q_stride_head % 2 == 0,
                        "fa_prefill: q must be aligned to two elements with even strides (element pairs are "
                        "read together)");
    }
    SQMIX_CHECK_ARG(a->scale > 0.f, "fa_prefill: scale must be positive");
    SQMIX_CHECK_ARG(a->rope_n_rot >= 0 && a->rope_n_rot <= 64 && a->rope_n_rot % 2 == 0 &&
                        (a->rope_n_rot == 0 || a->rope_freq_base > 0.f),
                    "fa_prefill: rope parameters (n_rot <= 64)");
    SQMIX_CHECK_ARG(a->n_new == 0, "fa_prefill: append the step's rows first (sqmix_kv_append_q4_0)");
    SQMIX_CHECK_ARG(a->n_splits >= 0 && a->n_splits <= 4096, "fa_prefill: n_splits (CTAs) = %d", a->n_splits);
    const int n_pairs = pf_pairs(a->n_splits);
    const size_t need = sqmix_fa_prefill_workspace_bytes(a->n_q, a->n_splits);
    if (a->workspace_bytes < need) {
        set_error("fa_prefill: workspace %zu bytes < %zu needed", a->workspace_bytes, need);
        return SQMIX_ENOSPC;
    }
    static std::atomic<uint64_t> attr_devices{0};
    {
        const cudaError_t e = set_smem_once(attr_devices, fa_prefill_kernel, static_cast<int>(kSmemBytes));
        if (e != cudaSuccess) return cuda_status(e, "fa_prefill smem attribute");
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    PfParams p;
    p.q = a->q;
    p.q_dtype = a->q_dtype;
    p.q_st = a->q_stride_tok;
    p.q_sh = a->q_stride_head;
    p.k_cache = static_cast<const uint8_t *>(a->k_cache);
    p.v_cache = static_cast<const uint8_t *>(a->v_cache);
    p.n_kv = a->n_kv;
    p.q_pos0 = a->q_pos0;
    p.capacity = a->capacity;
    p.T = a->n_q;
    p.n_mtiles = pf_n_mtiles(a->n_q);
    p.c = a->scale * 1.4426950408889634f;
    p.rope_n_rot = a->rope_n_rot;
    p.rope_theta_scale =
        a->rope_n_rot > 0 ? powf(a->rope_freq_base, -2.0f / static_cast<float>(a->rope_n_rot)) : 1.0f;
    p.rope_pos_offset = a->rope_pos_offset;
    p.ws = static_cast<uint8_t *>(a->workspace);
    p.items_max = pf_items_max(n_pairs, p.n_mtiles);
    {
        size_t ml, o, total;
        pf_ws_layout(n_pairs, p.n_mtiles, &ml, &o, &p.qimg_off, &total);
    }
    pf_prep_kernel<<<p.n_mtiles / 2 * kPairTok / 2 + 1, kPrepThreads, 0, st>>>(p, n_pairs);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_status(e, "fa_prefill prep launch");
    cudaLaunchAttribute pdl[1];
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
    {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * n_pairs);  // clusters of two (compile-time cluster dims)
        cfg.blockDim = dim3(kPfThreads);
        cfg.dynamicSmemBytes = kSmemBytes;
        cfg.stream = st;
        cfg.attrs = pdl;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, fa_prefill_kernel, p);
        if (e != cudaSuccess) return cuda_status(e, "fa_prefill launch");
    }
    PfMergeParams mp;
    mp.ws = p.ws;
    mp.items_max = p.items_max;
    mp.T = a->n_q;
    mp.gate = a->gate;
    mp.gate_dtype = a->gate_dtype;
    mp.g_st = a->gate_stride_tok;
    mp.g_sh = a->gate_stride_head;
    mp.out = a->out;
    mp.lse = a->lse;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a->n_q, 2);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cfg.attrs = pdl;
    cfg.numAttrs = 1;
    return cuda_status(cudaLaunchKernelEx(&cfg, fa_prefill_merge_kernel, mp), "fa_prefill merge launch");
}
