// FlashAttention prefill over the tiled q4_0 cache on the sm_100a tensor cores
// (tcgen05 / TMEM).  Replaces ggml_flash_attn_ext for T >= 1 query tokens
// (src/model/attn.rs:238-249) with the causal mask of src/model/graph.rs:553-559
// (query t sees keys j <= q_pos0 + t, j < n_kv), GQA 16 / 2 heads, head_dim 256,
// the partial RoPE of attn.rs:183-204 on Q and the sigmoid output gate of
// attn.rs:282-283.
//
// Work decomposition.  An M-tile is 16 query tokens x the 8 query heads of one KV
// head (128 rows, row r = 8 * token + head): the 8 heads share every K/V tile, so
// each dequantised tile feeds 128 rows.  An M-tile's key range is cut into items of
// L 64-key tiles (L chosen on the device so that there are about four items per
// CTA); a persistent grid of one CTA per SM takes items from a queue.  Each item
// leaves (m, l, O) partials per row; fa_prefill_merge_kernel combines the items of
// an M-tile, applies the gate and writes the output.  pf_setup_kernel builds the
// item table from the device scalars n_kv and q_pos0 (CUDA-graph friendly).
//
// One CTA (13 warps):
//   warp 0      TMEM allocation; lane 0 issues the MMAs: S = Q K^T (M 128, N 64,
//               K 256; Q read from tensor memory) into one of two TMEM S buffers,
//               then O += P V (M 128, N 256, K 64; P read from tensor memory) into
//               the TMEM O accumulator, in
//               the order S(0) S(1) PV(0) S(2) PV(1) ... so that the tensor core
//               computes the next S while the softmax warps work on the current one;
//   warps 1-4   softmax: thread = row; reads S from TMEM, online softmax in the
//               log2 domain with lazy rescaling (O is rescaled only when the row
//               maximum grows by more than 2^8), writes P (f16, two keys per
//               column) over the S buffer it has just read in tensor memory,
//               and at the end of an item reads O and writes the partials;
//   warps 5-12  producers: build Q (RoPE, f16) through a shared staging buffer into
//               tensor memory, and dequantise K and V tiles from q4_0 into
//               128-byte-swizzled shared memory (three stages; the raw q4_0 of the
//               next tile is loaded while the current one is converted).
// The contraction order of the head dimension is permuted so that each 16-byte
// chunk of the tiled cache dequantises into one 16-byte shared-memory chunk; Q uses
// the same permutation (K side) and the merge undoes the V-side one.
#include <math.h>

#include "common.cuh"
#include "sqmix.h"
#include "tc.cuh"

namespace sqmix {
namespace {

constexpr int kPfRows = 128;
constexpr int kPfTok = 16;
constexpr int kPfKeys = 64;
constexpr int kPfThreads = 13 * 32;
constexpr int kProdWarp0 = 5;
constexpr int kProdThreads = 256;
constexpr int kMaxMtiles = 512;  // T <= 4096

// shared memory (offsets from a 1024-byte aligned base)
constexpr int kNStage = 3;
constexpr uint32_t kStageOff = 0;       // 3 stages: K (4 x 8 KB regions) | V (4 x 8 KB)
constexpr uint32_t kStageBytes = 65536;
constexpr uint32_t kVInStage = 32768;
constexpr uint32_t kKvRegion = 8192;    // 64 keys x 128 B
constexpr uint32_t kPOff = 196608;      // Q staging buffer (128 rows x 512 B) at the
                                        // start of an item
constexpr uint32_t kRopeOff = 2 * kStageBytes + kVInStage;  // RoPE table while Q is built
constexpr uint32_t kBarOff = 229376;
constexpr uint32_t kSmemBytes = kBarOff + 256 + 1024;

// TMEM columns
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kOCol = 0;    // O: 256 columns f32
constexpr uint32_t kSCol = 256;  // S buffers: 2 x 64 columns
constexpr uint32_t kQCol = 384;  // Q: 128 columns (256 f16 per row, two per column)

constexpr float kRescaleLog2 = 8.0f;

// workspace layout
constexpr size_t kWsHeader = 256;  // [0] u32 err, [8] u32 queue, [12] u32 n_items, [16] u32 L
constexpr size_t kWsMtab = kWsHeader;                        // int4 per M-tile
constexpr size_t kWsItems = kWsMtab + kMaxMtiles * 16;       // int4 per item

__host__ __device__ inline size_t align256(size_t x) { return (x + 255) / 256 * 256; }
__host__ __device__ inline int pf_items_max(int n_ctas, int n_mtiles) { return 4 * n_ctas + n_mtiles + 1; }
__host__ __device__ inline void pf_ws_layout(int n_ctas, int n_mtiles, size_t *ml, size_t *o, size_t *total) {
    const size_t items = static_cast<size_t>(pf_items_max(n_ctas, n_mtiles));
    *ml = align256(kWsItems + items * 16);
    *o = align256(*ml + items * kPfRows * 2 * sizeof(float));
    *total = *o + items * kPfRows * 256 * sizeof(float);
}

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
};

__device__ __forceinline__ uint32_t *ws_err(uint8_t *ws) { return reinterpret_cast<uint32_t *>(ws); }
__device__ __forceinline__ uint32_t *ws_queue(uint8_t *ws) { return reinterpret_cast<uint32_t *>(ws + 8); }
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
__global__ void __launch_bounds__(kMaxMtiles) pf_setup_kernel(PfParams p, int n_ctas) {
    __shared__ int red[kMaxMtiles / 32];
    __shared__ int scan_a[kMaxMtiles], scan_b[kMaxMtiles];
    const int m = threadIdx.x;
    const int64_t n_kv = clamp_nkv(p, p.ws, m == 0);
    const int64_t q_pos0 = *p.q_pos0;
    int len = 0;  // 64-key tiles the M-tile sees
    if (m < p.n_mtiles) {
        int t_last = 16 * (m >> 1) + 15;
        if (t_last > p.T - 1) t_last = p.T - 1;
        int64_t lim = q_pos0 + t_last + 1;
        if (lim > n_kv) lim = n_kv;
        if (lim < 0) lim = 0;
        len = static_cast<int>((lim + kPfKeys - 1) / kPfKeys);
    }
    // total work W
    int v = len;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    int W = 0;
    for (int i = 0; i < kMaxMtiles / 32; ++i) W += red[i];
    int L = (W + 4 * n_ctas - 1) / (4 * n_ctas);
    if (L < 16) L = 16;
    const int nfull = len / L;
    const int rem = (len % L) > 0 ? 1 : 0;
    // inclusive scans (Hillis-Steele) of nfull and rem
    scan_a[m] = nfull;
    scan_b[m] = rem;
    __syncthreads();
    for (int off = 1; off < kMaxMtiles; off <<= 1) {
        const int a = m >= off ? scan_a[m - off] : 0;
        const int b = m >= off ? scan_b[m - off] : 0;
        __syncthreads();
        scan_a[m] += a;
        scan_b[m] += b;
        __syncthreads();
    }
    const int total_full = scan_a[kMaxMtiles - 1];
    const int total = total_full + scan_b[kMaxMtiles - 1];
    const int fbase = scan_a[m] - nfull;
    const int ritem = rem ? total_full + scan_b[m] - 1 : -1;
    int4 *mtab = reinterpret_cast<int4 *>(p.ws + kWsMtab);
    int4 *items = reinterpret_cast<int4 *>(p.ws + kWsItems);
    if (total > p.items_max) {  // cannot happen for L >= W / (4 n_ctas); guarded anyway
        if (m == 0) {
            atomicOr(ws_err(p.ws), 32u);
            *ws_nitems(p.ws) = 0;
            *ws_queue(p.ws) = 0;
        }
        if (m < p.n_mtiles) mtab[m] = make_int4(0, 0, -1, 0);
        return;
    }
    if (m < p.n_mtiles) {
        mtab[m] = make_int4(fbase, nfull, ritem, len);
        for (int k = 0; k < nfull; ++k) items[fbase + k] = make_int4(m, k * L, (k + 1) * L, 0);
        if (rem) items[ritem] = make_int4(m, nfull * L, len, 0);
    }
    if (m == 0) {
        *ws_nitems(p.ws) = static_cast<uint32_t>(total);
        *ws_queue(p.ws) = 0;
        reinterpret_cast<uint32_t *>(p.ws)[4] = static_cast<uint32_t>(L);
    }
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
__device__ __forceinline__ bool wait_or_abort(uint64_t *bar, uint32_t parity, volatile int *abort_flag,
                                              uint32_t *err, uint32_t bit) {
    if (*abort_flag) return false;
    if (mbar_wait(bar, parity)) return true;
    atomicOr(err, bit);
    *abort_flag = 1;
    return false;
}

// real head dimension of contraction (K-side) position p, 0..255
__device__ __forceinline__ int k_real_dim(int p) {
    const int i1 = p >> 7, c = (p >> 5) & 3, w = (p >> 3) & 3, e = p & 7;
    const int b = 4 * i1 + w;
    return 32 * b + 4 * c + (e & 3) + 16 * (e >> 2);
}
// real head dimension of output (V-side) column v, 0..255
__device__ __forceinline__ int v_real_dim(int v) {
    const int i = v >> 6, g = (v >> 3) & 7, w = (v >> 1) & 3, hi = v & 1;
    const int b = 2 * i + (w >> 1), m = w & 1;
    return 32 * b + 8 * m + g + 16 * hi;
}

struct SmemCtl {
    uint64_t kv_full[kNStage];
    uint64_t pv_done[kNStage];
    uint64_t s_full[2];
    uint64_t s_free[2];
    uint64_t p_full[2];
    uint64_t q_full;
    uint64_t o_free;
    uint64_t item_full[2];
    uint64_t item_empty[2];
    uint64_t final_bar;
    uint64_t rope_bar;
    uint64_t qs_bar;
    int4 item[2];
    uint32_t tmem_base;
    int abort_flag;
};
static_assert(sizeof(SmemCtl) <= 256, "control block");

// Raw q4_0 of one 64-key tile for one producer thread (2 K jobs + 2 V jobs).
struct RawTile {
    uint4 kn[2], vn[2], vs[2];
    uint2 ks[2];
};

__global__ void __launch_bounds__(kPfThreads, 1) fa_prefill_kernel(PfParams p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base_s = (raw + 1023u) & ~1023u;  // shared address of the aligned base
    uint8_t *base = smem_raw + (base_s - raw);
    SmemCtl *ctl = reinterpret_cast<SmemCtl *>(base + kBarOff);
    volatile int *abort_flag = &ctl->abort_flag;
    uint32_t *err = ws_err(p.ws);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kNStage; ++s) {
            mbar_init(&ctl->kv_full[s], kProdThreads);
            mbar_init(&ctl->pv_done[s], 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&ctl->s_full[s], 1);
            mbar_init(&ctl->s_free[s], kPfRows);
            mbar_init(&ctl->p_full[s], kPfRows);
            mbar_init(&ctl->item_full[s], 1);
            mbar_init(&ctl->item_empty[s], kPfThreads - 31);  // MMA lane + softmax + producers
        }
        mbar_init(&ctl->q_full, kProdThreads);
        mbar_init(&ctl->o_free, kPfRows);
        mbar_init(&ctl->final_bar, 1);
        mbar_init(&ctl->rope_bar, kProdThreads);
        mbar_init(&ctl->qs_bar, kProdThreads);
        ctl->abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tc::tmem_alloc(&ctl->tmem_base, kTmemCols);
        tc::tmem_relinquish();
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem = ctl->tmem_base;

    const int64_t n_kv = clamp_nkv(p, p.ws, false);
    const int64_t q_pos0 = *p.q_pos0;
    const int n_items = static_cast<int>(*ws_nitems(p.ws));
    const int4 *items = reinterpret_cast<const int4 *>(p.ws + kWsItems);
    const size_t ml_off = align256(kWsItems + static_cast<size_t>(p.items_max) * 16);
    const size_t o_off = align256(ml_off + static_cast<size_t>(p.items_max) * kPfRows * 2 * sizeof(float));
    float *part_ml = reinterpret_cast<float *>(p.ws + ml_off);
    float *part_o = reinterpret_cast<float *>(p.ws + o_off);

    // item ring: the producer leader fetches, every consumer thread copies and releases
    auto get_item = [&](int iter, int4 &it, bool leader) -> bool {
        const int slot = iter & 1;
        if (leader) {
            if (iter >= 2 && !wait_or_abort(&ctl->item_empty[slot], ((iter - 2) >> 1) & 1, abort_flag, err, 64u)) {
                it = make_int4(-1, 0, 0, -1);
                ctl->item[slot] = it;
                mbar_arrive(&ctl->item_full[slot]);
                return false;
            }
            const int q = static_cast<int>(atomicAdd(ws_queue(p.ws), 1u));
            int4 e = q < n_items ? items[q] : make_int4(-1, 0, 0, 0);
            e.w = q;
            ctl->item[slot] = e;
            mbar_arrive(&ctl->item_full[slot]);
        }
        if (!wait_or_abort(&ctl->item_full[slot], (iter >> 1) & 1, abort_flag, err, 64u)) return false;
        it = ctl->item[slot];
        mbar_arrive(&ctl->item_empty[slot]);
        return it.x >= 0;
    };
    // parity of the completion of tile jj on a barrier used once per kNStage tiles
    auto stage_parity = [](int jj) -> uint32_t { return static_cast<uint32_t>(jj / kNStage) & 1u; };

    const uint32_t idesc_s = tc::idesc_f16_f32(128, kPfKeys, 0, 0);
    const uint32_t idesc_pv = tc::idesc_f16_f32(128, 256, 0, 1);

    if (warp == 0) {
        // =========================== MMA issuer ===========================
        if (lane == 0) {
            int j = 0;
            bool ok = true;
            auto issue_s = [&](int jj) -> bool {
                const int sb = jj & 1, st = jj % kNStage;
                if (!wait_or_abort(&ctl->kv_full[st], stage_parity(jj), abort_flag, err, 1u)) return false;
                if (jj >= 2 && !wait_or_abort(&ctl->s_free[sb], ((jj - 2) >> 1) & 1, abort_flag, err, 1u))
                    return false;
                tc::fence_after();
#pragma unroll
                for (int ks = 0; ks < 16; ++ks) {
                    const uint64_t b = tc::desc_sw128(
                        base_s + kStageOff + st * kStageBytes + (ks >> 2) * kKvRegion + (ks & 3) * 32, 16, 1024);
                    tc::mma_ts(tmem + kSCol + sb * kPfKeys, tmem + kQCol + ks * 8, b, idesc_s, ks > 0 ? 1u : 0u);
                }
                tc::commit(&ctl->s_full[sb]);
                return true;
            };
            auto issue_pv = [&](int jj, bool first) -> bool {
                const int bb = jj & 1, st = jj % kNStage;
                if (!wait_or_abort(&ctl->p_full[bb], (jj >> 1) & 1, abort_flag, err, 1u)) return false;
                tc::fence_after();
#pragma unroll
                for (int ks = 0; ks < kPfKeys / 16; ++ks) {
                    // A = P (f16, two keys per column) in the first 32 columns of S buffer bb
                    const uint64_t b =
                        tc::desc_sw128(base_s + kStageOff + st * kStageBytes + kVInStage + ks * 2048, kKvRegion, 1024);
                    tc::mma_ts(tmem + kOCol, tmem + kSCol + bb * kPfKeys + ks * 8, b, idesc_pv,
                               (!first || ks > 0) ? 1u : 0u);
                }
                tc::commit(&ctl->pv_done[st]);
                return true;
            };
            for (int iter = 0; ok; ++iter) {
                int4 it;
                if (!get_item(iter, it, false)) break;
                const int n = it.z - it.y;
                if (!wait_or_abort(&ctl->q_full, iter & 1, abort_flag, err, 1u)) break;
                if (iter > 0 && !wait_or_abort(&ctl->o_free, (iter - 1) & 1, abort_flag, err, 1u)) break;
                tc::fence_after();
                const int jf = j;
                if (!issue_s(jf)) break;
                for (int t = 0; t < n; ++t) {
                    if (t + 1 < n && !issue_s(jf + t + 1)) { ok = false; break; }
                    if (!issue_pv(jf + t, t == 0)) { ok = false; break; }
                }
                j = jf + n;
            }
            // drain: every MMA issued so far completes before TMEM is released
            tc::commit(&ctl->final_bar);
            if (!mbar_wait(&ctl->final_bar, 0)) atomicOr(err, 128u);
        }
    } else if (warp < kProdWarp0) {
        // =========================== softmax ===========================
        const int r = 32 * (warp & 3) + lane;  // TMEM lane == row
        const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;
        // waits of a softmax warp end alike in all lanes: the tcgen05.ld/st that follow
        // are warp-collective
        auto wwait = [&](uint64_t *bar, uint32_t parity) -> bool {
            const bool r_ok = wait_or_abort(bar, parity, abort_flag, err, 2u);
            return __all_sync(0xffffffffu, r_ok);
        };
        int j = 0;
        for (int iter = 0;; ++iter) {
            int4 it;
            const bool got = get_item(iter, it, false);
            if (!__all_sync(0xffffffffu, got)) break;
            const int m = it.x, kt0 = it.y, kt1 = it.z, item = it.w;
            const int token = 16 * (m >> 1) + (r >> 3);
            int64_t lim = q_pos0 + token;
            if (lim > n_kv - 1) lim = n_kv - 1;
            if (token >= p.T) lim = -1;
            float m_run = -INFINITY, l_run = 0.f;
            bool ok = true;
            for (int kt = kt0; kt < kt1; ++kt, ++j) {
                const int b = j & 1;
                if (!wwait(&ctl->s_full[b], (j >> 1) & 1)) { ok = false; break; }
                tc::fence_after();
                uint32_t sr[2][32];
                tc::ld32(tmem + lane_base + kSCol + b * kPfKeys, sr[0]);
                tc::ld32(tmem + lane_base + kSCol + b * kPfKeys + 32, sr[1]);
                tc::fence_before();
                mbar_arrive(&ctl->s_free[b]);
                const int64_t key0 = static_cast<int64_t>(kt) * kPfKeys;
                float x[64];  // raw scores (scale applied below), -inf where masked
#pragma unroll
                for (int i = 0; i < 64; ++i) x[i] = __uint_as_float(sr[i >> 5][i & 31]);
                if (key0 + kPfKeys - 1 > lim) {
#pragma unroll
                    for (int i = 0; i < 64; ++i)
                        if (key0 + i > lim) x[i] = -INFINITY;
                }
                float mx[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) mx[i] = x[i];
#pragma unroll
                for (int i = 8; i < 64; ++i) mx[i & 7] = fmaxf(mx[i & 7], x[i]);
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
                    if (!wwait(&ctl->pv_done[jp % kNStage], stage_parity(jp))) {
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
                // p = 2^(c s - m): masked entries give 2^-inf = 0; a row with nothing
                // visible yet subtracts 0 instead of -inf
                const float msub = m_run == -INFINITY ? 0.f : m_run;
                float lsum[8];
                uint32_t ph[32];
#pragma unroll
                for (int i = 0; i < 64; i += 2) {
                    const float p0 = ex2(fmaf(x[i], p.c, -msub));
                    const float p1 = ex2(fmaf(x[i + 1], p.c, -msub));
                    lsum[(i >> 1) & 7] = (i < 16) ? p0 + p1 : lsum[(i >> 1) & 7] + (p0 + p1);
                    ph[i >> 1] = pack_half2(p0, p1);
                }
                l_run += ((lsum[0] + lsum[1]) + (lsum[2] + lsum[3])) + ((lsum[4] + lsum[5]) + (lsum[6] + lsum[7]));
                // P replaces S in the first 32 columns of S buffer b (read above).  The PV
                // of tile j - 2 that read the previous P there was issued before S(j),
                // and the MMAs of one thread run in issue order.
                tc::st32(tmem + lane_base + kSCol + b * kPfKeys, ph);
                tc::wait_st();
                tc::fence_before();
                mbar_arrive(&ctl->p_full[b]);
            }
            if (!ok) break;
            // ---- item epilogue: partial (m, l, O) of every row ----
            const int jl = j - 1;
            if (!wwait(&ctl->pv_done[jl % kNStage], stage_parity(jl))) break;
            tc::fence_after();
            float *orow = part_o + (static_cast<size_t>(item) * kPfRows + r) * 256;
#pragma unroll 1
            for (int ch = 0; ch < 8; ++ch) {
                uint32_t o[32];
                tc::ld32(tmem + lane_base + kOCol + ch * 32, o);
#pragma unroll
                for (int i = 0; i < 32; i += 4)
                    *reinterpret_cast<float4 *>(orow + ch * 32 + i) =
                        make_float4(__uint_as_float(o[i]), __uint_as_float(o[i + 1]), __uint_as_float(o[i + 2]),
                                    __uint_as_float(o[i + 3]));
            }
            tc::fence_before();
            mbar_arrive(&ctl->o_free);
            *reinterpret_cast<float2 *>(part_ml + (static_cast<size_t>(item) * kPfRows + r) * 2) =
                make_float2(m_run, l_run);
        }
    } else {
        // =========================== producers ===========================
        const int pt = threadIdx.x - kProdWarp0 * 32;  // 0..255
        const bool leader = pt == 0;
        float2 *rope_tab = reinterpret_cast<float2 *>(base + kRopeOff);  // 16 tokens x 32 pairs
        // TMEM rows this warp may write (its lane quarter) and which half of a staged block
        const int sp = warp & 3, hw = (warp - kProdWarp0) >> 2;
        int j = 0;
        uint32_t qph = 0;  // phases of qs_bar completed so far
        auto load_raw = [&](int kt, int kvh, RawTile &rw) {
            const int64_t key0 = static_cast<int64_t>(kt) * kPfKeys;
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int job = pt + kProdThreads * u;
                const int gi = job >> 7, ch = job & 127;
                const int i = ch >> 5, g = (ch >> 2) & 7, c = ch & 3;
                const int64_t unit = ((key0 / kGroupTokens + gi) * kHeadsKV + kvh) * kUnitBytes;
                rw.kn[u] = __ldg(reinterpret_cast<const uint4 *>(p.k_cache + unit + i * 512 + (4 * g + c) * 16));
                rw.ks[u] = __ldg(reinterpret_cast<const uint2 *>(p.k_cache + unit + kUnitQsBytes + g * 32 +
                                                                  (i >> 1) * 16 + 8 * (i & 1)));
                rw.vn[u] = __ldg(reinterpret_cast<const uint4 *>(p.v_cache + unit + i * 512 + (4 * g + c) * 16));
                rw.vs[u] = __ldg(reinterpret_cast<const uint4 *>(p.v_cache + unit + kUnitQsBytes + c * 64 + 16 * i));
            }
        };
        for (int iter = 0;; ++iter) {
            int4 it;
            if (!get_item(iter, it, leader)) break;
            const int m = it.x, kt0 = it.y, kt1 = it.z;
            const int kvh = m & 1;
            const int tok0 = 16 * (m >> 1);
            RawTile cur;
            load_raw(kt0, kvh, cur);  // first tile in flight while Q is built
            // previous item's MMAs are complete: Q (TMEM), stages and P buffers are free
            if (j > 0 && !wait_or_abort(&ctl->pv_done[(j - 1) % kNStage], stage_parity(j - 1), abort_flag, err, 4u))
                break;
            // ---- Q: RoPE, f16, contraction permutation; staged in shared memory, then
            // each thread moves its row's half into tensor memory ----
            const int half = p.rope_n_rot >> 1;
            for (int e = pt; e < kPfTok * 32; e += kProdThreads) {
                const int t = e >> 5, i = e & 31;
                rope_tab[e] = (i < half && tok0 + t < p.T)
                                  ? rope_cos_sin(q_pos0 + tok0 + t + p.rope_pos_offset, p.rope_theta_scale, i)
                                  : make_float2(1.f, 0.f);
            }
            // every producer's part of the RoPE table is written (bounded, unlike bar.sync)
            mbar_arrive(&ctl->rope_bar);
            if (!wait_or_abort(&ctl->rope_bar, iter & 1, abort_flag, err, 4u)) break;
            bool ok = true;
            for (int h = 0; h < 2 && ok; ++h) {
                // staging: 128 rows x 16 chunks (8 contraction positions each), 256 B per
                // row, chunk c of row r at position c ^ (r & 15)
#pragma unroll 4
                for (int job = pt; job < kPfRows * 16; job += kProdThreads) {
                    const int r = job >> 4, cl = job & 15, vc = h * 16 + cl;
                    const int token = tok0 + (r >> 3);
                    const int head = kvh * 8 + (r & 7);
                    uint32_t hv[4] = {0u, 0u, 0u, 0u};
                    if (token < p.T) {
                        const int64_t rbase = token * p.q_st + head * p.q_sh;
                        float v[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e)
                            v[e] = kv_row_elem(p.q, rbase, k_real_dim(vc * 8 + e), p.q_dtype, p.rope_n_rot,
                                               rope_tab + (r >> 3) * 32);
#pragma unroll
                        for (int e = 0; e < 4; ++e) hv[e] = pack_half2(v[2 * e], v[2 * e + 1]);
                    }
                    sts128(base_s + kPOff + r * 256 + ((cl ^ (r & 15)) << 4), make_uint4(hv[0], hv[1], hv[2], hv[3]));
                }
                mbar_arrive(&ctl->qs_bar);
                if (!wait_or_abort(&ctl->qs_bar, qph & 1, abort_flag, err, 4u)) { ok = false; break; }
                ++qph;
                {
                    const int r = 32 * sp + lane;
                    uint32_t qv[32];
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const int cl = hw * 8 + k;
                        uint4 x;
                        asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                                     : "=r"(x.x), "=r"(x.y), "=r"(x.z), "=r"(x.w)
                                     : "r"(base_s + kPOff + r * 256 + ((cl ^ (r & 15)) << 4)));
                        qv[4 * k] = x.x;
                        qv[4 * k + 1] = x.y;
                        qv[4 * k + 2] = x.z;
                        qv[4 * k + 3] = x.w;
                    }
                    tc::st32(tmem + (static_cast<uint32_t>(32 * sp) << 16) + kQCol + h * 64 + hw * 32, qv);
                    tc::wait_st();
                }
                if (h == 0) {  // the staging buffer is rewritten for the second half
                    mbar_arrive(&ctl->qs_bar);
                    if (!wait_or_abort(&ctl->qs_bar, qph & 1, abort_flag, err, 4u)) { ok = false; break; }
                    ++qph;
                }
            }
            if (!ok) break;
            tc::fence_before();
            mbar_arrive(&ctl->q_full);
            // ---- K / V tiles: the raw q4_0 of tile kt+1 is loaded while tile kt is converted ----
            for (int kt = kt0; kt < kt1; ++kt, ++j) {
                const int s = j % kNStage;
                RawTile nxt;
                if (kt + 1 < kt1) load_raw(kt + 1, kvh, nxt);
                const int64_t key0 = static_cast<int64_t>(kt) * kPfKeys;
                if (j >= kNStage &&
                    !wait_or_abort(&ctl->pv_done[s], stage_parity(j - kNStage), abort_flag, err, 4u)) {
                    ok = false;
                    break;
                }
                const uint32_t kst = base_s + kStageOff + s * kStageBytes;
                const uint32_t vst = kst + kVInStage;
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const int job = pt + kProdThreads * u;
                    const int gi = job >> 7, ch = job & 127;
                    const int i = ch >> 5, g = (ch >> 2) & 7, c = ch & 3;
                    // K: token row gi*16 + g + 8*(i>>1); blocks 4*(i&1) + w
                    {
                        const int row = gi * 16 + g + 8 * (i >> 1);
                        const bool live = key0 + row < n_kv;
                        const uint32_t w4[4] = {cur.kn[u].x, cur.kn[u].y, cur.kn[u].z, cur.kn[u].w};
                        const uint32_t d4[2] = {cur.ks[u].x, cur.ks[u].y};
                        const uint32_t rb = kst + ((i & 1) * 2 + (c >> 1)) * kKvRegion;
#pragma unroll
                        for (int w = 0; w < 4; ++w) {
                            uint4 outv = make_uint4(0u, 0u, 0u, 0u);
                            if (live) {
                                const __half2 dd = u32_as_h2(d4[w >> 1]);
                                const __half d1 = (w & 1) ? __high2half(dd) : __low2half(dd);
                                const __half2 d2 = __half2half2(d1);
                                const uint32_t lo = w4[w] & 0x0F0F0F0Fu;
                                const uint32_t hi = (w4[w] >> 4) & 0x0F0F0F0Fu;
                                outv = make_uint4(nib_pair(lo, 0x4140u, d2), nib_pair(lo, 0x4342u, d2),
                                                  nib_pair(hi, 0x4140u, d2), nib_pair(hi, 0x4342u, d2));
                            }
                            sts128(rb + swz(row, (c & 1) * 4 + w), outv);
                        }
                    }
                    // V: tokens {2c, 2c+8, 2c+1, 2c+9} (byte positions 0..3); blocks 2i + (w>>1)
                    {
                        const uint32_t w4[4] = {cur.vn[u].x, cur.vn[u].y, cur.vn[u].z, cur.vn[u].w};
                        const uint32_t d4[4] = {cur.vs[u].x, cur.vs[u].y, cur.vs[u].z, cur.vs[u].w};
                        const uint32_t rb = vst + i * kKvRegion;
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
                }
                tc::fence_proxy_async_smem();
                mbar_arrive(&ctl->kv_full[s]);
                if (kt + 1 < kt1) cur = nxt;
            }
            if (!ok) break;
        }
    }

    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    if (warp == 0) {
        __syncwarp();
        tc::tmem_dealloc(tmem, kTmemCols);
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

// grid (T, 2 KV heads), 256 threads: thread = output column (V-side order)
__global__ void __launch_bounds__(256) fa_prefill_merge_kernel(PfMergeParams p) {
    const int t = blockIdx.x, kvh = blockIdx.y, v = threadIdx.x;
    const int m = (t >> 4) * 2 + kvh;
    const int4 mt = reinterpret_cast<const int4 *>(p.ws + kWsMtab)[m];
    const size_t ml_off = align256(kWsItems + static_cast<size_t>(p.items_max) * 16);
    const size_t o_off = align256(ml_off + static_cast<size_t>(p.items_max) * kPfRows * 2 * sizeof(float));
    const float *part_ml = reinterpret_cast<const float *>(p.ws + ml_off);
    const float *part_o = reinterpret_cast<const float *>(p.ws + o_off);
    const int n_parts = mt.y + (mt.z >= 0 ? 1 : 0);
    const int dim = v_real_dim(v);
    for (int hq = 0; hq < 8; ++hq) {
        const int r = (t & 15) * 8 + hq;
        const int head = kvh * 8 + hq;
        float M = -INFINITY;
        for (int k = 0; k < n_parts; ++k) {
            const int item = k < mt.y ? mt.x + k : mt.z;
            M = fmaxf(M, __ldcg(part_ml + (static_cast<size_t>(item) * kPfRows + r) * 2));
        }
        float L = 0.f, acc = 0.f;
        if (M > -INFINITY) {
            for (int k = 0; k < n_parts; ++k) {
                const int item = k < mt.y ? mt.x + k : mt.z;
                const float2 ml = __ldcg(reinterpret_cast<const float2 *>(part_ml) + static_cast<size_t>(item) * kPfRows + r);
                const float w = ex2(ml.x - M);
                L += ml.y * w;
                acc += __ldcg(part_o + (static_cast<size_t>(item) * kPfRows + r) * 256 + v) * w;
            }
        }
        float o = L > 0.f ? acc / L : 0.f;
        if (p.gate) {
            const float gv = load_act(p.gate, t * p.g_st + head * p.g_sh + dim, p.gate_dtype);
            o *= 1.f / (1.f + expf(-gv));
        }
        p.out[(static_cast<size_t>(t) * 16 + head) * 256 + dim] = o;
        if (p.lse && v == 0)
            p.lse[t * 16 + head] = L > 0.f ? (M + log2f(L)) * 0.6931471805599453f : -INFINITY;
    }
}

}  // namespace
}  // namespace sqmix

using namespace sqmix;

extern "C" size_t sqmix_fa_prefill_workspace_bytes(int32_t n_q, int32_t n_ctas) {
    if (n_ctas <= 0) n_ctas = sqmix_device_sm_count(-1);
    if (n_q < 1) n_q = 1;
    const int n_mtiles = 2 * ((n_q + kPfTok - 1) / kPfTok);
    size_t a, b, total;
    pf_ws_layout(n_ctas, n_mtiles, &a, &b, &total);
    return total;
}

extern "C" int sqmix_fa_prefill(const sqmix_fa_args *a, sqmix_stream_t stream) {
    SQMIX_CHECK_ARG(a != nullptr, "fa_prefill: null args");
    SQMIX_CHECK_ARG(!a->q_norm && !a->k_norm,
                    "fa_prefill: q_norm / k_norm are decode-only; normalise with sqmix_head_norm first");
    SQMIX_CHECK_ARG(a->q && a->k_cache && a->v_cache && a->n_kv && a->q_pos0 && a->out && a->workspace,
                    "fa_prefill: null pointer argument");
    SQMIX_CHECK_ARG(a->n_q >= 1 && a->n_q <= kPfTok * kMaxMtiles / 2, "fa_prefill: n_q=%d (1..%d)", a->n_q,
                    kPfTok * kMaxMtiles / 2);
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
    SQMIX_CHECK_ARG(a->scale > 0.f, "fa_prefill: scale must be positive");
    SQMIX_CHECK_ARG(a->rope_n_rot >= 0 && a->rope_n_rot <= 64 && a->rope_n_rot % 2 == 0 &&
                        (a->rope_n_rot == 0 || a->rope_freq_base > 0.f),
                    "fa_prefill: rope parameters (n_rot <= 64)");
    SQMIX_CHECK_ARG(a->n_new == 0, "fa_prefill: append the step's rows first (sqmix_kv_append_q4_0)");
    const int n_ctas = a->n_splits > 0 ? a->n_splits : sqmix_device_sm_count(-1);
    SQMIX_CHECK_ARG(n_ctas >= 1 && n_ctas <= 4096, "fa_prefill: n_splits (CTAs) = %d", n_ctas);
    const size_t need = sqmix_fa_prefill_workspace_bytes(a->n_q, n_ctas);
    if (a->workspace_bytes < need) {
        set_error("fa_prefill: workspace %zu bytes < %zu needed", a->workspace_bytes, need);
        return SQMIX_ENOSPC;
    }
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(fa_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(kSmemBytes));
        if (e != cudaSuccess) return cuda_status(e, "fa_prefill smem attribute");
        attr_set = true;
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
    p.n_mtiles = 2 * ((a->n_q + kPfTok - 1) / kPfTok);
    p.c = a->scale * 1.4426950408889634f;
    p.rope_n_rot = a->rope_n_rot;
    p.rope_theta_scale =
        a->rope_n_rot > 0 ? powf(a->rope_freq_base, -2.0f / static_cast<float>(a->rope_n_rot)) : 1.0f;
    p.rope_pos_offset = a->rope_pos_offset;
    p.ws = static_cast<uint8_t *>(a->workspace);
    p.items_max = pf_items_max(n_ctas, p.n_mtiles);
    pf_setup_kernel<<<1, kMaxMtiles, 0, st>>>(p, n_ctas);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_status(e, "fa_prefill setup launch");
    fa_prefill_kernel<<<n_ctas, kPfThreads, kSmemBytes, st>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_status(e, "fa_prefill launch");
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
    fa_prefill_merge_kernel<<<dim3(a->n_q, 2), 256, 0, st>>>(mp);
    return cuda_status(cudaGetLastError(), "fa_prefill merge launch");
}
