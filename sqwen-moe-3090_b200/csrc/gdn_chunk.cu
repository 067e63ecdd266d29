// gdn_chunk.cu -- chunked gated delta net for prefill (ggml_gated_delta_net over T
// tokens, src/model/gdn.rs:489-500, recurrence gdn.rs:9-24), chunk size 64.
//
// Per token (one head, state S[i][j], key i, value j):
//     S <- e^{g_t} S;   delta_t = beta_t (v_t - S^T k_t);   S <- S + k_t delta_t^T;
//     o_t = S^T q_t / sqrt(128)
// Within a chunk of C tokens with cumulative log-decay G_t = g_1 + ... + g_t and the
// state S0 at the chunk start, the deltas solve a unit lower-triangular system
//     (I + A) Delta = diag(beta e^G) K (-S0) + diag(beta) V,
//     A_ts = beta_t e^{G_t - G_s} (k_t . k_s)            (s < t)
// so with W = (I + A)^-1 diag(beta e^G) K and U = (I + A)^-1 diag(beta) V:
//     Delta = U - W S0
//     O     = diag(e^G) Q S0 / sqrt(128) + (Q K^T o D) Delta / sqrt(128),
//             D_ts = e^{G_t - G_s} (s <= t)
//     S_C   = e^{G_C} S0 + (K o e^{G_C - G})^T Delta.
// gdn_chunk_prep_kernel computes everything that does not depend on the state (W, U,
// the scaled Q, K and the masked Q K^T) for all chunks and heads in parallel and
// stores the matrices the scan multiplies with as split-bf16 tcgen05 operand images;
// gdn_chunk_scan_kernel then walks the chunks of each head in order, one CTA per
// (sequence, head, 32 value columns; value columns evolve independently), with the
// three chunk products on the tensor cores (tcgen05, f32 accumulators in TMEM).
// Every exponent is a difference G_t - G_s <= 0 or G_t <= 0, so nothing overflows.
//
// Snapshot planes (slot s = state after T - s tokens, gdn.rs:484-538) are produced by
// running the last n_snap - 1 tokens through the recurrent kernel of gdn.cu.
#include <math.h>

#include "common.cuh"
#include "sqmix.h"
#include "tc.cuh"

namespace sqmix {

// gdn.cu: the recurrent kernel over tokens [tok_off, tok_off + n_tok) reading plane
// plane_in (< 0: the caller's sel / plane 0) and writing n_snap snapshot slots
int gdn_launch_recurrent(const sqmix_gdn_args *a, int plane_in, int64_t tok_off, int n_tok, int n_snap,
                         bool state_ready,
                         cudaStream_t st);

namespace {

constexpr int kC = 64;     // chunk length
constexpr int kD = 128;    // head dim
constexpr int kSN = 32;    // value columns per scan CTA
// Per (sequence, head, chunk) in the workspace.  The four chunk matrices the scan
// multiplies with are stored as bf16 pairs x = hi + lo (hi = bf16(x), lo = bf16(x - hi))
// in the shared-memory image of the tcgen05 operand layout, so that one bulk copy
// brings them in: 128-byte swizzle, row r at r * 128 bytes, 16-byte chunk q stored at
// q ^ (r & 7); MN-major images have blocks of 64 MN elements x rows of the contraction
// index.
//   A1 = [W ; Qs]  K-major: rows = tokens (W, then Qs; 128 rows), two regions of 64
//                  key dims (the same 128-byte swizzle, rows of the M index)
//   A3 = M         MN = token t, K = token s            (64 rows)
//   A4 = K'^T      MN = key index i (2 blocks), K = t   (64 rows)
// U stays f32 [64 t][128 j]; scalars: [0] e^{G_C}.
constexpr int64_t kA1Bytes = 2 * 2 * kD * 128;  // (hi | lo) x (W | Qs) blocks of 128 rows
constexpr int64_t kA3Bytes = 2 * kC * 128;      // (hi | lo) x one block of 64 rows
constexpr int64_t kA4Bytes = 2 * 2 * kC * 128;  // (hi | lo) x two blocks of 64 rows
constexpr int64_t kOffA1 = 0;                   // byte offsets in the chunk record
constexpr int64_t kOffA3 = kOffA1 + kA1Bytes;
constexpr int64_t kOffA4 = kOffA3 + kA3Bytes;
constexpr int64_t kOffUb = kOffA4 + kA4Bytes;   // U f32
constexpr int64_t kOffSb = kOffUb + kC * kD * 4;  // scalars
constexpr int64_t kChunkBytes = kOffSb + 256;
constexpr int64_t kChunkFloats = kChunkBytes / 4;
constexpr int64_t kWsHeaderFloats = 64;  // [0] u32 device status bits (bounded waits)

struct ChunkParams {
    const void *q, *k, *v;
    int dtype;
    int64_t qk_st, v_st, qk_sseq, v_sseq;
    const float *g, *beta;
    int n_seqs, T_all, T, h_k, h_v, n_chunks;
    int h_v_off;                   // layer index of value head 0 (value-head sharding)
    const float *dt_bias, *ssm_a;  // gate epilogue (ssm_a NULL: g, beta as given)
    float l2_eps;
    float *ws;
    float *state;
    int n_planes;
    const int32_t *sel;
    int plane_out;
    float *out;
};

__device__ __forceinline__ uint8_t *chunk_ws(const ChunkParams &p, int seq, int h, int c) {
    return reinterpret_cast<uint8_t *>(p.ws + kWsHeaderFloats +
                                       ((static_cast<int64_t>(seq) * p.h_v + h) * p.n_chunks + c) * kChunkFloats);
}

// bf16 pair of x: hi = bf16(x), lo = bf16(x - hi) (x = hi + lo to ~2^-16 relative)
__device__ __forceinline__ void split_bf16(float x, __nv_bfloat16 &hi, __nv_bfloat16 &lo) {
    hi = __float2bfloat16_rn(x);
    lo = __float2bfloat16_rn(x - __bfloat162float(hi));
}
// split_bf16 of two values at once, as packed words (a in the low half): the same
// roundings with paired conversions
__device__ __forceinline__ void split_bf16x2(float a, float b, uint32_t &hi, uint32_t &lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    const float2 hf = __bfloat1622float2(h);
    const __nv_bfloat162 l = __floats2bfloat162_rn(a - hf.x, b - hf.y);
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = *reinterpret_cast<const uint32_t *>(&l);
}
// One 64-element row r of an MN-major 128-byte-swizzled block, as hi and lo images
// (generic-proxy stores; the row is 128 bytes, chunk q at q ^ (r & 7)).
__device__ __forceinline__ void store_mn_row(uint8_t *blk_hi, uint8_t *blk_lo, int r, const float *v) {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        uint32_t h[4], l[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) split_bf16x2(v[8 * q + 2 * e], v[8 * q + 2 * e + 1], h[e], l[e]);
        const int off = r * 128 + ((q ^ (r & 7)) << 4);
        *reinterpret_cast<uint4 *>(blk_hi + off) = make_uint4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<uint4 *>(blk_lo + off) = make_uint4(l[0], l[1], l[2], l[3]);
    }
}

// ---- phase 1: state-independent chunk quantities -----------------------------------
// grid (n_chunks, h_v, n_seqs), 256 threads, dynamic smem kPrepSmem
constexpr int kLd = kD + 4;   // padded row stride of the [64][128] tiles
constexpr int kLdA = kC + 4;  // row stride of A (16-byte row quads)
// [K ; Q] as the split-bf16 K-major operand of the tcgen05 product [K ; Q] K^T: two
// regions (key dims 0..63, 64..127) of 128 rows (K tokens, then Q tokens) x 128 bytes,
// hi then lo; B = the first 64 rows (K) of the same image
constexpr int kKQImgBytes = 2 * 2 * 128 * 128;
constexpr size_t kPrepF32 = (3 * kC * kLd + kC * kLdA + kC * (kC + 1) + 4 * kC) * sizeof(float);
constexpr size_t kPrepImg = (kPrepF32 + 1023) / 1024 * 1024;
constexpr size_t kPrepSmem = kPrepImg + kKQImgBytes + 64 + 1024;  // + barrier, TMEM slot, alignment

__global__ void __launch_bounds__(256) gdn_chunk_prep_kernel(ChunkParams p) {
    extern __shared__ uint8_t prep_raw[];
    // q, k, v, g and beta come from the kernels before (programmatic dependent launch);
    // the trigger comes after the wait, so the scan may read what was written two
    // launches back (the state) before its own wait.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" :::);
    float *sm = reinterpret_cast<float *>((reinterpret_cast<uintptr_t>(prep_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *kq_img = reinterpret_cast<uint8_t *>(sm) + kPrepImg;
    uint64_t *mma_bar = reinterpret_cast<uint64_t *>(kq_img + kKQImgBytes);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(kq_img + kKQImgBytes + 32);
    float *Ks = sm;                  // [64][kLd]  k (L2-normalised)
    float *Qs = Ks + kC * kLd;       // [64][kLd]  q
    float *Vs = Qs + kC * kLd;       // [64][kLd]  v
    float *A = Vs + kC * kLd;        // [64][kLdA] (transposed) beta_t e^{G_t - G_s} k_t.k_s, s < t
    float *Mq = A + kC * kLdA;       // [64][65]   e^{G_t - G_s} q_t.k_s / sqrt(128), s <= t
    float *G = Mq + kC * (kC + 1);   // [64] cumulative log decay
    float *bt = G + kC;              // [64] beta
    float *gg = bt + kC;             // [64] g
    const int c = blockIdx.x, h = blockIdx.y, seq = blockIdx.z;
    const int hk = (p.h_v_off + h) % p.h_k;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t0 = c * kC;
    const int n_valid = min(kC, p.T - t0);

    // The raw gates of token tid, loaded with the rows below (one round trip for both).
    float graw = 0.f, braw = 0.f;
    if (tid < kC && tid < n_valid) {
        const int64_t gb = (static_cast<int64_t>(seq) * p.T_all + t0 + tid) * p.h_v + h;
        graw = p.g[gb];
        braw = p.beta[gb];
    }
    // rows: warp w loads rows w, w+8, ..., w+56.  The raw words of every row are loaded
    // before any is converted, so all 24 loads of a thread are in flight together.
    {
        float4 kk[8], qq[8], vv[8];
        const bool f32 = p.dtype == SQMIX_F32;
        uint4 rk[8], rq[8], rv[8];  // f32: the values; 16-bit types: the first 8 bytes
#pragma unroll
        for (int r = 0; r < 8; ++r) {
            const int t = warp + 8 * r;
            rk[r] = rq[r] = rv[r] = make_uint4(0u, 0u, 0u, 0u);
            if (t < n_valid) {
                const int64_t qk_off = seq * p.qk_sseq + (t0 + t) * p.qk_st + static_cast<int64_t>(hk) * kD + 4 * lane;
                const int64_t v_off = seq * p.v_sseq + (t0 + t) * p.v_st + static_cast<int64_t>(h) * kD + 4 * lane;
                if (f32) {
                    rk[r] = *reinterpret_cast<const uint4 *>(static_cast<const float *>(p.k) + qk_off);
                    rq[r] = *reinterpret_cast<const uint4 *>(static_cast<const float *>(p.q) + qk_off);
                    rv[r] = *reinterpret_cast<const uint4 *>(static_cast<const float *>(p.v) + v_off);
                } else {
                    const uint2 a = *reinterpret_cast<const uint2 *>(static_cast<const uint16_t *>(p.k) + qk_off);
                    const uint2 b = *reinterpret_cast<const uint2 *>(static_cast<const uint16_t *>(p.q) + qk_off);
                    const uint2 c2 = *reinterpret_cast<const uint2 *>(static_cast<const uint16_t *>(p.v) + v_off);
                    rk[r] = make_uint4(a.x, a.y, 0u, 0u);
                    rq[r] = make_uint4(b.x, b.y, 0u, 0u);
                    rv[r] = make_uint4(c2.x, c2.y, 0u, 0u);
                }
            }
        }
        auto cvt = [&](const uint4 &w) -> float4 {
            if (f32) return make_float4(__uint_as_float(w.x), __uint_as_float(w.y), __uint_as_float(w.z), __uint_as_float(w.w));
            if (p.dtype == SQMIX_BF16) {
                const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w.x));
                const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w.y));
                return make_float4(a.x, a.y, b.x, b.y);
            }
            const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&w.x));
            const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&w.y));
            return make_float4(a.x, a.y, b.x, b.y);
        };
#pragma unroll
        for (int r = 0; r < 8; ++r) {
            kk[r] = cvt(rk[r]);
            qq[r] = cvt(rq[r]);
            vv[r] = cvt(rv[r]);
        }
        // L2 norm factors of the 16 rows (q and k), the 5-step reductions interleaved
        float fk[8], fq[8];
        if (p.l2_eps > 0.f) {  // rms_norm(x, eps/n) * n^-1/2 (gdn.rs:133-142)
#pragma unroll
            for (int r = 0; r < 8; ++r) {
                fk[r] = kk[r].x * kk[r].x + kk[r].y * kk[r].y + kk[r].z * kk[r].z + kk[r].w * kk[r].w;
                fq[r] = qq[r].x * qq[r].x + qq[r].y * qq[r].y + qq[r].z * qq[r].z + qq[r].w * qq[r].w;
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1)
#pragma unroll
                for (int r = 0; r < 8; ++r) {
                    fk[r] += __shfl_xor_sync(0xffffffffu, fk[r], off);
                    fq[r] += __shfl_xor_sync(0xffffffffu, fq[r], off);
                }
            // every lane holds the 16 sums; lane i < 16 turns sum i (k rows, then q rows)
            // into its factor and the warp shares them (one square root and division per
            // lane instead of sixteen, the same arithmetic)
            const float r2 = 1.0f / sqrtf(128.0f);
            float mine = fk[0];
#pragma unroll
            for (int r = 0; r < 8; ++r) {
                mine = lane == r ? fk[r] : mine;
                mine = lane == 8 + r ? fq[r] : mine;
            }
            const float f = 1.0f / sqrtf(mine / 128.0f + p.l2_eps / 128.0f) * r2;
#pragma unroll
            for (int r = 0; r < 8; ++r) {
                fk[r] = __shfl_sync(0xffffffffu, f, r);
                fq[r] = __shfl_sync(0xffffffffu, f, 8 + r);
            }
        }
#pragma unroll
        for (int r = 0; r < 8; ++r) {
            const int t = warp + 8 * r;
            float4 k4 = kk[r], q4 = qq[r];
            if (p.l2_eps > 0.f && t < n_valid) {
                k4 = make_float4(k4.x * fk[r], k4.y * fk[r], k4.z * fk[r], k4.w * fk[r]);
                q4 = make_float4(q4.x * fq[r], q4.y * fq[r], q4.z * fq[r], q4.w * fq[r]);
            }
            *reinterpret_cast<float4 *>(Ks + t * kLd + 4 * lane) = k4;
            *reinterpret_cast<float4 *>(Qs + t * kLd + 4 * lane) = q4;
            *reinterpret_cast<float4 *>(Vs + t * kLd + 4 * lane) = vv[r];
            // dims 4 lane .. 4 lane + 3: region lane / 16, 16-byte chunk (lane % 16) / 2,
            // half (lane % 2); rows t (K) and 64 + t (Q)
            const float kx[4] = {k4.x, k4.y, k4.z, k4.w}, qx[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
            for (int which = 0; which < 2; ++which) {
                const float *xv = which ? qx : kx;
                const int row = t + 64 * which;
                uint32_t hw[2], lw[2];
#pragma unroll
                for (int e = 0; e < 2; ++e) split_bf16x2(xv[2 * e], xv[2 * e + 1], hw[e], lw[e]);
                const int off = (lane >> 4) * 16384 + row * 128 + ((((lane & 15) >> 1) ^ (row & 7)) << 4) + (lane & 1) * 8;
                *reinterpret_cast<uint2 *>(kq_img + off) = make_uint2(hw[0], hw[1]);
                *reinterpret_cast<uint2 *>(kq_img + kKQImgBytes / 2 + off) = make_uint2(lw[0], lw[1]);
            }
        }
    }
    if (tid < kC) {
        float gv = 0.f, bv = 0.f;
        if (tid < n_valid) {
            gv = graw;
            bv = braw;
            gdn_gates(gv, bv, p.dt_bias, p.ssm_a, p.h_v_off + h);
        }
        gg[tid] = gv;
        bt[tid] = bv;
    }
    __syncthreads();
    if (warp == 0) {  // inclusive scan of g over the chunk (two values per lane)
        float a0 = gg[2 * lane], a1 = gg[2 * lane + 1];
        float sc = a0 + a1;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const float y = __shfl_up_sync(0xffffffffu, sc, off);
            if (lane >= off) sc += y;
        }
        const float excl = sc - (a0 + a1);
        G[2 * lane] = excl + a0;
        G[2 * lane + 1] = excl + a0 + a1;
        // g is consumed: its slots now hold e^{G_t}
        gg[2 * lane] = expf(excl + a0);
        gg[2 * lane + 1] = expf(excl + a0 + a1);
    }
    __syncthreads();
    const float *eG = gg;

    // [K K^T ; Q K^T] = [K ; Q] K^T on the tensor cores (split bf16, f32 in TMEM), then
    // thread = row: A_ts = beta_t e^{G_t - G_s} k_t.k_s (s < t), Mq_ts = e^{G_t - G_s}
    // q_t.k_s / sqrt(128) (s <= t)
    if (tid == 0) {
        mbar_init(mma_bar, 1);
        fence_mbar_init();
    }
    if (warp == 0) tc::tmem_alloc(tmem_slot, 256);
    tc::fence_proxy_async_smem();  // the operand images (generic stores) -> tensor core
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t img = smem_u32(kq_img);
    const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;
    bool mok = true;
    if (tid == 0) {
        constexpr uint32_t idesc = tc::idesc_bf16_f32(128, kC, 0, 0);
#pragma unroll 1
        for (int ks = 0; ks < kD / 16; ++ks) {
            const uint32_t ko = (ks >> 2) * 16384 + (ks & 3) * 32;  // region, 16 dims within it
            const uint64_t ah = tc::desc_sw128(img + ko, 16, 1024);
            const uint64_t al = tc::desc_sw128(img + kKQImgBytes / 2 + ko, 16, 1024);
            tc::mma_ss(tmem, al, ah, idesc, ks > 0 ? 1u : 0u);
            tc::mma_ss(tmem, ah, al, idesc, 1u);
            tc::mma_ss(tmem, ah, ah, idesc, 1u);
        }
        tc::commit(mma_bar);
    }
    mok = mbar_wait(mma_bar, 0) && mok;
    tc::fence_after();
    float *At = A;  // [64 s][kLdA] holds A transposed: At[s][t] = A_ts
    if (warp < 4) {  // TMEM lanes 0..127 = rows: K K^T (0..63) into At, Q K^T (64..127) into Mq
        const int t = tid & 63;
        uint32_t raw[32];
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            tc::ld32(tmem + lane_base + 32 * hf, raw);
            if (tid < kC) {
#pragma unroll
                for (int i = 0; i < 32; ++i) At[(32 * hf + i) * kLdA + t] = __uint_as_float(raw[i]);
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) Mq[t * (kC + 1) + 32 * hf + i] = __uint_as_float(raw[i]);
            }
        }
    }
    tc::fence_before();
    __syncthreads();
    {  // decay, beta and the masks, 4 x 4 entries per thread
        const int tb = tid >> 4, sb = tid & 15;
        const float rsd = 1.0f / sqrtf(128.0f);
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int t = tb + 16 * a, s2 = sb + 16 * b;
                const float dec = s2 <= t ? expf(G[t] - G[s2]) : 0.f;
                At[s2 * kLdA + t] = s2 < t ? bt[t] * dec * At[s2 * kLdA + t] : 0.f;
                Mq[t * (kC + 1) + s2] = dec * Mq[t * (kC + 1) + s2] * rsd;
            }
    }
    // B = [diag(beta e^G) K | diag(beta) V] (K index s = token, N = 256) as the MN-major
    // split-bf16 image over the consumed [K ; Q] image: 4 blocks of 64 columns x 64 rows.
    // Warp w builds block w / 2, rows 32 (w % 2) + lane: the rows a quarter-warp reads
    // (stride kLd) and the 16-byte chunks it stores (swizzled by row) fall in distinct
    // banks (four lanes per row, one per block, hit the same banks four ways).
    {
        const int s2 = tid & 63, blk = tid >> 6;
        const float *src = blk < 2 ? Ks + s2 * kLd + 64 * blk : Vs + s2 * kLd + 64 * (blk - 2);
        const float f = bt[s2] * (blk < 2 ? eG[s2] : 1.f);
        float v[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) v[i] = src[i] * f;
        store_mn_row(kq_img + blk * kC * 128, kq_img + 4 * kC * 128 + blk * kC * 128, s2, v);
    }
    __syncthreads();  // A complete; V consumed (its space takes the T image below)
    // T = (I + A)^-1 by right-looking forward substitution: a warp solves 8 columns,
    // lane l holding rows l and l + 32 of each.  At step s, row s of every
    // column is final; it is broadcast from its lane and subtracted, times A_ts, from
    // all rows t (A_ts = 0 for t <= s, so earlier rows are unchanged).  A is read
    // transposed (At[s][t]: conflict-free).  Column j of T is row j of the MN-major
    // image of T (K index j, M = t), written as split bf16.
    uint8_t *t_img = reinterpret_cast<uint8_t *>(Vs);  // hi 8 KB | lo 8 KB (1024-aligned)
    {
        const int l = lane;
        // column block of this warp: warps w and w + 4 (one scheduler) take blocks w and
        // 7 - w, whose chains (63 - 8 block steps) add up to the same length on every
        // scheduler
        const int cb = warp < 4 ? warp : 11 - warp;
        float x[8][2];
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
            const int col = 8 * cb + cc;
            x[cc][0] = l == col ? 1.f : 0.f;
            x[cc][1] = l + 32 == col ? 1.f : 0.f;
        }
        // Steps that change nothing are skipped (the chain of columns 8b .. 8b + 7 starts at
        // row 8b: the rows above are zero; from step 32 on, rows < 32 are final since
        // A_ts = 0 for t < s), so block b takes 63 - 8b steps and the second half updates
        // one row per lane.  The skipped updates would add exact zeros.
        const int s_first = 8 * cb;
#pragma unroll 2
        for (int s2 = s_first; s2 < 32; ++s2) {
            const float a0 = At[s2 * kLdA + l], a1 = At[s2 * kLdA + l + 32];
#pragma unroll
            for (int cc = 0; cc < 8; ++cc) {
                const float xs = __shfl_sync(0xffffffffu, x[cc][0], s2);
                x[cc][0] = fmaf(-a0, xs, x[cc][0]);
                x[cc][1] = fmaf(-a1, xs, x[cc][1]);
            }
        }
#pragma unroll 2
        for (int s2 = s_first > 32 ? s_first : 32; s2 < kC - 1; ++s2) {
            const float a1 = At[s2 * kLdA + l + 32];
#pragma unroll
            for (int cc = 0; cc < 8; ++cc) {
                const float xs = __shfl_sync(0xffffffffu, x[cc][1], s2 - 32);
                x[cc][1] = fmaf(-a1, xs, x[cc][1]);
            }
        }
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
            const int col = 8 * cb + cc;
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int t = l + 32 * e;
                __nv_bfloat16 vh, vl;
                split_bf16(x[cc][e], vh, vl);
                const int off = col * 128 + ((((t >> 3) ^ (col & 7)) & 7) << 4) + (t & 7) * 2;
                *reinterpret_cast<__nv_bfloat16 *>(t_img + off) = vh;
                *reinterpret_cast<__nv_bfloat16 *>(t_img + kC * 128 + off) = vl;
            }
        }
    }
    tc::fence_proxy_async_smem();
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    // [W | U] = T B: M 128 (rows 64..127 read the bytes after T and are ignored), N 256,
    // K 64, into TMEM columns 0..255
    if (tid == 0) {
        constexpr uint32_t idesc = tc::idesc_bf16_f32(128, 256, 1, 1);
        const uint32_t timg = smem_u32(t_img);
#pragma unroll 1
        for (int ks = 0; ks < kC / 16; ++ks) {
            const uint32_t ko = ks * 2048;
            const uint64_t ah = tc::desc_sw128(timg + ko, kC * 128, 1024);
            const uint64_t al = tc::desc_sw128(timg + kC * 128 + ko, kC * 128, 1024);
            const uint64_t bh = tc::desc_sw128(img + ko, kC * 128, 1024);
            const uint64_t bl = tc::desc_sw128(img + 4 * kC * 128 + ko, kC * 128, 1024);
            tc::mma_ss(tmem, al, bh, idesc, ks > 0 ? 1u : 0u);
            tc::mma_ss(tmem, ah, bl, idesc, 1u);
            tc::mma_ss(tmem, ah, bh, idesc, 1u);
        }
        tc::commit(mma_bar);
    }
    mok = mbar_wait(mma_bar, 1) && mok;
    if (!mok && tid == 0) atomicOr(reinterpret_cast<uint32_t *>(p.ws), 8u);
    tc::fence_after();

    // ---- epilogue: the chunk record --------------------------------------------------
    //   warps 0, 1: W rows t (TMEM lanes 0..63, columns 0..127) -> A1 rows t (K-major)
    //   warps 4, 5: U rows t (TMEM lanes 0..63, columns 128..255) -> U f32
    //   warps 2, 3: Qs rows t -> A1 rows 64 + t;  warps 6, 7: K' rows t (A4);
    //   warps 4, 5 also M rows s (A3), so that no warp converts more than two row images
    uint8_t *wsc = chunk_ws(p, seq, h, c);
    float *Ub = reinterpret_cast<float *>(wsc + kOffUb);
    const float GC = G[kC - 1];
    if (warp == 0 || warp == 1 || warp == 4 || warp == 5) {
        const int t = tid & 63;
        const int cb = warp < 4 ? 0 : 128;
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {  // 64 columns at a time
            float v[64];
            uint32_t raw[32];
            tc::ld32(tmem + lane_base + cb + 64 * hf, raw);
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(raw[i]);
            tc::ld32(tmem + lane_base + cb + 64 * hf + 32, raw);
#pragma unroll
            for (int i = 0; i < 32; ++i) v[32 + i] = __uint_as_float(raw[i]);
            if (cb == 0) {
                store_mn_row(wsc + kOffA1 + hf * 16384, wsc + kOffA1 + kA1Bytes / 2 + hf * 16384, t, v);
            } else {
                float4 *urow = reinterpret_cast<float4 *>(Ub + t * kD + 64 * hf);
#pragma unroll
                for (int q = 0; q < 16; ++q) urow[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
            }
        }
        if (cb != 0) {  // warps 4, 5 (U needs no conversion): M rows s (A3) as well
            float v[kC];
#pragma unroll
            for (int t2 = 0; t2 < kC; ++t2) v[t2] = Mq[t2 * (kC + 1) + t];
            store_mn_row(wsc + kOffA3, wsc + kOffA3 + kA3Bytes / 2, t, v);
        }
    } else if (warp == 2 || warp == 3) {
        const int t = tid - 64;
        const float f = eG[t] * (1.0f / sqrtf(128.0f));
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            float v[64];
#pragma unroll
            for (int i = 0; i < 64; ++i) v[i] = Qs[t * kLd + 64 * hf + i] * f;
            store_mn_row(wsc + kOffA1 + hf * 16384, wsc + kOffA1 + kA1Bytes / 2 + hf * 16384, 64 + t, v);
        }
    } else {
        const int t = tid - 192;
        const float dk = expf(GC - G[t]);
#pragma unroll
        for (int blk = 0; blk < 2; ++blk) {
            float v[64];
#pragma unroll
            for (int i = 0; i < 64; ++i) v[i] = Ks[t * kLd + 64 * blk + i] * dk;
            store_mn_row(wsc + kOffA4 + blk * kC * 128, wsc + kOffA4 + kA4Bytes / 2 + blk * kC * 128, t, v);
        }
    }
    if (tid == 0) reinterpret_cast<float *>(wsc + kOffSb)[0] = expf(GC);
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    if (warp == 0) {
        if (!mok) {  // never release TMEM under a running MMA
            tc::commit(mma_bar);
            mbar_wait(mma_bar, 0);
        }
        tc::tmem_dealloc(tmem, 256);
    }
}

// ---- phase 2: walk the chunks of one (sequence, head, 32 value columns) -------------
// grid (kD / kSN, h_v, n_seqs), 128 threads (thread = TMEM lane = accumulator row,
// all kSN columns of it); dynamic smem kScanSmem.  Per chunk, three split-bf16 tcgen05 MMA groups (hi*hi + hi*lo + lo*hi,
// f32 accumulators in tensor memory):
//   D1  = [W ; Qs] S0          M 128 (tokens of W, then of Qs; A K-major), N 32, K 128
//   Delta = U - D1[0:64]       (rows 0..63, written back as the bf16 B operand)
//   D1 += [0 ; M] Delta        (the O half: O = Qs S0 + M Delta)
//   D4  = K'^T Delta           M 128 (key index), N 32, K 64
//   S  <- e^{G_C} S0 + D4      (thread i keeps row i of the f32 state block in registers)
// The operand images of chunk c+1 are brought in by 1-D bulk copies (TMA, no
// multicast) as soon as the MMAs of chunk c have read the buffers.
constexpr uint32_t kSmA1 = 0;                                   // 64 KB: hi | lo, each 2 regions
constexpr uint32_t kSmA3 = kSmA1 + kA1Bytes;                    // 32 KB: hi | lo, each zero | M
constexpr uint32_t kSmA4 = kSmA3 + 2 * kA3Bytes;                // 32 KB: hi | lo
// B operands K-major (rows = the kSN value columns j, 128-byte rows of 64 contraction
// elements, same swizzle): S0 (K = key index i: 2 regions of kSN rows) and Delta
// (K = token t: 1 region)
constexpr uint32_t kBSRegion = kSN * 128;
constexpr uint32_t kSmBS = kSmA4 + kA4Bytes;                    // 8 KB: hi | lo
constexpr uint32_t kSmBD = kSmBS + 2 * 2 * kBSRegion;           // 4 KB: hi | lo
constexpr uint32_t kSmBar = kSmBD + 2 * kBSRegion;
constexpr size_t kScanSmem = kSmBar + 64 + 1024;                // + alignment slack
constexpr uint32_t kTmemCols = 2 * kSN;                          // D1 at 0, D4 at kSN

// Column kidx (contraction index) of a K-major block whose rows are the kSN value
// columns: v[j] -> row j, as split bf16 (2-byte stores; a warp's 32 consecutive kidx
// fill 64 contiguous bytes of a row).
__device__ __forceinline__ void store_k_col(uint8_t *hi, uint8_t *lo, uint32_t region_bytes, int kidx,
                                            const float *v) {
    const uint32_t base = (kidx >> 6) * region_bytes + (kidx & 7) * 2;
    const int q = (kidx & 63) >> 3;
#pragma unroll
    for (int j = 0; j < kSN; ++j) {
        __nv_bfloat16 vh, vl;
        split_bf16(v[j], vh, vl);
        const uint32_t off = base + j * 128 + ((q ^ (j & 7)) << 4);
        *reinterpret_cast<__nv_bfloat16 *>(hi + off) = vh;
        *reinterpret_cast<__nv_bfloat16 *>(lo + off) = vl;
    }
}

__device__ __forceinline__ void ld32f(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    tc::ld32(taddr, r);
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__global__ void __launch_bounds__(128) gdn_chunk_scan_kernel(ChunkParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sb = smem_u32(sm);
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + kSmBar);  // [0] A1, [1] A3|A4, [2] MMA done
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sm + kSmBar + 32);
    __shared__ int abort_flag;
    uint32_t *err = reinterpret_cast<uint32_t *>(p.ws);
    const int jb = blockIdx.x, h = blockIdx.y, seq = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5;
    auto issue_a1 = [&](int c) {
        const uint8_t *w = chunk_ws(p, seq, h, c);
        mbar_arrive_expect_tx(&bars[0], static_cast<uint32_t>(kA1Bytes));
        bulk_g2s(sm + kSmA1, w + kOffA1, static_cast<uint32_t>(kA1Bytes), &bars[0]);
    };
    auto issue_a34 = [&](int c) {
        const uint8_t *w = chunk_ws(p, seq, h, c);
        mbar_arrive_expect_tx(&bars[1], static_cast<uint32_t>(kA3Bytes + kA4Bytes));
        // M into the second (non-zero) block of each of A3's hi and lo halves
        bulk_g2s(sm + kSmA3 + kA3Bytes / 2, w + kOffA3, static_cast<uint32_t>(kA3Bytes / 2), &bars[1]);
        bulk_g2s(sm + kSmA3 + kA3Bytes + kA3Bytes / 2, w + kOffA3 + kA3Bytes / 2, static_cast<uint32_t>(kA3Bytes / 2),
                 &bars[1]);
        bulk_g2s(sm + kSmA4, w + kOffA4, static_cast<uint32_t>(kA4Bytes), &bars[1]);
    };
    // A3's first block (rows of tokens that receive no M Delta: the W half of D1) is zero
    for (int e = tid; e < static_cast<int>(kA3Bytes / 2 / 16); e += 128) {
        reinterpret_cast<uint4 *>(sm + kSmA3)[e] = make_uint4(0u, 0u, 0u, 0u);
        reinterpret_cast<uint4 *>(sm + kSmA3 + kA3Bytes)[e] = make_uint4(0u, 0u, 0u, 0u);
    }
    if (tid == 0) {
        for (int i = 0; i < 3; ++i) mbar_init(&bars[i], 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0) tc::tmem_alloc(tmem_slot, kTmemCols);
    tc::fence_proxy_async_smem();
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem = *tmem_slot;
    const int row = tid;  // accumulator row (TMEM lane)
    const uint32_t lane_base = static_cast<uint32_t>(32 * warp) << 16;
    // row i = row of the state block, columns j0 .. j0 + kSN - 1: S[i][j] at ((h*128 + j)*128 + i).
    // The state and sel were written two or more launches back (the prep kernel triggers
    // this launch only after its own dependency wait): read before this kernel's wait.
    const int64_t plane_elems = static_cast<int64_t>(p.h_v) * kD * kD;
    float *st_seq = p.state + static_cast<int64_t>(seq) * p.n_planes * plane_elems;
    int plane = p.sel ? p.sel[seq] : 0;
    plane = min(max(plane, 0), p.n_planes - 1);
    const int j0 = jb * kSN;
    float srow[kSN];
#pragma unroll
    for (int j = 0; j < kSN; ++j) srow[j] = st_seq[plane * plane_elems + (static_cast<int64_t>(h) * kD + j0 + j) * kD + row];
    store_k_col(sm + kSmBS, sm + kSmBS + 2 * kBSRegion, kBSRegion, row, srow);
    // the chunk records come from the prep kernel
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" :::);
    if (tid == 0) {
        issue_a1(0);
        issue_a34(0);
    }

    constexpr uint32_t idesc = tc::idesc_bf16_f32(128, kSN, 1, 0);
    // split-bf16 products: (A hi, B hi), (A hi, B lo), (A lo, B hi); A MN-major, B the
    // K-major Delta (one region: 16 contraction elements = 32 bytes per step)
    auto mma3 = [&](uint32_t d, uint32_t a, uint32_t a_lo, uint32_t a_lbo, uint32_t b, uint32_t b_lo, int ksteps,
                    bool accumulate) {
#pragma unroll 1
        for (int ks = 0; ks < ksteps; ++ks) {
            const uint32_t ko = ks * 2048;  // 16 rows of the contraction index
            const uint64_t ah = tc::desc_sw128(a + ko, a_lbo, 1024), al = tc::desc_sw128(a + a_lo + ko, a_lbo, 1024);
            const uint64_t bh = tc::desc_sw128(b + ks * 32, 16, 1024), bl = tc::desc_sw128(b + b_lo + ks * 32, 16, 1024);
            tc::mma_ss(d, al, bh, idesc, (accumulate || ks > 0) ? 1u : 0u);
            tc::mma_ss(d, ah, bl, idesc, 1u);
            tc::mma_ss(d, ah, bh, idesc, 1u);
        }
    };
    bool ok = true;
    int mma_phase = 0;
    int last_a1 = 0, last_a34 = 0;  // chunk of the latest copies issued (thread 0)
    // every thread takes the same branch after a wait (the loop has block barriers)
    auto wait_bar = [&](uint64_t *bar, uint32_t parity, uint32_t bit) -> bool {
        bool r = !abort_flag;
        if (r && !mbar_wait(bar, parity)) {
            atomicOr(err, bit);
            abort_flag = 1;
            r = false;
        }
        return __syncthreads_and(r) != 0;
    };
    tc::fence_proxy_async_smem();
    __syncthreads();
    for (int c = 0; c < p.n_chunks && ok; ++c) {
        const uint8_t *wsc = chunk_ws(p, seq, h, c);
        const float eGC = reinterpret_cast<const float *>(wsc + kOffSb)[0];
        float u[kSN];
        if (row < kC) {
            const float4 *ur = reinterpret_cast<const float4 *>(wsc + kOffUb + (static_cast<int64_t>(row) * kD + j0) * 4);
#pragma unroll
            for (int q = 0; q < kSN / 4; ++q) {
                const float4 x = ur[q];
                u[4 * q] = x.x;
                u[4 * q + 1] = x.y;
                u[4 * q + 2] = x.z;
                u[4 * q + 3] = x.w;
            }
        }
        if (!wait_bar(&bars[0], c & 1, 1u)) { ok = false; break; }
        // ---- D1 = [W ; Qs] S0 ----
        if (tid == 0) {  // A1 is K-major: region ks / 4, 16 key dims within it
            tc::fence_after();
            constexpr uint32_t idesc1 = tc::idesc_bf16_f32(128, kSN, 0, 0);
#pragma unroll 1
            for (int ks = 0; ks < kD / 16; ++ks) {
                const uint32_t ka = (ks >> 2) * 16384 + (ks & 3) * 32, kb = (ks >> 2) * kBSRegion + (ks & 3) * 32;
                const uint64_t ah = tc::desc_sw128(sb + kSmA1 + ka, 16, 1024);
                const uint64_t al = tc::desc_sw128(sb + kSmA1 + kA1Bytes / 2 + ka, 16, 1024);
                const uint64_t bh = tc::desc_sw128(sb + kSmBS + kb, 16, 1024);
                const uint64_t bl = tc::desc_sw128(sb + kSmBS + 2 * kBSRegion + kb, 16, 1024);
                tc::mma_ss(tmem, al, bh, idesc1, ks > 0 ? 1u : 0u);
                tc::mma_ss(tmem, ah, bl, idesc1, 1u);
                tc::mma_ss(tmem, ah, bh, idesc1, 1u);
            }
            tc::commit(&bars[2]);
        }
        if (!wait_bar(&bars[2], mma_phase++ & 1, 2u)) { ok = false; break; }
        tc::fence_after();
        if (tid == 0 && c + 1 < p.n_chunks) {  // A1 has been read
            issue_a1(c + 1);
            last_a1 = c + 1;
        }
        // ---- Delta = U - W S0 (rows t = 0..63) as the bf16 B operand ----
        if (row < kC) {  // warps 0, 1
            float d[kSN];
            ld32f(tmem + lane_base, d);
#pragma unroll
            for (int j = 0; j < kSN; ++j) d[j] = u[j] - d[j];
            store_k_col(sm + kSmBD, sm + kSmBD + kBSRegion, kBSRegion, row, d);
        }
        tc::fence_proxy_async_smem();
        tc::fence_before();
        if (!wait_bar(&bars[1], c & 1, 4u)) { ok = false; break; }
        // ---- D1 += [0 ; M] Delta ;  D4 = K'^T Delta ----
        if (tid == 0) {
            tc::fence_after();
            mma3(tmem, sb + kSmA3, static_cast<uint32_t>(kA3Bytes), static_cast<uint32_t>(kA3Bytes / 2), sb + kSmBD,
                 kBSRegion, kC / 16, true);
            mma3(tmem + kSN, sb + kSmA4, static_cast<uint32_t>(kA4Bytes / 2), kC * 128, sb + kSmBD, kBSRegion, kC / 16,
                 false);
            tc::commit(&bars[2]);
        }
        if (!wait_bar(&bars[2], mma_phase++ & 1, 2u)) { ok = false; break; }
        tc::fence_after();
        if (tid == 0 && c + 1 < p.n_chunks) {  // A3 and A4 have been read
            issue_a34(c + 1);
            last_a34 = c + 1;
        }
        // ---- outputs O (rows 64..127 of D1 = tokens 0..63) ----
        if (row >= kC) {  // warps 2, 3
            const int t = c * kC + (row - kC);
            float o[kSN];
            ld32f(tmem + lane_base, o);
            if (t < p.T) {
                float4 *orow = reinterpret_cast<float4 *>(
                    p.out + ((static_cast<int64_t>(seq) * p.T_all + t) * p.h_v + h) * kD + j0);
#pragma unroll
                for (int q = 0; q < kSN / 4; ++q) orow[q] = make_float4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
            }
        }
        // ---- S = e^{G_C} S0 + K'^T Delta (row i = tid) ----
        {
            float d4[kSN];
            ld32f(tmem + lane_base + kSN, d4);
#pragma unroll
            for (int j = 0; j < kSN; ++j) srow[j] = fmaf(eGC, srow[j], d4[j]);
            store_k_col(sm + kSmBS, sm + kSmBS + 2 * kBSRegion, kBSRegion, row, srow);
        }
        tc::fence_proxy_async_smem();
        tc::fence_before();
        __syncthreads();
    }
    if (!ok) {
        // never exit with a bulk copy still writing into shared memory, nor before the
        // issued MMAs are complete (their tensor memory is released below)
        if (tid == 0) {
            mbar_wait(&bars[0], last_a1 & 1);
            mbar_wait(&bars[1], last_a34 & 1);
            tc::commit(&bars[2]);
            mbar_wait(&bars[2], mma_phase & 1);
        }
    } else {
#pragma unroll
        for (int j = 0; j < kSN; ++j)
            st_seq[p.plane_out * plane_elems + (static_cast<int64_t>(h) * kD + j0 + j) * kD + row] = srow[j];
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    if (warp == 0) tc::tmem_dealloc(tmem, kTmemCols);
}

}  // namespace
}  // namespace sqmix

using namespace sqmix;

extern "C" size_t sqmix_gdn_prefill_workspace_bytes(int32_t n_seqs, int32_t n_tokens, int32_t h_v) {
    if (n_seqs < 1 || n_tokens < 1 || h_v < 1) return 0;
    const int64_t n_chunks = (n_tokens + kC - 1) / kC;
    return (kWsHeaderFloats + static_cast<size_t>(n_seqs) * h_v * n_chunks * kChunkFloats) * sizeof(float);
}

extern "C" int sqmix_gdn_prefill(const sqmix_gdn_args *a, void *workspace, size_t workspace_bytes,
                                 sqmix_stream_t stream) {
    SQMIX_CHECK_ARG(a != nullptr, "gdn_prefill: null args");
    SQMIX_CHECK_ARG(a->q && a->k && a->v && a->g && a->beta && a->state && a->out && workspace,
                    "gdn_prefill: null pointer argument");
    SQMIX_CHECK_ARG(a->dtype == SQMIX_F32 || a->dtype == SQMIX_F16 || a->dtype == SQMIX_BF16,
                    "gdn_prefill: dtype %d", a->dtype);
    SQMIX_CHECK_ARG(a->h_k >= 1 && a->h_v >= 1 && a->h_v_offset >= 0, "gdn_prefill: h_k=%d h_v=%d h_v_offset=%d",
                    a->h_k, a->h_v, a->h_v_offset);
    SQMIX_CHECK_ARG(a->n_seqs >= 1 && a->n_seqs <= 65535 && a->n_tokens >= 1, "gdn_prefill: n_seqs=%d T=%d",
                    a->n_seqs, a->n_tokens);
    SQMIX_CHECK_ARG(a->n_planes >= 1, "gdn_prefill: n_planes=%d", a->n_planes);
    SQMIX_CHECK_ARG(a->n_snap >= 1 && a->n_snap <= a->n_tokens && a->n_snap <= a->n_planes,
                    "gdn_prefill: n_snap=%d must be in [1, min(T=%d, n_planes=%d)]", a->n_snap, a->n_tokens,
                    a->n_planes);
    SQMIX_CHECK_ARG(a->qk_stride_tok >= (int64_t)a->h_k * 128 && a->v_stride_tok >= (int64_t)a->h_v * 128,
                    "gdn_prefill: token strides too small");
    SQMIX_CHECK_ARG((reinterpret_cast<uintptr_t>(a->state) & 15) == 0 &&
                        (reinterpret_cast<uintptr_t>(workspace) & 15) == 0,
                    "gdn_prefill: state and workspace must be 16-byte aligned");
    SQMIX_CHECK_ARG(a->qk_stride_tok % 4 == 0 && a->qk_stride_seq % 4 == 0 && a->v_stride_tok % 4 == 0 &&
                        a->v_stride_seq % 4 == 0,
                    "gdn_prefill: q/k/v strides must be multiples of 4 elements");
    {
        const uintptr_t align = a->dtype == SQMIX_F32 ? 15 : 7;
        SQMIX_CHECK_ARG(((reinterpret_cast<uintptr_t>(a->q) | reinterpret_cast<uintptr_t>(a->k) |
                          reinterpret_cast<uintptr_t>(a->v)) & align) == 0,
                        "gdn_prefill: q/k/v base pointers must be %d-byte aligned", (int)align + 1);
    }
    const size_t need = sqmix_gdn_prefill_workspace_bytes(a->n_seqs, a->n_tokens, a->h_v);
    if (workspace_bytes < need) {
        set_error("gdn_prefill: workspace %zu bytes < %zu needed", workspace_bytes, need);
        return SQMIX_ENOSPC;
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    // tokens [0, T_chunk) go through the chunked form, the last n_snap - 1 through the
    // recurrent kernel, which writes the snapshot slots
    const int T_chunk = a->n_tokens - (a->n_snap - 1);
    static std::atomic<uint64_t> prep_devices{0}, scan_devices{0};
    {
        cudaError_t e = set_smem_once(prep_devices, gdn_chunk_prep_kernel, static_cast<int>(kPrepSmem));
        if (e == cudaSuccess) e = set_smem_once(scan_devices, gdn_chunk_scan_kernel, static_cast<int>(kScanSmem));
        if (e != cudaSuccess) return cuda_status(e, "gdn_prefill smem attribute");
    }
    ChunkParams p;
    p.q = a->q;
    p.k = a->k;
    p.v = a->v;
    p.dtype = a->dtype;
    p.qk_st = a->qk_stride_tok;
    p.v_st = a->v_stride_tok;
    p.qk_sseq = a->qk_stride_seq;
    p.v_sseq = a->v_stride_seq;
    p.g = a->g;
    p.beta = a->beta;
    p.h_v_off = a->h_v_offset;
    p.dt_bias = a->dt_bias;
    p.ssm_a = a->ssm_a;
    p.n_seqs = a->n_seqs;
    p.T_all = a->n_tokens;
    p.T = T_chunk;
    p.h_k = a->h_k;
    p.h_v = a->h_v;
    p.n_chunks = (T_chunk + kC - 1) / kC;
    p.l2_eps = a->l2_eps;
    p.ws = static_cast<float *>(workspace);
    p.state = a->state;
    p.n_planes = a->n_planes;
    p.sel = a->sel;
    p.plane_out = a->n_snap - 1;
    p.out = a->out;
    // both kernels with programmatic stream serialisation: the prep overlaps the tail of
    // the kernel before it, the scan's set-up and state load the prep's last CTAs
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.n_chunks, a->h_v, a->n_seqs);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = kPrepSmem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, gdn_chunk_prep_kernel, p);
    if (e != cudaSuccess) return cuda_status(e, "gdn_prefill prep launch");
    cfg.gridDim = dim3(kD / kSN, a->h_v, a->n_seqs);
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = kScanSmem;
    e = cudaLaunchKernelEx(&cfg, gdn_chunk_scan_kernel, p);
    if (e != cudaSuccess) return cuda_status(e, "gdn_prefill scan launch");
    if (a->n_snap > 1)
        // the tail reads the plane the scan kernel just wrote: no early state read
        return gdn_launch_recurrent(a, a->n_snap - 1, T_chunk, a->n_snap - 1, a->n_snap - 1, false, st);
    return SQMIX_OK;
}
