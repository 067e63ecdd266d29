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
// the scaled Q, K and the masked Q K^T) for all chunks and heads in parallel;
// gdn_chunk_scan_kernel then walks the chunks of each head in order, one CTA per
// (sequence, head, 32 value columns): value columns evolve independently.
// Every exponent is a difference G_t - G_s <= 0 or G_t <= 0, so nothing overflows.
//
// Snapshot planes (slot s = state after T - s tokens, gdn.rs:484-538) are produced by
// running the last n_snap - 1 tokens through the recurrent kernel of gdn.cu.
#include <math.h>

#include "common.cuh"
#include "sqmix.h"

namespace sqmix {

// gdn.cu: the recurrent kernel over tokens [tok_off, tok_off + n_tok) reading plane
// plane_in (< 0: the caller's sel / plane 0) and writing n_snap snapshot slots
int gdn_launch_recurrent(const sqmix_gdn_args *a, int plane_in, int64_t tok_off, int n_tok, int n_snap,
                         cudaStream_t st);

namespace {

constexpr int kC = 64;     // chunk length
constexpr int kD = 128;    // head dim
constexpr int kJB = 32;    // value columns per scan CTA
// per (sequence, head, chunk) in the workspace, in floats; W, Q and M are stored
// transposed (contraction index major) so that the scan reads 4 rows per vector load
constexpr int64_t kOffW = 0;                // W^T  [128 i][64 t]
constexpr int64_t kOffU = kOffW + kC * kD;  // U    [64 t][128 j]
constexpr int64_t kOffQ = kOffU + kC * kD;  // Qs^T [128 i][64 t]  q e^G / sqrt(128)
constexpr int64_t kOffK = kOffQ + kC * kD;  // K'   [64 t][128 i]  k e^{G_C - G}
constexpr int64_t kOffM = kOffK + kC * kD;  // M^T  [64 s][64 t]   (Q K^T o D)^T / sqrt(128)
constexpr int64_t kOffS = kOffM + kC * kC;  // scalars: [0] e^{G_C}
constexpr int64_t kChunkFloats = kOffS + 64;
constexpr int64_t kWsHeaderFloats = 64;  // [0] u32 device status bits (bounded waits)

struct ChunkParams {
    const void *q, *k, *v;
    int dtype;
    int64_t qk_st, v_st, qk_sseq, v_sseq;
    const float *g, *beta;
    int n_seqs, T_all, T, h_k, h_v, n_chunks;
    float l2_eps;
    float *ws;
    float *state;
    int n_planes;
    const int32_t *sel;
    int plane_out;
    float *out;
};

__device__ __forceinline__ float warp_sum32(float x) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
    return x;
}

// 4 consecutive elements of a q/k/v row (offset a multiple of 4) as f32
__device__ __forceinline__ float4 load4v(const void *p, int64_t i, int dtype) {
    if (dtype == SQMIX_F32) return *reinterpret_cast<const float4 *>(static_cast<const float *>(p) + i);
    const uint2 r = *reinterpret_cast<const uint2 *>(static_cast<const uint16_t *>(p) + i);
    if (dtype == SQMIX_BF16) {
        const __nv_bfloat162 x = *reinterpret_cast<const __nv_bfloat162 *>(&r.x);
        const __nv_bfloat162 y = *reinterpret_cast<const __nv_bfloat162 *>(&r.y);
        return make_float4(__low2float(x), __high2float(x), __low2float(y), __high2float(y));
    }
    const __half2 x = *reinterpret_cast<const __half2 *>(&r.x);
    const __half2 y = *reinterpret_cast<const __half2 *>(&r.y);
    return make_float4(__low2float(x), __high2float(x), __low2float(y), __high2float(y));
}

__device__ __forceinline__ float *chunk_ws(const ChunkParams &p, int seq, int h, int c) {
    return p.ws + kWsHeaderFloats + ((static_cast<int64_t>(seq) * p.h_v + h) * p.n_chunks + c) * kChunkFloats;
}

// ---- phase 1: state-independent chunk quantities -----------------------------------
// grid (n_chunks, h_v, n_seqs), 256 threads, dynamic smem kPrepSmem
constexpr int kLd = kD + 4;   // padded row stride of the [64][128] tiles
constexpr int kLdA = kC + 4;  // row stride of A (16-byte row quads)
constexpr size_t kPrepSmem = (3 * kC * kLd + kC * kLdA + kC * (kC + 1) + 4 * kC) * sizeof(float);

__global__ void __launch_bounds__(256) gdn_chunk_prep_kernel(ChunkParams p) {
    extern __shared__ __align__(16) float sm[];
    float *Ks = sm;                  // [64][kLd]  k (L2-normalised)
    float *Qs = Ks + kC * kLd;       // [64][kLd]  q
    float *Vs = Qs + kC * kLd;       // [64][kLd]  v
    float *A = Vs + kC * kLd;        // [64][kLdA] beta_t e^{G_t - G_s} k_t.k_s, s < t (0 elsewhere)
    float *Mq = A + kC * kLdA;       // [64][65]   e^{G_t - G_s} q_t.k_s / sqrt(128), s <= t
    float *G = Mq + kC * (kC + 1);   // [64] cumulative log decay
    float *bt = G + kC;              // [64] beta
    float *gg = bt + kC;             // [64] g
    const int c = blockIdx.x, h = blockIdx.y, seq = blockIdx.z;
    const int hk = h % p.h_k;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t0 = c * kC;
    const int n_valid = min(kC, p.T - t0);

    // rows: warp w loads rows w, w+8, ..., w+56 (all loads issued before use)
    {
        float4 kk[8], qq[8], vv[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) {
            const int t = warp + 8 * r;
            kk[r] = qq[r] = vv[r] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (t < n_valid) {
                const int64_t qk_off = seq * p.qk_sseq + (t0 + t) * p.qk_st + static_cast<int64_t>(hk) * kD + 4 * lane;
                const int64_t v_off = seq * p.v_sseq + (t0 + t) * p.v_st + static_cast<int64_t>(h) * kD + 4 * lane;
                kk[r] = load4v(p.k, qk_off, p.dtype);
                qq[r] = load4v(p.q, qk_off, p.dtype);
                vv[r] = load4v(p.v, v_off, p.dtype);
            }
        }
#pragma unroll
        for (int r = 0; r < 8; ++r) {
            const int t = warp + 8 * r;
            float4 k4 = kk[r], q4 = qq[r];
            if (p.l2_eps > 0.f && t < n_valid) {  // rms_norm(x, eps/n) * n^-1/2 (gdn.rs:133-142)
                const float sk = warp_sum32(k4.x * k4.x + k4.y * k4.y + k4.z * k4.z + k4.w * k4.w);
                const float sq = warp_sum32(q4.x * q4.x + q4.y * q4.y + q4.z * q4.z + q4.w * q4.w);
                const float r2 = 1.0f / sqrtf(128.0f);
                const float fk = 1.0f / sqrtf(sk / 128.0f + p.l2_eps / 128.0f) * r2;
                const float fq = 1.0f / sqrtf(sq / 128.0f + p.l2_eps / 128.0f) * r2;
                k4 = make_float4(k4.x * fk, k4.y * fk, k4.z * fk, k4.w * fk);
                q4 = make_float4(q4.x * fq, q4.y * fq, q4.z * fq, q4.w * fq);
            }
            *reinterpret_cast<float4 *>(Ks + t * kLd + 4 * lane) = k4;
            *reinterpret_cast<float4 *>(Qs + t * kLd + 4 * lane) = q4;
            *reinterpret_cast<float4 *>(Vs + t * kLd + 4 * lane) = vv[r];
        }
    }
    if (tid < kC) {
        const int64_t gb = (static_cast<int64_t>(seq) * p.T_all + t0 + tid) * p.h_v + h;
        gg[tid] = tid < n_valid ? p.g[gb] : 0.f;
        bt[tid] = tid < n_valid ? p.beta[gb] : 0.f;
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
    }
    __syncthreads();

    // K K^T and Q K^T, 4x4 outputs per thread: rows tb + 16a, columns sb + 16b
    {
        const int tb = tid >> 4, sb = tid & 15;
        float kk[4][4] = {}, qk[4][4] = {};
#pragma unroll 4
        for (int i = 0; i < kD; ++i) {
            float kt[4], qt[4], ks[4];
#pragma unroll
            for (int a = 0; a < 4; ++a) {
                kt[a] = Ks[(tb + 16 * a) * kLd + i];
                qt[a] = Qs[(tb + 16 * a) * kLd + i];
                ks[a] = Ks[(sb + 16 * a) * kLd + i];
            }
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    kk[a][b] = fmaf(kt[a], ks[b], kk[a][b]);
                    qk[a][b] = fmaf(qt[a], ks[b], qk[a][b]);
                }
        }
        const float rsd = 1.0f / sqrtf(128.0f);
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int t = tb + 16 * a, s2 = sb + 16 * b;
                const float dec = s2 <= t ? expf(G[t] - G[s2]) : 0.f;
                A[t * kLdA + s2] = s2 < t ? bt[t] * dec * kk[a][b] : 0.f;
                Mq[t * (kC + 1) + s2] = dec * qk[a][b] * rsd;
            }
    }
    __syncthreads();
    float *wsc = chunk_ws(p, seq, h, c);
    // forward substitution of (I + A) X = [beta e^G K | beta V], one thread per column,
    // the column held in registers; A_ts = 0 for s >= t, so whole 4-groups are summed
    {
        const int col = tid & 127;
        const bool is_w = tid < kD;
        const float *src = is_w ? Ks : Vs;
        float x[kC];
#pragma unroll
        for (int t = 0; t < kC; ++t) x[t] = src[t * kLd + col] * bt[t] * (is_w ? expf(G[t]) : 1.f);
#pragma unroll
        for (int t = 1; t < kC; ++t) {
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int s4 = 0; s4 < t; s4 += 4) {
                const float4 a = *reinterpret_cast<const float4 *>(A + t * kLdA + s4);
                float &ac = acc[(s4 >> 2) & 3];
                ac = fmaf(a.x, x[s4], ac);
                ac = fmaf(a.y, x[s4 + 1], ac);
                ac = fmaf(a.z, x[s4 + 2], ac);
                ac = fmaf(a.w, x[s4 + 3], ac);
            }
            x[t] -= (acc[0] + acc[1]) + (acc[2] + acc[3]);
        }
        if (is_w) {  // W^T row col: 64 contiguous floats
#pragma unroll
            for (int t = 0; t < kC; t += 4)
                *reinterpret_cast<float4 *>(wsc + kOffW + col * kC + t) = make_float4(x[t], x[t + 1], x[t + 2], x[t + 3]);
        } else {
#pragma unroll
            for (int t = 0; t < kC; ++t) wsc[kOffU + t * kD + col] = x[t];
        }
    }
    // Qs^T (threads 0..127) and K' (threads 128..255), from the tiles still in shared memory
    {
        const float GC = G[kC - 1];
        const int col = tid & 127;
        if (tid < kD) {
            const float rsd = 1.0f / sqrtf(128.0f);
#pragma unroll 4
            for (int t = 0; t < kC; t += 4) {
                float4 v;
                v.x = Qs[t * kLd + col] * expf(G[t]) * rsd;
                v.y = Qs[(t + 1) * kLd + col] * expf(G[t + 1]) * rsd;
                v.z = Qs[(t + 2) * kLd + col] * expf(G[t + 2]) * rsd;
                v.w = Qs[(t + 3) * kLd + col] * expf(G[t + 3]) * rsd;
                *reinterpret_cast<float4 *>(wsc + kOffQ + col * kC + t) = v;
            }
        } else {
            for (int t = 0; t < kC; ++t) wsc[kOffK + t * kD + col] = Ks[t * kLd + col] * expf(GC - G[t]);
        }
        for (int e = tid; e < kC * kC; e += 256) wsc[kOffM + e] = Mq[(e & 63) * (kC + 1) + (e >> 6)];
        if (tid == 0) wsc[kOffS] = expf(GC);
    }
}

// ---- phase 2: walk the chunks of one (sequence, head, 32 value columns) -------------
// grid (kD / kJB, h_v, n_seqs), 256 threads, dynamic smem kScanSmem.  The chunk tiles
// are brought in by 1-D bulk copies (TMA, no multicast): W^T and Q^T of chunk c+1 as
// soon as chunk c has used them, M^T and K' likewise.
constexpr int kLdS = kJB + 2;  // S and Delta rows (float2 column pairs)
constexpr size_t kScanFloats = static_cast<size_t>(kD) * kLdS + kC * kLdS + 3 * kD * kC + kC * kC;
constexpr size_t kScanSmem = kScanFloats * sizeof(float) + 64;
constexpr uint32_t kBytesWQ = 2 * kD * kC * sizeof(float);
constexpr uint32_t kBytesMK = (kC * kC + kC * kD) * sizeof(float);

__global__ void __launch_bounds__(256) gdn_chunk_scan_kernel(ChunkParams p) {
    extern __shared__ __align__(16) float sm[];
    float *S = sm;                  // [128 i][kLdS]  state columns of this block
    float *Dl = S + kD * kLdS;      // [64 t][kLdS]   Delta
    float *WT = Dl + kC * kLdS;     // [128 i][64 t]
    float *QT = WT + kD * kC;       // [128 i][64 t]  (contiguous after WT: one W|Q copy pair)
    float *MT = QT + kD * kC;       // [64 s][64 t]
    float *Kp = MT + kC * kC;       // [64 t][128 i]  (contiguous after MT)
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + kScanFloats);  // [0] W|Q, [1] M|K'
    __shared__ int abort_flag;
    uint32_t *err = reinterpret_cast<uint32_t *>(p.ws);
    const int jb = blockIdx.x, h = blockIdx.y, seq = blockIdx.z;
    const int tid = threadIdx.x;
    auto issue_wq = [&](int c) {
        const float *w = chunk_ws(p, seq, h, c);
        mbar_arrive_expect_tx(&bars[0], kBytesWQ);
        bulk_g2s(WT, w + kOffW, kD * kC * sizeof(float), &bars[0]);
        bulk_g2s(QT, w + kOffQ, kD * kC * sizeof(float), &bars[0]);
    };
    auto issue_mk = [&](int c) {
        const float *w = chunk_ws(p, seq, h, c);
        mbar_arrive_expect_tx(&bars[1], kBytesMK);
        bulk_g2s(MT, w + kOffM, kC * kC * sizeof(float), &bars[1]);
        bulk_g2s(Kp, w + kOffK, kC * kD * sizeof(float), &bars[1]);
    };
    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {
        issue_wq(0);
        issue_mk(0);
    }
    const int64_t plane_elems = static_cast<int64_t>(p.h_v) * kD * kD;
    float *st_seq = p.state + static_cast<int64_t>(seq) * p.n_planes * plane_elems;
    int plane = p.sel ? p.sel[seq] : 0;
    plane = min(max(plane, 0), p.n_planes - 1);
    // S[i][j] at ((h*128 + j)*128 + i)
    for (int e = tid; e < kD * kJB; e += 256) {
        const int j = e >> 7, i = e & 127;
        S[i * kLdS + j] = st_seq[plane * plane_elems + (static_cast<int64_t>(h) * kD + jb * kJB + j) * kD + i];
    }
    __syncthreads();
    // Delta / O tiles: rows r0..r0+3 (tokens), columns c0, c0+1; S tile: rows i0..i0+7
    const int r0 = 4 * (tid >> 4), c0 = 2 * (tid & 15);
    const int i0 = 8 * (tid >> 4);
    bool ok = true;
    int last_wq = 0, last_mk = 0;  // chunk of the latest copies issued (thread 0)
    // every thread takes the same branch after a wait (the loop has block barriers)
    auto wait = [&](int which, int c) -> bool {
        bool r = !abort_flag;
        if (r && !mbar_wait(&bars[which], c & 1)) {
            atomicOr(err, 1u);
            abort_flag = 1;
            r = false;
        }
        return __syncthreads_and(r) != 0;
    };
    int c = 0;
    for (; c < p.n_chunks; ++c) {
        const float *wsc = chunk_ws(p, seq, h, c);
        const float eGC = wsc[kOffS];
        float2 u[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) u[a] = *reinterpret_cast<const float2 *>(wsc + kOffU + (r0 + a) * kD + jb * kJB + c0);
        if (!wait(0, c)) { ok = false; break; }
        // Delta = U - W S0 and the first part of O = Qs S0
        float d[4][2], o[4][2];
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            d[a][0] = u[a].x;
            d[a][1] = u[a].y;
            o[a][0] = o[a][1] = 0.f;
        }
#pragma unroll 4
        for (int i = 0; i < kD; ++i) {
            const float2 sv = *reinterpret_cast<const float2 *>(S + i * kLdS + c0);
            const float4 w = *reinterpret_cast<const float4 *>(WT + i * kC + r0);
            const float4 q = *reinterpret_cast<const float4 *>(QT + i * kC + r0);
            const float wv[4] = {w.x, w.y, w.z, w.w}, qv[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int a = 0; a < 4; ++a) {
                d[a][0] = fmaf(-wv[a], sv.x, d[a][0]);
                d[a][1] = fmaf(-wv[a], sv.y, d[a][1]);
                o[a][0] = fmaf(qv[a], sv.x, o[a][0]);
                o[a][1] = fmaf(qv[a], sv.y, o[a][1]);
            }
        }
#pragma unroll
        for (int a = 0; a < 4; ++a) *reinterpret_cast<float2 *>(Dl + (r0 + a) * kLdS + c0) = make_float2(d[a][0], d[a][1]);
        __syncthreads();  // Delta complete; S0, W and Q fully read
        if (tid == 0 && c + 1 < p.n_chunks) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue_wq(c + 1);
            last_wq = c + 1;
        }
        if (!wait(1, c)) { ok = false; break; }
        // O += M Delta
#pragma unroll 4
        for (int s2 = 0; s2 < kC; ++s2) {
            const float2 dv = *reinterpret_cast<const float2 *>(Dl + s2 * kLdS + c0);
            const float4 m = *reinterpret_cast<const float4 *>(MT + s2 * kC + r0);
            const float mv[4] = {m.x, m.y, m.z, m.w};
#pragma unroll
            for (int a = 0; a < 4; ++a) {
                o[a][0] = fmaf(mv[a], dv.x, o[a][0]);
                o[a][1] = fmaf(mv[a], dv.y, o[a][1]);
            }
        }
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            const int t = c * kC + r0 + a;
            if (t < p.T)
                *reinterpret_cast<float2 *>(p.out + ((static_cast<int64_t>(seq) * p.T_all + t) * p.h_v + h) * kD +
                                            jb * kJB + c0) = make_float2(o[a][0], o[a][1]);
        }
        // S = e^{G_C} S0 + K'^T Delta (each thread rewrites only its own entries)
        {
            float acc[8][2];
#pragma unroll
            for (int a = 0; a < 8; ++a) {
                const float2 sv = *reinterpret_cast<const float2 *>(S + (i0 + a) * kLdS + c0);
                acc[a][0] = eGC * sv.x;
                acc[a][1] = eGC * sv.y;
            }
#pragma unroll 2
            for (int t = 0; t < kC; ++t) {
                const float2 dv = *reinterpret_cast<const float2 *>(Dl + t * kLdS + c0);
                const float4 k0 = *reinterpret_cast<const float4 *>(Kp + t * kD + i0);
                const float4 k1 = *reinterpret_cast<const float4 *>(Kp + t * kD + i0 + 4);
                const float kv[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
#pragma unroll
                for (int a = 0; a < 8; ++a) {
                    acc[a][0] = fmaf(kv[a], dv.x, acc[a][0]);
                    acc[a][1] = fmaf(kv[a], dv.y, acc[a][1]);
                }
            }
#pragma unroll
            for (int a = 0; a < 8; ++a)
                *reinterpret_cast<float2 *>(S + (i0 + a) * kLdS + c0) = make_float2(acc[a][0], acc[a][1]);
        }
        __syncthreads();  // M, K' and Delta fully read; S updated
        if (tid == 0 && c + 1 < p.n_chunks) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue_mk(c + 1);
            last_mk = c + 1;
        }
    }
    if (!ok) {
        // never exit with a bulk copy still writing into shared memory
        if (tid == 0) {
            mbar_wait(&bars[0], last_wq & 1);
            mbar_wait(&bars[1], last_mk & 1);
        }
        return;
    }
    __syncthreads();
    for (int e = tid; e < kD * kJB; e += 256) {
        const int j = e >> 7, i = e & 127;
        st_seq[p.plane_out * plane_elems + (static_cast<int64_t>(h) * kD + jb * kJB + j) * kD + i] = S[i * kLdS + j];
    }
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
    SQMIX_CHECK_ARG(a->h_k >= 1 && a->h_v >= 1 && a->h_v % a->h_k == 0,
                    "gdn_prefill: h_v=%d must be a multiple of h_k=%d", a->h_v, a->h_k);
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
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(gdn_chunk_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(kPrepSmem));
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(gdn_chunk_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(kScanSmem));
        if (e != cudaSuccess) return cuda_status(e, "gdn_prefill smem attribute");
        attr_set = true;
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
    gdn_chunk_prep_kernel<<<dim3(p.n_chunks, a->h_v, a->n_seqs), 256, kPrepSmem, st>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_status(e, "gdn_prefill prep launch");
    gdn_chunk_scan_kernel<<<dim3(kD / kJB, a->h_v, a->n_seqs), 256, kScanSmem, st>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_status(e, "gdn_prefill scan launch");
    if (a->n_snap > 1)
        return gdn_launch_recurrent(a, a->n_snap - 1, T_chunk, a->n_snap - 1, a->n_snap - 1, st);
    return SQMIX_OK;
}
