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
// per (sequence, head, chunk) in the workspace, in floats
constexpr int64_t kOffW = 0;
constexpr int64_t kOffU = kOffW + kC * kD;
constexpr int64_t kOffQ = kOffU + kC * kD;
constexpr int64_t kOffK = kOffQ + kC * kD;
constexpr int64_t kOffM = kOffK + kC * kD;
constexpr int64_t kOffS = kOffM + kC * kC;  // scalars: [0] e^{G_C}
constexpr int64_t kChunkFloats = kOffS + 64;

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

// ---- phase 1: state-independent chunk quantities -----------------------------------
// grid (n_chunks, h_v, n_seqs), 256 threads, dynamic smem kPrepSmem
constexpr int kLd = kD + 4;  // padded row stride of the [64][128] tiles
constexpr size_t kPrepSmem = (3 * kC * kLd + 2 * kC * (kC + 1) + 4 * kC) * sizeof(float);

__global__ void __launch_bounds__(256) gdn_chunk_prep_kernel(ChunkParams p) {
    extern __shared__ float sm[];
    float *Ks = sm;                  // [64][kLd]  k, later beta e^G k -> W
    float *Qs = Ks + kC * kLd;       // [64][kLd]  q
    float *Vs = Qs + kC * kLd;       // [64][kLd]  beta v -> U
    float *A = Vs + kC * kLd;        // [64][65]
    float *Mq = A + kC * (kC + 1);   // [64][65]
    float *G = Mq + kC * (kC + 1);   // [64] cumulative log decay
    float *bt = G + kC;              // [64] beta
    float *gg = bt + kC;             // [64] g
    const int c = blockIdx.x, h = blockIdx.y, seq = blockIdx.z;
    const int hk = h % p.h_k;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t0 = c * kC;
    const int n_valid = min(kC, p.T - t0);

    // rows: warp w loads rows w, w+8, ...; 4 elements per lane
    for (int t = warp; t < kC; t += 8) {
        float4 kk = make_float4(0.f, 0.f, 0.f, 0.f), qq = kk, vv = kk;
        if (t < n_valid) {
            const int64_t qk_off = seq * p.qk_sseq + (t0 + t) * p.qk_st + static_cast<int64_t>(hk) * kD + 4 * lane;
            const int64_t v_off = seq * p.v_sseq + (t0 + t) * p.v_st + static_cast<int64_t>(h) * kD + 4 * lane;
            kk = make_float4(load_act(p.k, qk_off, p.dtype), load_act(p.k, qk_off + 1, p.dtype),
                             load_act(p.k, qk_off + 2, p.dtype), load_act(p.k, qk_off + 3, p.dtype));
            qq = make_float4(load_act(p.q, qk_off, p.dtype), load_act(p.q, qk_off + 1, p.dtype),
                             load_act(p.q, qk_off + 2, p.dtype), load_act(p.q, qk_off + 3, p.dtype));
            vv = make_float4(load_act(p.v, v_off, p.dtype), load_act(p.v, v_off + 1, p.dtype),
                             load_act(p.v, v_off + 2, p.dtype), load_act(p.v, v_off + 3, p.dtype));
            if (p.l2_eps > 0.f) {  // rms_norm(x, eps/n) * n^-1/2 (gdn.rs:133-142)
                const float sk = warp_sum32(kk.x * kk.x + kk.y * kk.y + kk.z * kk.z + kk.w * kk.w);
                const float sq = warp_sum32(qq.x * qq.x + qq.y * qq.y + qq.z * qq.z + qq.w * qq.w);
                const float r2 = 1.0f / sqrtf(128.0f);
                const float fk = 1.0f / sqrtf(sk / 128.0f + p.l2_eps / 128.0f) * r2;
                const float fq = 1.0f / sqrtf(sq / 128.0f + p.l2_eps / 128.0f) * r2;
                kk = make_float4(kk.x * fk, kk.y * fk, kk.z * fk, kk.w * fk);
                qq = make_float4(qq.x * fq, qq.y * fq, qq.z * fq, qq.w * fq);
            }
        }
        *reinterpret_cast<float4 *>(Ks + t * kLd + 4 * lane) = kk;
        *reinterpret_cast<float4 *>(Qs + t * kLd + 4 * lane) = qq;
        *reinterpret_cast<float4 *>(Vs + t * kLd + 4 * lane) = vv;
    }
    if (tid < kC) {
        const int64_t gb = (static_cast<int64_t>(seq) * p.T_all + t0 + tid) * p.h_v + h;
        gg[tid] = tid < n_valid ? p.g[gb] : 0.f;
        bt[tid] = tid < n_valid ? p.beta[gb] : 0.f;
    }
    __syncthreads();
    if (warp == 0) {  // inclusive scan of g over the chunk (two values per lane)
        float a0 = gg[2 * lane], a1 = gg[2 * lane + 1];
        float s = a0 + a1;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const float y = __shfl_up_sync(0xffffffffu, s, off);
            if (lane >= off) s += y;
        }
        const float excl = s - (a0 + a1);
        G[2 * lane] = excl + a0;
        G[2 * lane + 1] = excl + a0 + a1;
    }
    __syncthreads();

    // K K^T and Q K^T, 4x4 outputs per thread
    {
        const int tb = tid >> 4, sb = tid & 15;  // rows tb + 16a, columns sb + 16b
        float kk[4][4] = {}, qk[4][4] = {};
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
                const int t = tb + 16 * a, s = sb + 16 * b;
                const float dec = s <= t ? expf(G[t] - G[s]) : 0.f;
                A[t * (kC + 1) + s] = s < t ? bt[t] * dec * kk[a][b] : 0.f;
                Mq[t * (kC + 1) + s] = dec * qk[a][b] * rsd;
            }
    }
    __syncthreads();
    // right-hand sides: beta e^G k and beta v
    for (int e = tid; e < kC * kD; e += 256) {
        const int t = e >> 7, i = e & 127;
        Ks[t * kLd + i] *= bt[t] * expf(G[t]);
        Vs[t * kLd + i] *= bt[t];
    }
    __syncthreads();
    // forward substitution, one thread per column of [W | U]: X_t -= sum_{s<t} A_ts X_s
    {
        float *X = tid < kD ? Ks + tid : Vs + (tid - kD);
        for (int t = 1; t < kC; ++t) {
            float acc = X[t * kLd];
            const float *Ar = A + t * (kC + 1);
            for (int s = 0; s < t; ++s) acc = fmaf(-Ar[s], X[s * kLd], acc);
            X[t * kLd] = acc;
        }
    }
    __syncthreads();
    // outputs: W, U, Q e^G / sqrt(d), K e^{G_C - G}, M
    float *wsc = p.ws + ((static_cast<int64_t>(seq) * p.h_v + h) * p.n_chunks + c) * kChunkFloats;
    const float GC = G[kC - 1];
    const float rsd = 1.0f / sqrtf(128.0f);
    for (int e = tid; e < kC * kD / 4; e += 256) {
        const int t = e >> 5, i4 = (e & 31) * 4;
        const float4 w = *reinterpret_cast<const float4 *>(Ks + t * kLd + i4);
        const float4 u = *reinterpret_cast<const float4 *>(Vs + t * kLd + i4);
        float4 qv = *reinterpret_cast<const float4 *>(Qs + t * kLd + i4);
        const float fq = expf(G[t]) * rsd;
        qv = make_float4(qv.x * fq, qv.y * fq, qv.z * fq, qv.w * fq);
        *reinterpret_cast<float4 *>(wsc + kOffW + t * kD + i4) = w;
        *reinterpret_cast<float4 *>(wsc + kOffU + t * kD + i4) = u;
        *reinterpret_cast<float4 *>(wsc + kOffQ + t * kD + i4) = qv;
    }
    __syncthreads();
    // K e^{G_C - G}: Ks was overwritten by W, so reload k rows (l2-normalised again)
    for (int t = warp; t < kC; t += 8) {
        float4 kk = make_float4(0.f, 0.f, 0.f, 0.f);
        if (t < n_valid) {
            const int64_t qk_off = seq * p.qk_sseq + (t0 + t) * p.qk_st + static_cast<int64_t>(hk) * kD + 4 * lane;
            kk = make_float4(load_act(p.k, qk_off, p.dtype), load_act(p.k, qk_off + 1, p.dtype),
                             load_act(p.k, qk_off + 2, p.dtype), load_act(p.k, qk_off + 3, p.dtype));
            if (p.l2_eps > 0.f) {
                const float sk = warp_sum32(kk.x * kk.x + kk.y * kk.y + kk.z * kk.z + kk.w * kk.w);
                const float fk = 1.0f / sqrtf(sk / 128.0f + p.l2_eps / 128.0f) / sqrtf(128.0f);
                kk = make_float4(kk.x * fk, kk.y * fk, kk.z * fk, kk.w * fk);
            }
        }
        const float f = expf(GC - G[t]);
        *reinterpret_cast<float4 *>(wsc + kOffK + t * kD + 4 * lane) =
            make_float4(kk.x * f, kk.y * f, kk.z * f, kk.w * f);
    }
    for (int e = tid; e < kC * kC; e += 256) wsc[kOffM + e] = Mq[(e >> 6) * (kC + 1) + (e & 63)];
    if (tid == 0) wsc[kOffS] = expf(GC);
}

// ---- phase 2: walk the chunks of one (sequence, head, 32 value columns) -------------
// grid (kD / kJB, h_v, n_seqs), 256 threads, dynamic smem kScanSmem
constexpr int kLdS = kJB + 1;
constexpr size_t kScanSmem =
    (static_cast<size_t>(kD) * kLdS + kC * kLdS + 3 * kC * kLd + kC * (kC + 1)) * sizeof(float);

__global__ void __launch_bounds__(256) gdn_chunk_scan_kernel(ChunkParams p) {
    extern __shared__ float sm[];
    float *S = sm;                  // [128][kLdS]   S[i][j] of this column block
    float *Dl = S + kD * kLdS;      // [64][kLdS]    Delta
    float *Wt = Dl + kC * kLdS;     // [64][kLd]
    float *Qt = Wt + kC * kLd;      // [64][kLd]
    float *Kt = Qt + kC * kLd;      // [64][kLd]
    float *Mt = Kt + kC * kLd;      // [64][65]
    const int jb = blockIdx.x, h = blockIdx.y, seq = blockIdx.z;
    const int tid = threadIdx.x;
    const int64_t plane_elems = static_cast<int64_t>(p.h_v) * kD * kD;
    float *st_seq = p.state + static_cast<int64_t>(seq) * p.n_planes * plane_elems;
    int plane = p.sel ? p.sel[seq] : 0;
    plane = min(max(plane, 0), p.n_planes - 1);
    // S[i][j] at ((h*128 + j)*128 + i): thread loads column j rows i
    for (int e = tid; e < kD * kJB; e += 256) {
        const int j = e >> 7, i = e & 127;
        S[i * kLdS + j] = st_seq[plane * plane_elems + (static_cast<int64_t>(h) * kD + jb * kJB + j) * kD + i];
    }
    // thread tiles: Delta / O: rows 4*(tid>>4)..+3, cols 2*(tid&15)..+1 (64 x 32 outputs)
    const int r0 = 4 * (tid >> 4), c0 = 2 * (tid & 15);
    // S update: rows 8*(tid>>4)..+7 (i), cols 2*(tid&15)..+1 (j) -> 16 outputs
    const int i0 = 8 * (tid >> 4);
    for (int c = 0; c < p.n_chunks; ++c) {
        const float *wsc = p.ws + ((static_cast<int64_t>(seq) * p.h_v + h) * p.n_chunks + c) * kChunkFloats;
        __syncthreads();  // previous chunk finished with the tiles
        for (int e = tid; e < kC * kD / 4; e += 256) {
            const int t = e >> 5, i4 = (e & 31) * 4;
            *reinterpret_cast<float4 *>(Wt + t * kLd + i4) = *reinterpret_cast<const float4 *>(wsc + kOffW + t * kD + i4);
            *reinterpret_cast<float4 *>(Qt + t * kLd + i4) = *reinterpret_cast<const float4 *>(wsc + kOffQ + t * kD + i4);
            *reinterpret_cast<float4 *>(Kt + t * kLd + i4) = *reinterpret_cast<const float4 *>(wsc + kOffK + t * kD + i4);
        }
        for (int e = tid; e < kC * kC; e += 256) Mt[(e >> 6) * (kC + 1) + (e & 63)] = wsc[kOffM + e];
        const float eGC = wsc[kOffS];
        __syncthreads();
        // Delta = U - W S0
        {
            float acc[4][2];
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int b = 0; b < 2; ++b) acc[a][b] = wsc[kOffU + (r0 + a) * kD + jb * kJB + c0 + b];
            for (int i = 0; i < kD; ++i) {
                const float s0 = S[i * kLdS + c0], s1 = S[i * kLdS + c0 + 1];
#pragma unroll
                for (int a = 0; a < 4; ++a) {
                    const float w = Wt[(r0 + a) * kLd + i];
                    acc[a][0] = fmaf(-w, s0, acc[a][0]);
                    acc[a][1] = fmaf(-w, s1, acc[a][1]);
                }
            }
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int b = 0; b < 2; ++b) Dl[(r0 + a) * kLdS + c0 + b] = acc[a][b];
        }
        __syncthreads();
        // O = Qs S0 + M Delta
        {
            float acc[4][2] = {};
            for (int i = 0; i < kD; ++i) {
                const float s0 = S[i * kLdS + c0], s1 = S[i * kLdS + c0 + 1];
#pragma unroll
                for (int a = 0; a < 4; ++a) {
                    const float q = Qt[(r0 + a) * kLd + i];
                    acc[a][0] = fmaf(q, s0, acc[a][0]);
                    acc[a][1] = fmaf(q, s1, acc[a][1]);
                }
            }
            for (int s = 0; s < kC; ++s) {
                const float d0 = Dl[s * kLdS + c0], d1 = Dl[s * kLdS + c0 + 1];
#pragma unroll
                for (int a = 0; a < 4; ++a) {
                    const float mv = Mt[(r0 + a) * (kC + 1) + s];
                    acc[a][0] = fmaf(mv, d0, acc[a][0]);
                    acc[a][1] = fmaf(mv, d1, acc[a][1]);
                }
            }
#pragma unroll
            for (int a = 0; a < 4; ++a) {
                const int t = c * kC + r0 + a;
                if (t < p.T) {
#pragma unroll
                    for (int b = 0; b < 2; ++b)
                        p.out[((static_cast<int64_t>(seq) * p.T_all + t) * p.h_v + h) * kD + jb * kJB + c0 + b] =
                            acc[a][b];
                }
            }
        }
        __syncthreads();  // S0 fully read
        // S = e^{G_C} S0 + K'^T Delta
        {
            float acc[8][2];
#pragma unroll
            for (int a = 0; a < 8; ++a) {
                acc[a][0] = eGC * S[(i0 + a) * kLdS + c0];
                acc[a][1] = eGC * S[(i0 + a) * kLdS + c0 + 1];
            }
            for (int t = 0; t < kC; ++t) {
                const float d0 = Dl[t * kLdS + c0], d1 = Dl[t * kLdS + c0 + 1];
#pragma unroll
                for (int a = 0; a < 8; ++a) {
                    const float kv = Kt[t * kLd + i0 + a];
                    acc[a][0] = fmaf(kv, d0, acc[a][0]);
                    acc[a][1] = fmaf(kv, d1, acc[a][1]);
                }
            }
#pragma unroll
            for (int a = 0; a < 8; ++a) {
                S[(i0 + a) * kLdS + c0] = acc[a][0];
                S[(i0 + a) * kLdS + c0 + 1] = acc[a][1];
            }
        }
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
    return static_cast<size_t>(n_seqs) * h_v * n_chunks * kChunkFloats * sizeof(float);
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
