// gdn_layer.cu -- a whole GDN mixer decode step (T <= 2 tokens) in one launch.
//
// Replaces, for decode and the 2-token MTP verify, the chain of a GDN layer between
// its projections (src/model/gdn.rs:264-577):
//   ggml_concat(conv history, qkv^T) -> ggml_ssm_conv -> ggml_silu      (gdn.rs:290-360)
//   -> l2_norm(q), l2_norm(k)                                           (gdn.rs:436-441)
//   -> beta = sigmoid(b), g = softplus(alpha + dt_bias) * ssm_a          (gdn.rs:268-287)
//   -> ggml_gated_delta_net with the plane select and snapshot slots    (gdn.rs:445-538)
//   -> norm_gated(o, ssm_norm, z) = rms_norm(o) * w * silu(z)            (gdn.rs:150-181)
//   and the conv-history write-back per slot                            (graph.rs:913-961)
// which the unfused path runs as three launches (sqmix_gdn_conv, sqmix_gdn_decode,
// sqmix_head_norm).
//
// Decomposition: one cluster of 4 * R CTAs per q/k head hk (R = H_v / H_k value heads
// read it: hk, hk + H_k, ...), CTA rank m * 4 + u handling value head hk + m * H_k,
// value columns 32u .. 32u + 31.  With qwen35moe's 16 q/k and 32 value heads that is
// 16 clusters of 8 = 128 CTAs per sequence.  A CTA (256 threads):
//   1. before the grid-dependency wait: its conv taps, the norm weight and, under
//      SQMIX_GDN_STATE_READY, its 32 state columns (4 per warp, 16 bytes per lane) and
//      the conv history of the selected plane; after it, x, the raw gates and z in one
//      batch of loads;
//   2. conv + SiLU of the head's 128 q and 128 k channels (thread = channel) and of its
//      32 v channels; q and k L2-normalised per token (warp sums, then shared memory);
//   3. arrives on the cluster barrier once its reads of the conv-history plane are done
//      (every CTA of the cluster reads the same q/k history, so none may overwrite it
//      before all have read it);
//   4. the delta-rule recurrence, warp = 4 columns (as gdn_recurrent_kernel), snapshot
//      slots written while the state is in registers;
//   5. waits for phase 1 of the cluster barrier, then stores its 32 columns' share of
//      the head's sum of o^2 into the shared memory of the head's 4 CTAs (distributed
//      shared memory), passes phase 2 and writes rms_norm(o) * w * silu(z);
//   6. the conv-history slots: rank 0 writes the q/k channels, every CTA its v channels.
// The two cluster barriers are hardware barriers of co-scheduled CTAs: no spin loops.
#include <math.h>

#include "common.cuh"

namespace sqmix {

namespace {

constexpr int kLayerK = 4;  // conv taps (ssm_d_conv of qwen35moe)

struct GdnLayerParams {
    const void *x;
    int x_dtype;
    int64_t x_st, x_ss;
    const float *conv_w;  // [C][K]
    float *conv_state;    // [n_seqs][n_planes][C][K-1]
    const float *alpha, *bproj, *dt_bias, *ssm_a;
    float *state;         // [n_seqs][n_planes][H_v][128][128]
    int n_planes;
    const int32_t *sel;
    int n_snap, n_seqs, T, h_k, h_v, ratio;
    float l2_eps;
    const void *z;
    int z_dtype;
    int64_t z_st, z_ss;
    const float *norm_w;
    int64_t norm_w_sh;
    float norm_eps;
    float *out;           // [n_seqs][T][H_v][128]
    int state_ready;
};

__device__ __forceinline__ float silu_f(float y) { return y / (1.0f + expf(-y)); }

__device__ __forceinline__ void cluster_arrive() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr_cl, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr_cl), "f"(v) : "memory");
}

__global__ void __launch_bounds__(256, 1) gdn_layer_kernel(GdnLayerParams p) {
    constexpr int K = kLayerK;
    __shared__ float qs[2][128], ks[2][128], vs[2][32], os[2][32];
    __shared__ float red[8][2];
    __shared__ float nsum[4][2];  // the head's 4 CTAs' sums of o^2 (per token)
    __shared__ float gate_g[2], gate_b[2];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int csize = 4 * p.ratio;
    const int rank = static_cast<int>(cluster_ctarank());
    const int hk = blockIdx.x / csize;
    const int m = rank >> 2, u = rank & 3;
    const int hv = hk + m * p.h_k;
    const int seq = blockIdx.y;
    const int col0 = 32 * u;
    const int C = (2 * p.h_k + p.h_v) * 128;

    // ---- 1. taps and (optionally) the state before the dependency wait ------------
    const int ch = tid < 128 ? hk * 128 + tid : p.h_k * 128 + hk * 128 + (tid - 128);  // q | k channel
    const int chv = 2 * p.h_k * 128 + hv * 128 + col0 + lane;                           // v channel (warp 0)
    const float4 wq = *reinterpret_cast<const float4 *>(p.conv_w + static_cast<size_t>(ch) * K);
    float4 wv = make_float4(0.f, 0.f, 0.f, 0.f);
    if (warp == 0) wv = *reinterpret_cast<const float4 *>(p.conv_w + static_cast<size_t>(chv) * K);
    const int64_t plane_elems = static_cast<int64_t>(p.h_v) * 128 * 128;
    float *st_seq = p.state + static_cast<int64_t>(seq) * p.n_planes * plane_elems;
    const int j0 = col0 + 4 * warp;  // this warp's first value column
    const int64_t col_off = (static_cast<int64_t>(hv) * 128 + j0) * 128 + 4 * lane;
    const size_t cplane = static_cast<size_t>(C) * (K - 1);
    float *cst = p.conv_state + static_cast<size_t>(seq) * p.n_planes * cplane;
    // conv_input rows 0..K-2 (history) and K-1.. (the T new rows), q|k channel and v channel
    float in[K - 1 + 2], inv[K - 1 + 2] = {};
    float4 S[4];
    // The state columns and the conv history of the selected plane: under
    // SQMIX_GDN_STATE_READY the previous kernel writes neither, so they are read before
    // the dependency wait; the rest (x, the gates, z: the projections' outputs) after it,
    // all issued together.
    auto load_planes = [&]() {
        int plane = p.sel ? p.sel[seq] : 0;
        plane = min(max(plane, 0), p.n_planes - 1);
#pragma unroll
        for (int c = 0; c < 4; ++c)
            S[c] = *reinterpret_cast<const float4 *>(st_seq + plane * plane_elems + col_off + c * 128);
#pragma unroll
        for (int r = 0; r < K - 1; ++r) in[r] = cst[plane * cplane + static_cast<size_t>(ch) * (K - 1) + r];
        if (warp == 0) {
#pragma unroll
            for (int r = 0; r < K - 1; ++r) inv[r] = cst[plane * cplane + static_cast<size_t>(chv) * (K - 1) + r];
        }
    };
    const float nw = warp == 0 && p.norm_w ? p.norm_w[static_cast<int64_t>(hv) * p.norm_w_sh + col0 + lane] : 1.0f;
    if (p.state_ready) load_planes();
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" :::);
    if (!p.state_ready) load_planes();

    // ---- 2. conv + SiLU (+ L2 norm of q, k) ----------------------------------------
    const int64_t xb = static_cast<int64_t>(seq) * p.x_ss;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        in[K - 1 + t] = t < p.T ? load_act(p.x, xb + t * p.x_st + ch, p.x_dtype) : 0.f;
        if (warp == 0) inv[K - 1 + t] = t < p.T ? load_act(p.x, xb + t * p.x_st + chv, p.x_dtype) : 0.f;
    }
    float graw = 0.f, braw = 0.f;  // the raw gates of token tid / 2 (threads 0 .. 2T-1)
    if (tid < 2 * p.T) {
        const int64_t gi = (static_cast<int64_t>(seq) * p.T + (tid >> 1)) * p.h_v + hv;
        graw = p.alpha[gi];
        braw = p.bproj[gi];
    }
    float zv[2] = {0.f, 0.f};
    if (warp == 0 && p.z) {
#pragma unroll
        for (int t = 0; t < 2; ++t)
            if (t < p.T)
                zv[t] = load_act(p.z, static_cast<int64_t>(seq) * p.z_ss + t * p.z_st + static_cast<int64_t>(hv) * 128 +
                                          col0 + lane,
                                 p.z_dtype);
    }
    // every CTA of the cluster has read its history plane: the writers may go ahead
    // once all have arrived (they wait at the end)
    cluster_arrive();
    const float wqa[4] = {wq.x, wq.y, wq.z, wq.w}, wva[4] = {wv.x, wv.y, wv.z, wv.w};
    float y[2];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        float s = 0.f, sv = 0.f;
#pragma unroll
        for (int k = 0; k < K; ++k) {
            s = __fadd_rn(s, __fmul_rn(in[t + k], wqa[k]));
            sv = __fadd_rn(sv, __fmul_rn(inv[t + k], wva[k]));
        }
        y[t] = silu_f(s);
        if (warp == 0 && t < p.T) vs[t][lane] = silu_f(sv);
        float ss = y[t] * y[t];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        if (lane == 0) red[warp][t] = ss;
    }
    if (tid < 2 * p.T) {  // gate epilogue, one token per thread pair: g (even), beta (odd)
        const int t = tid >> 1;
        float g = graw, b = braw;
        gdn_gates(g, b, p.dt_bias, p.ssm_a, hv);
        if (tid & 1)
            gate_b[t] = b;
        else
            gate_g[t] = g;
    }
    __syncthreads();
    {  // x / ||x|| as scale(rms_norm(x, eps / 128), 1 / sqrt(128)), gdn.rs:133-142
        const int w0 = tid < 128 ? 0 : 4;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            const float ss = red[w0][t] + red[w0 + 1][t] + red[w0 + 2][t] + red[w0 + 3][t];
            const float sc = p.l2_eps > 0.f ? 1.0f / sqrtf(ss / 128.0f + p.l2_eps / 128.0f) : 1.0f;
            const float s2 = p.l2_eps > 0.f ? 1.0f / sqrtf(128.0f) : 1.0f;
            const float yn = (y[t] * sc) * s2;
            if (tid < 128)
                qs[t][tid] = yn;
            else
                ks[t][tid - 128] = yn;
        }
    }
    __syncthreads();

    // ---- 4. recurrence: warp = 4 value columns, lane = keys 4 lane .. 4 lane + 3 ----
    const float inv_sqrt_d = 1.0f / sqrtf(128.0f);
    for (int t = 0; t < p.T; ++t) {
        const float4 kk = *reinterpret_cast<const float4 *>(&ks[t][4 * lane]);
        const float4 qq = *reinterpret_cast<const float4 *>(&qs[t][4 * lane]);
        const float decay = expf(gate_g[t]);
        const float bt = gate_b[t];
        float skv[4], sq[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            S[c].x *= decay;
            S[c].y *= decay;
            S[c].z *= decay;
            S[c].w *= decay;
            skv[c] = S[c].x * kk.x + S[c].y * kk.y + S[c].z * kk.z + S[c].w * kk.w;
            sq[c] = S[c].x * qq.x + S[c].y * qq.y + S[c].z * qq.z + S[c].w * qq.w;
        }
        float kq = kk.x * qq.x + kk.y * qq.y + kk.z * qq.z + kk.w * qq.w;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                skv[c] += __shfl_xor_sync(0xffffffffu, skv[c], off);
                sq[c] += __shfl_xor_sync(0xffffffffu, sq[c], off);
            }
            kq += __shfl_xor_sync(0xffffffffu, kq, off);
        }
        float o[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const float delta = (vs[t][4 * warp + c] - skv[c]) * bt;
            S[c].x = fmaf(kk.x, delta, S[c].x);
            S[c].y = fmaf(kk.y, delta, S[c].y);
            S[c].z = fmaf(kk.z, delta, S[c].z);
            S[c].w = fmaf(kk.w, delta, S[c].w);
            o[c] = fmaf(delta, kq, sq[c]) * inv_sqrt_d;
        }
        if (lane == 0) {
#pragma unroll
            for (int c = 0; c < 4; ++c) os[t][4 * warp + c] = o[c];
        }
        const int slot = p.T - 1 - t;
        if (slot < p.n_snap) {
#pragma unroll
            for (int c = 0; c < 4; ++c)
                *reinterpret_cast<float4 *>(st_seq + slot * plane_elems + col_off + c * 128) = S[c];
        }
    }
    __syncthreads();

    // ---- 5. norm_gated: the head's sum of o^2 over its 4 CTAs, by DSMEM -----------
    // (after the phase-1 wait: every CTA of the cluster is running and has read its conv
    // history, so remote shared memory may be written)
    cluster_wait();
    float ov[2] = {0.f, 0.f};
    if (warp == 0) {
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            ov[t] = t < p.T ? os[t][lane] : 0.f;
            float s2 = ov[t] * ov[t];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, off);
            if (lane < 4)  // lane i writes into the head's CTA i (rank m * 4 + i)
                st_cluster_f32(mapa_shared(smem_u32(&nsum[u][t]), static_cast<uint32_t>(m * 4 + lane)), s2);
        }
    }
    cluster_arrive();  // phase 2: this CTA's shares of the norm sums are stored
    // ---- 6. conv-history slots: plane s <- conv_input rows [T - s, T - s + K - 1) ---
    // (every CTA of the cluster has read the history plane: phase 1 above).  Issued
    // between the phase-2 arrive and wait: before the arrive, its release would wait for
    // these global stores; here they drain while the head's norm sums arrive.
    for (int s = 0; s < p.n_snap; ++s) {
        const int r0 = p.T - s;
        if (rank == 0) {  // the q/k channels of this head, once per cluster
#pragma unroll
            for (int r = 0; r < K - 1; ++r) {
                float v = 0.f;
#pragma unroll
                for (int rr = 0; rr < K - 1 + 2; ++rr)
                    if (rr == r0 + r) v = in[rr];
                cst[s * cplane + static_cast<size_t>(ch) * (K - 1) + r] = v;
            }
        }
        if (warp == 0) {  // this CTA's v channels
#pragma unroll
            for (int r = 0; r < K - 1; ++r) {
                float v = 0.f;
#pragma unroll
                for (int rr = 0; rr < K - 1 + 2; ++rr)
                    if (rr == r0 + r) v = inv[rr];
                cst[s * cplane + static_cast<size_t>(chv) * (K - 1) + r] = v;
            }
        }
    }
    cluster_wait();
    if (warp == 0) {
        const int col = col0 + lane;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            if (t >= p.T) break;
            const float tot = nsum[0][t] + nsum[1][t] + nsum[2][t] + nsum[3][t];
            float yv = ov[t] * (1.0f / sqrtf(tot / 128.0f + p.norm_eps));
            yv = yv * nw;
            if (p.z) yv = yv * silu_f(zv[t]);
            p.out[((static_cast<int64_t>(seq) * p.T + t) * p.h_v + hv) * 128 + col] = yv;
        }
    }
}

}  // namespace
}  // namespace sqmix

using namespace sqmix;

extern "C" int sqmix_gdn_layer_decode(const sqmix_gdn_layer_args *a, sqmix_stream_t stream) {
    SQMIX_CHECK_ARG(a != nullptr, "gdn_layer_decode: null args");
    SQMIX_CHECK_ARG(a->x && a->conv_weight && a->conv_state && a->alpha && a->beta && a->ssm_a && a->state && a->out,
                    "gdn_layer_decode: null pointer argument");
    SQMIX_CHECK_ARG(a->x_dtype == SQMIX_F32 || a->x_dtype == SQMIX_F16 || a->x_dtype == SQMIX_BF16,
                    "gdn_layer_decode: x dtype %d", a->x_dtype);
    SQMIX_CHECK_ARG(!a->z || a->z_dtype == SQMIX_F32 || a->z_dtype == SQMIX_F16 || a->z_dtype == SQMIX_BF16,
                    "gdn_layer_decode: z dtype %d", a->z_dtype);
    SQMIX_CHECK_ARG(a->n_tokens == 1 || a->n_tokens == 2,
                    "gdn_layer_decode: n_tokens=%d (1 or 2; longer chunks: sqmix_gdn_conv + sqmix_gdn_prefill)",
                    a->n_tokens);
    SQMIX_CHECK_ARG(a->kernel == kLayerK, "gdn_layer_decode: kernel=%d (supported: %d)", a->kernel, kLayerK);
    SQMIX_CHECK_ARG(a->h_k >= 1 && (a->h_v == a->h_k || a->h_v == 2 * a->h_k),
                    "gdn_layer_decode: h_v=%d must be h_k or 2 h_k (h_k=%d)", a->h_v, a->h_k);
    SQMIX_CHECK_ARG(a->n_seqs >= 1 && a->n_seqs <= 65535, "gdn_layer_decode: n_seqs=%d", a->n_seqs);
    SQMIX_CHECK_ARG(a->n_planes >= 1 && a->n_snap >= 1 && a->n_snap <= a->n_planes && a->n_snap <= a->n_tokens,
                    "gdn_layer_decode: n_snap=%d must be in [1, min(T=%d, n_planes=%d)]", a->n_snap, a->n_tokens,
                    a->n_planes);
    const int64_t C = (2 * static_cast<int64_t>(a->h_k) + a->h_v) * 128;
    SQMIX_CHECK_ARG(a->x_stride_tok >= C && (a->n_seqs == 1 || a->x_stride_seq >= a->n_tokens * a->x_stride_tok),
                    "gdn_layer_decode: x strides (rows of >= %lld channels)", (long long)C);
    SQMIX_CHECK_ARG(a->l2_eps >= 0.f && a->norm_eps >= 0.f, "gdn_layer_decode: eps must be >= 0");
    SQMIX_CHECK_ARG((reinterpret_cast<uintptr_t>(a->conv_weight) & 15) == 0 &&
                        (reinterpret_cast<uintptr_t>(a->state) & 15) == 0,
                    "gdn_layer_decode: conv_weight and state must be 16-byte aligned");
    SQMIX_CHECK_ARG((a->flags & ~SQMIX_GDN_STATE_READY) == 0, "gdn_layer_decode: unknown flags 0x%x", a->flags);
    GdnLayerParams p;
    p.x = a->x;
    p.x_dtype = a->x_dtype;
    p.x_st = a->x_stride_tok;
    p.x_ss = a->x_stride_seq;
    p.conv_w = a->conv_weight;
    p.conv_state = a->conv_state;
    p.alpha = a->alpha;
    p.bproj = a->beta;
    p.dt_bias = a->dt_bias;
    p.ssm_a = a->ssm_a;
    p.state = a->state;
    p.n_planes = a->n_planes;
    p.sel = a->sel;
    p.n_snap = a->n_snap;
    p.n_seqs = a->n_seqs;
    p.T = a->n_tokens;
    p.h_k = a->h_k;
    p.h_v = a->h_v;
    p.ratio = a->h_v / a->h_k;
    p.l2_eps = a->l2_eps;
    p.z = a->z;
    p.z_dtype = a->z_dtype;
    p.z_st = a->z_stride_tok;
    p.z_ss = a->z_stride_seq;
    p.norm_w = a->norm_weight;
    p.norm_w_sh = a->norm_weight_stride_head;
    p.norm_eps = a->norm_eps;
    p.out = a->out;
    p.state_ready = (a->flags & SQMIX_GDN_STATE_READY) != 0;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 4 * p.ratio;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(4 * p.ratio * a->h_k), static_cast<unsigned>(a->n_seqs));
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = reinterpret_cast<cudaStream_t>(stream);
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cuda_status(cudaLaunchKernelEx(&cfg, gdn_layer_kernel, p), "gdn_layer_decode launch");
}
