// gdn_front.cu -- the GDN front end (short causal convolution + SiLU + q/k L2 norm,
// with the conv-history planes) and the per-head RMS norms of both mixers.
//
// Replaces, per GDN layer step (src/model/gdn.rs:290-441, src/model/graph.rs:913-961):
//   ggml_concat(conv history, qkv^T) -> ggml_ssm_conv -> ggml_silu -> views of q/k/v
//   -> l2_norm(q), l2_norm(k), and the per-slot ggml_cpy of the conv tails;
// and the norms (attn.rs:66-84 head_rms_norm of Q and K; gdn.rs:150-181 norm_gated).
//
// Both kernels are HBM/latency-bound elementwise work with one reduction per head,
// and both are launched with programmatic stream serialisation:
//   gdn_conv_kernel: one warp per (128-channel head block, token chunk, sequence),
//     four channels per lane (vector loads of x, taps and history); the chunk's
//     tokens are loaded at once and the L2 norm of a q/k head is a warp reduction.
//     Only the first chunk reads the history plane, and the same warp writes the
//     history slots after it has read everything it needs, so the in-place update
//     of the resident planes has no cross-warp hazard.
//   head_norm_kernel: one warp per (token, head) row.
#include <math.h>

#include "common.cuh"

namespace sqmix {

struct ConvParams {
    const void *x;
    int64_t x_st, x_ss;
    const float *w;
    float *state;
    int n_planes;
    const int32_t *sel;
    int n_snap;
    int T, C, n_qk;
    float eps;
    float *out;
};

__device__ __forceinline__ float silu(float y) { return y / (1.0f + expf(-y)); }

// Four consecutive elements of x (16-byte f32, 8-byte bf16/f16 loads).
template <int DT>
__device__ __forceinline__ float4 ld4(const void *p, int64_t i) {
    if constexpr (DT == SQMIX_F32) {
        return *reinterpret_cast<const float4 *>(static_cast<const float *>(p) + i);
    } else if constexpr (DT == SQMIX_BF16) {
        const uint2 r = *reinterpret_cast<const uint2 *>(static_cast<const __nv_bfloat16 *>(p) + i);
        const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&r.x));
        const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&r.y));
        return make_float4(a.x, a.y, b.x, b.y);
    } else {
        const uint2 r = *reinterpret_cast<const uint2 *>(static_cast<const __half *>(p) + i);
        const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&r.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&r.y));
        return make_float4(a.x, a.y, b.x, b.y);
    }
}
__device__ __forceinline__ float at4(const float4 &v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }

// One warp per (128-channel head block, TC-token chunk, sequence); lane L owns
// channels 4L..4L+3 of the block, so x rows, taps and history move as 8/16-byte
// vectors and the per-head L2 norm is a warp reduction.  The warp of the first chunk
// is the only one that reads the history plane of its channels and the only one that
// writes their history slots (after its reads), so the in-place update is race-free.
// Launched with programmatic stream serialisation: the taps are loaded before the
// grid dependency wait.
template <int K, int TC, int DT>
__global__ void __launch_bounds__(128) gdn_conv_kernel(ConvParams p) {
    const int lane = threadIdx.x & 31;
    const int hb = blockIdx.x * 4 + (threadIdx.x >> 5);
    const int seq = blockIdx.z;
    const int t0 = blockIdx.y * TC;
    const bool live = hb * 128 < p.C;
    const int c0 = hb * 128 + 4 * lane;
    float w[4][K];
    if (live) {
        const float4 *wv = reinterpret_cast<const float4 *>(p.w + static_cast<size_t>(c0) * K);
#pragma unroll
        for (int i = 0; i < K; ++i) {  // 4 channels x K taps = K float4
            const float4 v = wv[i];
#pragma unroll
            for (int e = 0; e < 4; ++e) w[(4 * i + e) / K][(4 * i + e) % K] = at4(v, e);
        }
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" :::);
    if (!live) return;
    const int nt = min(TC, p.T - t0);
    const int64_t xb = static_cast<int64_t>(seq) * p.x_ss + c0;
    const size_t plane_elems = static_cast<size_t>(p.C) * (K - 1);
    float *planes = p.state + static_cast<size_t>(seq) * p.n_planes * plane_elems;

    // conv_input rows t0 .. t0 + TC + K - 2 of the four channels
    float in[TC + K - 1][4];
    if (t0 == 0) {
        const int sel = min(max(p.sel ? p.sel[seq] : 0, 0), p.n_planes - 1);  // as the recurrence does
        const float4 *hv =
            reinterpret_cast<const float4 *>(planes + sel * plane_elems + static_cast<size_t>(c0) * (K - 1));
#pragma unroll
        for (int i = 0; i < K - 1; ++i) {  // 4 channels x (K-1) rows = K-1 float4
            const float4 v = hv[i];
#pragma unroll
            for (int e = 0; e < 4; ++e) in[(4 * i + e) % (K - 1)][(4 * i + e) / (K - 1)] = at4(v, e);
        }
    } else {
#pragma unroll
        for (int r = 0; r < K - 1; ++r) {
            const float4 v = ld4<DT>(p.x, xb + static_cast<int64_t>(t0 - (K - 1) + r) * p.x_st);
            in[r][0] = v.x;
            in[r][1] = v.y;
            in[r][2] = v.z;
            in[r][3] = v.w;
        }
    }
#pragma unroll
    for (int j = 0; j < TC; ++j) {
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (j < nt) v = ld4<DT>(p.x, xb + static_cast<int64_t>(t0 + j) * p.x_st);
        in[K - 1 + j][0] = v.x;
        in[K - 1 + j][1] = v.y;
        in[K - 1 + j][2] = v.z;
        in[K - 1 + j][3] = v.w;
    }
    const bool norm = p.eps > 0.f && hb * 128 < p.n_qk;
    float *o = p.out + (static_cast<size_t>(seq) * p.T + t0) * p.C + c0;
    float y[TC][4];
#pragma unroll
    for (int j = 0; j < TC; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            float s = 0.f;
#pragma unroll
            for (int k = 0; k < K; ++k) s = __fadd_rn(s, __fmul_rn(in[j + k][e], w[e][k]));
            y[j][e] = silu(s);
        }
    if (norm) {  // x / ||x|| as scale(rms_norm(x, eps / 128), 1 / sqrt(128)), gdn.rs:133-142
        float ss[TC];
#pragma unroll
        for (int j = 0; j < TC; ++j) ss[j] = y[j][0] * y[j][0] + y[j][1] * y[j][1] + y[j][2] * y[j][2] + y[j][3] * y[j][3];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1)
#pragma unroll
            for (int j = 0; j < TC; ++j) ss[j] += __shfl_xor_sync(0xffffffffu, ss[j], off);
        // every lane holds the TC sums; lane j turns token j's into its factor and the
        // warp shares them (one square root and division per lane instead of TC)
        float mine = ss[0];
#pragma unroll
        for (int j = 1; j < TC; ++j) mine = lane == j ? ss[j] : mine;
        const float f = 1.0f / sqrtf(mine / 128.0f + p.eps / 128.0f);
        const float s2 = 1.0f / sqrtf(128.0f);
#pragma unroll
        for (int j = 0; j < TC; ++j) {
            const float sc = __shfl_sync(0xffffffffu, f, j);
#pragma unroll
            for (int e = 0; e < 4; ++e) y[j][e] = (y[j][e] * sc) * s2;
        }
    }
#pragma unroll
    for (int j = 0; j < TC; ++j)
        if (j < nt)
            *reinterpret_cast<float4 *>(o + static_cast<size_t>(j) * p.C) =
                make_float4(y[j][0], y[j][1], y[j][2], y[j][3]);

    // History slots (first chunk only, after all of its reads): plane s <- conv_input
    // rows [max(T - s, 0), +K-1).  Rows held in in[] (the history and this chunk's x
    // rows) are taken from there; later x rows are reloaded.
    if (t0 == 0) {
        for (int s = 0; s < p.n_snap; ++s) {
            const int r0 = max(p.T - s, 0);
            float vals[K - 1][4];
#pragma unroll
            for (int r = 0; r < K - 1; ++r) {
                const int row = r0 + r;
                if (row < K - 1 + nt) {
#pragma unroll
                    for (int rr = 0; rr < K - 1 + TC; ++rr)
                        if (rr == row)
#pragma unroll
                            for (int e = 0; e < 4; ++e) vals[r][e] = in[rr][e];
                } else {
                    const float4 v = ld4<DT>(p.x, xb + static_cast<int64_t>(row - (K - 1)) * p.x_st);
                    vals[r][0] = v.x;
                    vals[r][1] = v.y;
                    vals[r][2] = v.z;
                    vals[r][3] = v.w;
                }
            }
            float4 *dst = reinterpret_cast<float4 *>(planes + s * plane_elems + static_cast<size_t>(c0) * (K - 1));
#pragma unroll
            for (int i = 0; i < K - 1; ++i) {
                float4 v;
                v.x = vals[(4 * i + 0) % (K - 1)][(4 * i + 0) / (K - 1)];
                v.y = vals[(4 * i + 1) % (K - 1)][(4 * i + 1) / (K - 1)];
                v.z = vals[(4 * i + 2) % (K - 1)][(4 * i + 2) / (K - 1)];
                v.w = vals[(4 * i + 3) % (K - 1)][(4 * i + 3) / (K - 1)];
                dst[i] = v;
            }
        }
    }
}

struct NormParams {
    const void *x;
    int64_t x_st, x_sh;
    const float *w;
    int64_t w_sh;
    const void *z;
    int64_t z_st, z_sh;
    int T, H;
    float eps;
    float *out;
    int64_t o_st, o_sh;
};

// One warp per (token, head) row of 32 * VPL elements; lane L holds elements
// VPL*L .. VPL*L + VPL - 1 (vector loads).  y = x * (1 / sqrt(mean + eps)) [* w]
// [* silu(z)] -- the multiplication order of rms_norm -> mul -> mul.  The row is read
// completely before it is written (in place is allowed).  Launched with programmatic
// stream serialisation.
template <int VPL, int XT, int ZT>
__global__ void __launch_bounds__(256) head_norm_kernel(NormParams p) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" :::);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + warp;
    if (row >= static_cast<int64_t>(p.T) * p.H) return;
    const int t = static_cast<int>(row / p.H), h = static_cast<int>(row % p.H);
    const int e0 = VPL * lane;
    float v[VPL];
#pragma unroll
    for (int i = 0; i < VPL; i += 4) {
        const float4 a = ld4<XT>(p.x, t * p.x_st + h * p.x_sh + e0 + i);
        v[i] = a.x;
        v[i + 1] = a.y;
        v[i + 2] = a.z;
        v[i + 3] = a.w;
    }
    float s2 = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) s2 = fmaf(v[i], v[i], s2);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, off);
    const float scale = 1.0f / sqrtf(s2 / static_cast<float>(32 * VPL) + p.eps);
#pragma unroll
    for (int i = 0; i < VPL; ++i) v[i] = v[i] * scale;
    if (p.w) {
        const float *w = p.w + h * p.w_sh + e0;
#pragma unroll
        for (int i = 0; i < VPL; i += 4) {
            const float4 a = *reinterpret_cast<const float4 *>(w + i);
            v[i] = v[i] * a.x;
            v[i + 1] = v[i + 1] * a.y;
            v[i + 2] = v[i + 2] * a.z;
            v[i + 3] = v[i + 3] * a.w;
        }
    }
    if constexpr (ZT >= 0) {
#pragma unroll
        for (int i = 0; i < VPL; i += 4) {
            const float4 a = ld4<ZT>(p.z, t * p.z_st + h * p.z_sh + e0 + i);
            v[i] = v[i] * silu(a.x);
            v[i + 1] = v[i + 1] * silu(a.y);
            v[i + 2] = v[i + 2] * silu(a.z);
            v[i + 3] = v[i + 3] * silu(a.w);
        }
    }
    float *o = p.out + t * p.o_st + h * p.o_sh + e0;
#pragma unroll
    for (int i = 0; i < VPL; i += 4)
        *reinterpret_cast<float4 *>(o + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
}

}  // namespace sqmix

using namespace sqmix;

static bool float_dtype(int dt) { return dt == SQMIX_F32 || dt == SQMIX_F16 || dt == SQMIX_BF16; }

static cudaLaunchConfig_t pdl_config(dim3 grid, dim3 block, cudaStream_t st, cudaLaunchAttribute *attr) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cfg;
}

template <int K, int TC>
static cudaError_t launch_conv(const cudaLaunchConfig_t &cfg, int dtype, const ConvParams &p) {
    switch (dtype) {
        case SQMIX_F32: return cudaLaunchKernelEx(&cfg, gdn_conv_kernel<K, TC, SQMIX_F32>, p);
        case SQMIX_BF16: return cudaLaunchKernelEx(&cfg, gdn_conv_kernel<K, TC, SQMIX_BF16>, p);
        default: return cudaLaunchKernelEx(&cfg, gdn_conv_kernel<K, TC, SQMIX_F16>, p);
    }
}

// One token (decode): single-row chunks; otherwise 8-token chunks.
template <int K>
static cudaError_t launch_conv_k(cudaLaunchConfig_t cfg, int dtype, int T, const ConvParams &p) {
    if (T == 1) return launch_conv<K, 1>(cfg, dtype, p);
    cfg.gridDim.y = (T + 7) / 8;
    return launch_conv<K, 8>(cfg, dtype, p);
}

static bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

extern "C" int sqmix_gdn_conv(const sqmix_gdn_conv_args *a, sqmix_stream_t stream) {
    SQMIX_CHECK_ARG(a != nullptr, "gdn_conv: null args");
    SQMIX_CHECK_ARG(a->x && a->weight && a->conv_state && a->out, "gdn_conv: null pointer argument");
    SQMIX_CHECK_ARG(float_dtype(a->x_dtype), "gdn_conv: x dtype %d", a->x_dtype);
    SQMIX_CHECK_ARG(a->n_seqs >= 1 && a->n_tokens >= 1, "gdn_conv: n_seqs=%d n_tokens=%d", a->n_seqs,
                    a->n_tokens);
    SQMIX_CHECK_ARG(a->kernel >= 2 && a->kernel <= 8, "gdn_conv: kernel=%d (supported: 2..8)", a->kernel);
    SQMIX_CHECK_ARG(a->head_dim == 128, "gdn_conv: head_dim=%d (supported: 128)", a->head_dim);
    SQMIX_CHECK_ARG(a->channels >= 128 && a->channels % 128 == 0, "gdn_conv: channels=%d must be a multiple of 128",
                    a->channels);
    SQMIX_CHECK_ARG(a->n_qk_channels >= 0 && a->n_qk_channels <= a->channels && a->n_qk_channels % 128 == 0,
                    "gdn_conv: n_qk_channels=%d", a->n_qk_channels);
    SQMIX_CHECK_ARG(a->l2_eps >= 0.f, "gdn_conv: l2_eps must be >= 0");
    SQMIX_CHECK_ARG(a->n_planes >= 1 && a->n_snap >= 1 && a->n_snap <= a->n_planes,
                    "gdn_conv: n_snap=%d n_planes=%d", a->n_snap, a->n_planes);
    SQMIX_CHECK_ARG(a->x_stride_tok >= a->channels && a->x_stride_tok % 4 == 0 &&
                        (a->n_seqs == 1 || (a->x_stride_seq >= a->x_stride_tok && a->x_stride_seq % 4 == 0)),
                    "gdn_conv: x strides (multiples of 4 elements, rows of >= C)");
    SQMIX_CHECK_ARG(aligned16(a->x) && aligned16(a->weight) && aligned16(a->conv_state) && aligned16(a->out),
                    "gdn_conv: x, weight, conv_state and out must be 16-byte aligned");
    ConvParams p;
    p.x = a->x;
    p.x_st = a->x_stride_tok;
    p.x_ss = a->x_stride_seq;
    p.w = a->weight;
    p.state = a->conv_state;
    p.n_planes = a->n_planes;
    p.sel = a->sel;
    p.n_snap = a->n_snap;
    p.T = a->n_tokens;
    p.C = a->channels;
    p.n_qk = a->n_qk_channels;
    p.eps = a->l2_eps;
    p.out = a->out;
    cudaLaunchAttribute attr[1];
    const cudaLaunchConfig_t cfg = pdl_config(dim3((a->channels / 128 + 3) / 4, a->n_tokens, a->n_seqs), dim3(128),
                                              reinterpret_cast<cudaStream_t>(stream), attr);
    cudaError_t e;
    switch (a->kernel) {
        case 2: e = launch_conv_k<2>(cfg, a->x_dtype, a->n_tokens, p); break;
        case 3: e = launch_conv_k<3>(cfg, a->x_dtype, a->n_tokens, p); break;
        case 4: e = launch_conv_k<4>(cfg, a->x_dtype, a->n_tokens, p); break;
        case 5: e = launch_conv_k<5>(cfg, a->x_dtype, a->n_tokens, p); break;
        case 6: e = launch_conv_k<6>(cfg, a->x_dtype, a->n_tokens, p); break;
        case 7: e = launch_conv_k<7>(cfg, a->x_dtype, a->n_tokens, p); break;
        default: e = launch_conv_k<8>(cfg, a->x_dtype, a->n_tokens, p); break;
    }
    return cuda_status(e, "gdn_conv launch");
}

template <int VPL, int XT>
static cudaError_t launch_norm_z(const cudaLaunchConfig_t &cfg, int z_dtype, bool has_z, const NormParams &p) {
    if (!has_z) return cudaLaunchKernelEx(&cfg, head_norm_kernel<VPL, XT, -1>, p);
    switch (z_dtype) {
        case SQMIX_F32: return cudaLaunchKernelEx(&cfg, head_norm_kernel<VPL, XT, SQMIX_F32>, p);
        case SQMIX_BF16: return cudaLaunchKernelEx(&cfg, head_norm_kernel<VPL, XT, SQMIX_BF16>, p);
        default: return cudaLaunchKernelEx(&cfg, head_norm_kernel<VPL, XT, SQMIX_F16>, p);
    }
}

template <int VPL>
static cudaError_t launch_norm(const cudaLaunchConfig_t &cfg, int x_dtype, int z_dtype, bool has_z,
                               const NormParams &p) {
    switch (x_dtype) {
        case SQMIX_F32: return launch_norm_z<VPL, SQMIX_F32>(cfg, z_dtype, has_z, p);
        case SQMIX_BF16: return launch_norm_z<VPL, SQMIX_BF16>(cfg, z_dtype, has_z, p);
        default: return launch_norm_z<VPL, SQMIX_F16>(cfg, z_dtype, has_z, p);
    }
}

extern "C" int sqmix_head_norm(const sqmix_head_norm_args *a, sqmix_stream_t stream) {
    SQMIX_CHECK_ARG(a != nullptr, "head_norm: null args");
    SQMIX_CHECK_ARG(a->x && a->out, "head_norm: null pointer argument");
    SQMIX_CHECK_ARG(float_dtype(a->x_dtype), "head_norm: x dtype %d", a->x_dtype);
    SQMIX_CHECK_ARG(!a->z || float_dtype(a->z_dtype), "head_norm: z dtype %d", a->z_dtype);
    SQMIX_CHECK_ARG(a->n_tokens >= 1 && a->n_heads >= 1, "head_norm: n_tokens=%d n_heads=%d", a->n_tokens,
                    a->n_heads);
    SQMIX_CHECK_ARG(a->head_dim == 128 || a->head_dim == 256, "head_norm: head_dim=%d (supported: 128, 256)",
                    a->head_dim);
    SQMIX_CHECK_ARG(a->eps >= 0.f, "head_norm: eps must be >= 0");
    SQMIX_CHECK_ARG(a->x_stride_tok % 4 == 0 && a->x_stride_head % 4 == 0 && a->out_stride_tok % 4 == 0 &&
                        a->out_stride_head % 4 == 0 && a->weight_stride_head % 4 == 0 &&
                        (!a->z || (a->z_stride_tok % 4 == 0 && a->z_stride_head % 4 == 0)),
                    "head_norm: strides must be multiples of 4 elements");
    SQMIX_CHECK_ARG(aligned16(a->x) && aligned16(a->out) && aligned16(a->weight) && aligned16(a->z),
                    "head_norm: x, out, weight and z must be 16-byte aligned");
    NormParams p;
    p.x = a->x;
    p.x_st = a->x_stride_tok;
    p.x_sh = a->x_stride_head;
    p.w = a->weight;
    p.w_sh = a->weight_stride_head;
    p.z = a->z;
    p.z_st = a->z_stride_tok;
    p.z_sh = a->z_stride_head;
    p.T = a->n_tokens;
    p.H = a->n_heads;
    p.eps = a->eps;
    p.out = a->out;
    p.o_st = a->out_stride_tok;
    p.o_sh = a->out_stride_head;
    const int64_t rows = static_cast<int64_t>(a->n_tokens) * a->n_heads;
    SQMIX_CHECK_ARG(rows <= 8LL * 0x7fffffff, "head_norm: too many rows");
    cudaLaunchAttribute attr[1];
    const cudaLaunchConfig_t cfg = pdl_config(dim3(static_cast<unsigned>((rows + 7) / 8)), dim3(256),
                                              reinterpret_cast<cudaStream_t>(stream), attr);
    const cudaError_t e = a->head_dim == 128 ? launch_norm<4>(cfg, a->x_dtype, a->z_dtype, a->z != nullptr, p)
                                             : launch_norm<8>(cfg, a->x_dtype, a->z_dtype, a->z != nullptr, p);
    return cuda_status(e, "head_norm launch");
}
