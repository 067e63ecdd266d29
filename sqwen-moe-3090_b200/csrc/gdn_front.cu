// gdn_front.cu -- the GDN front end (short causal convolution + SiLU + q/k L2 norm,
// with the conv-history planes) and the per-head RMS norms of both mixers.
//
// Replaces, per GDN layer step (src/model/gdn.rs:290-441, src/model/graph.rs:913-961):
//   ggml_concat(conv history, qkv^T) -> ggml_ssm_conv -> ggml_silu -> views of q/k/v
//   -> l2_norm(q), l2_norm(k), and the per-slot ggml_cpy of the conv tails;
// and the norms (attn.rs:66-84 head_rms_norm of Q and K; gdn.rs:150-181 norm_gated).
//
// Both kernels are HBM/latency-bound elementwise work with one reduction per head:
//   gdn_conv_kernel: one CTA per (head-wide block of channels, 16-token chunk,
//     sequence), one thread per channel.  A thread keeps its channel's K taps and a
//     sliding window of K-1 conv inputs in registers; the chunk's tokens are loaded
//     at once (coalesced across channels).  The L2 norm of a q/k head is a block
//     reduction per token (warp shuffles + one shared-memory pass for the chunk).
//     Only the first chunk reads the history plane, and the same CTA writes the
//     history slots after it has read everything it needs, so the in-place update
//     of the resident planes has no cross-CTA hazard.
//   head_norm_kernel: one warp per (token, head) row.
#include <math.h>

#include "common.cuh"

namespace sqmix {

constexpr int kConvChunk = 16;  // tokens per CTA

struct ConvParams {
    const void *x;
    int x_dtype;
    int64_t x_st, x_ss;
    const float *w;
    float *state;
    int n_planes;
    const int32_t *sel;
    int n_snap;
    int T, C, d, n_qk;
    float eps;
    float *out;
};

__device__ __forceinline__ float silu(float y) { return y / (1.0f + expf(-y)); }

template <int K>
__global__ void __launch_bounds__(256) gdn_conv_kernel(ConvParams p) {
    __shared__ float red[8][kConvChunk];
    const int c = blockIdx.x * p.d + threadIdx.x;
    const int seq = blockIdx.z;
    const int t0 = blockIdx.y * kConvChunk;
    const int nt = min(kConvChunk, p.T - t0);
    const int64_t xbase = static_cast<int64_t>(seq) * p.x_ss + c;
    const size_t plane_elems = static_cast<size_t>(p.C) * (K - 1);
    float *planes = p.state + static_cast<size_t>(seq) * p.n_planes * plane_elems;

    float w[K];
#pragma unroll
    for (int k = 0; k < K; ++k) w[k] = p.w[static_cast<size_t>(c) * K + k];
    // History: the first chunk reads plane sel; later chunks start inside x.
    float hist[K - 1];
    if (t0 == 0) {
        const int sel = p.sel ? p.sel[seq] : 0;
        const float *h = planes + static_cast<size_t>(sel) * plane_elems + static_cast<size_t>(c) * (K - 1);
#pragma unroll
        for (int r = 0; r < K - 1; ++r) hist[r] = h[r];
    }
    // conv_input rows t0 .. t0 + nt + K - 2 for this channel: win[0..K-2] then xv[]
    float in[kConvChunk + K - 1];
#pragma unroll
    for (int r = 0; r < K - 1; ++r)
        in[r] = t0 == 0 ? hist[r] : load_act(p.x, xbase + static_cast<int64_t>(t0 - (K - 1) + r) * p.x_st, p.x_dtype);
#pragma unroll
    for (int j = 0; j < kConvChunk; ++j)
        in[K - 1 + j] = j < nt ? load_act(p.x, xbase + static_cast<int64_t>(t0 + j) * p.x_st, p.x_dtype) : 0.f;

    float y[kConvChunk];
#pragma unroll
    for (int j = 0; j < kConvChunk; ++j) {
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < K; ++k) s = __fadd_rn(s, __fmul_rn(in[j + k], w[k]));
        y[j] = silu(s);
    }

    // L2 norm per head of the q/k channels (block = one head): x / ||x|| as
    // scale(rms_norm(x, eps / d), 1 / sqrt(d)), gdn.rs:133-142.
    if (p.eps > 0.f && blockIdx.x * p.d < p.n_qk) {
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
#pragma unroll
        for (int j = 0; j < kConvChunk; ++j) {
            float s2 = y[j] * y[j];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, off);
            if (lane == 0) red[warp][j] = s2;
        }
        __syncthreads();
        const float fd = static_cast<float>(p.d);
        const float s_d = 1.0f / sqrtf(fd);
#pragma unroll
        for (int j = 0; j < kConvChunk; ++j) {
            float sum = 0.f;
            for (int i = 0; i < nw; ++i) sum += red[i][j];
            const float sc = 1.0f / sqrtf(sum / fd + p.eps / fd);
            y[j] = (y[j] * sc) * s_d;
        }
    }
    float *o = p.out + (static_cast<size_t>(seq) * p.T + t0) * p.C + c;
#pragma unroll
    for (int j = 0; j < kConvChunk; ++j)
        if (j < nt) o[static_cast<size_t>(j) * p.C] = y[j];

    // History slots (first chunk only, after all of its reads): plane s <- conv_input
    // rows [max(T - s, 0), +K-1), row r being hist[r] for r < K-1, else x[r - (K-1)].
    if (t0 == 0) {
        for (int s = 0; s < p.n_snap; ++s) {
            const int r0 = max(p.T - s, 0);
            float *dst = planes + static_cast<size_t>(s) * plane_elems + static_cast<size_t>(c) * (K - 1);
#pragma unroll
            for (int r = 0; r < K - 1; ++r) {
                const int row = r0 + r;
                dst[r] = row < K - 1 ? hist[row]
                                     : load_act(p.x, xbase + static_cast<int64_t>(row - (K - 1)) * p.x_st, p.x_dtype);
            }
        }
    }
}

struct NormParams {
    const void *x;
    int x_dtype;
    int64_t x_st, x_sh;
    const float *w;
    int64_t w_sh;
    const void *z;
    int z_dtype;
    int64_t z_st, z_sh;
    int T, H, d;
    float eps;
    float *out;
    int64_t o_st, o_sh;
};

// One warp per (token, head): sum of squares, then y = x * (1 / sqrt(mean + eps))
// [* w] [* silu(z)] -- the multiplication order of rms_norm -> mul -> mul.
__global__ void __launch_bounds__(256) head_norm_kernel(NormParams p) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + warp;
    if (row >= static_cast<int64_t>(p.T) * p.H) return;
    const int t = static_cast<int>(row / p.H), h = static_cast<int>(row % p.H);
    const int64_t xb = t * p.x_st + h * p.x_sh;
    float s2 = 0.f;
    for (int i = lane; i < p.d; i += 32) {
        const float v = load_act(p.x, xb + i, p.x_dtype);
        s2 = fmaf(v, v, s2);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, off);
    const float scale = 1.0f / sqrtf(s2 / static_cast<float>(p.d) + p.eps);
    const float *w = p.w ? p.w + h * p.w_sh : nullptr;
    const int64_t zb = t * p.z_st + h * p.z_sh;
    float *o = p.out + t * p.o_st + h * p.o_sh;
    for (int i = lane; i < p.d; i += 32) {
        float y = load_act(p.x, xb + i, p.x_dtype) * scale;
        if (w) y = y * w[i];
        if (p.z) y = y * silu(load_act(p.z, zb + i, p.z_dtype));
        o[i] = y;
    }
}

}  // namespace sqmix

using namespace sqmix;

static bool float_dtype(int dt) { return dt == SQMIX_F32 || dt == SQMIX_F16 || dt == SQMIX_BF16; }

extern "C" int sqmix_gdn_conv(const sqmix_gdn_conv_args *a, sqmix_stream_t stream) {
    SQMIX_CHECK_ARG(a != nullptr, "gdn_conv: null args");
    SQMIX_CHECK_ARG(a->x && a->weight && a->conv_state && a->out, "gdn_conv: null pointer argument");
    SQMIX_CHECK_ARG(float_dtype(a->x_dtype), "gdn_conv: x dtype %d", a->x_dtype);
    SQMIX_CHECK_ARG(a->n_seqs >= 1 && a->n_tokens >= 1, "gdn_conv: n_seqs=%d n_tokens=%d", a->n_seqs,
                    a->n_tokens);
    SQMIX_CHECK_ARG(a->kernel >= 2 && a->kernel <= 8, "gdn_conv: kernel=%d (supported: 2..8)", a->kernel);
    SQMIX_CHECK_ARG(a->head_dim >= 32 && a->head_dim <= 256 && a->head_dim % 32 == 0,
                    "gdn_conv: head_dim=%d must be a multiple of 32 in [32, 256]", a->head_dim);
    SQMIX_CHECK_ARG(a->channels >= a->head_dim && a->channels % a->head_dim == 0,
                    "gdn_conv: channels=%d must be a multiple of head_dim=%d", a->channels, a->head_dim);
    SQMIX_CHECK_ARG(a->n_qk_channels >= 0 && a->n_qk_channels <= a->channels &&
                        a->n_qk_channels % a->head_dim == 0,
                    "gdn_conv: n_qk_channels=%d", a->n_qk_channels);
    SQMIX_CHECK_ARG(a->l2_eps >= 0.f, "gdn_conv: l2_eps must be >= 0");
    SQMIX_CHECK_ARG(a->n_planes >= 1 && a->n_snap >= 1 && a->n_snap <= a->n_planes,
                    "gdn_conv: n_snap=%d n_planes=%d", a->n_snap, a->n_planes);
    SQMIX_CHECK_ARG(a->x_stride_tok >= a->channels && (a->n_seqs == 1 || a->x_stride_seq >= a->x_stride_tok),
                    "gdn_conv: x strides");
    ConvParams p;
    p.x = a->x;
    p.x_dtype = a->x_dtype;
    p.x_st = a->x_stride_tok;
    p.x_ss = a->x_stride_seq;
    p.w = a->weight;
    p.state = a->conv_state;
    p.n_planes = a->n_planes;
    p.sel = a->sel;
    p.n_snap = a->n_snap;
    p.T = a->n_tokens;
    p.C = a->channels;
    p.d = a->head_dim;
    p.n_qk = a->n_qk_channels;
    p.eps = a->l2_eps;
    p.out = a->out;
    const dim3 grid(a->channels / a->head_dim, (a->n_tokens + kConvChunk - 1) / kConvChunk, a->n_seqs);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    switch (a->kernel) {
        case 2: gdn_conv_kernel<2><<<grid, a->head_dim, 0, st>>>(p); break;
        case 3: gdn_conv_kernel<3><<<grid, a->head_dim, 0, st>>>(p); break;
        case 4: gdn_conv_kernel<4><<<grid, a->head_dim, 0, st>>>(p); break;
        case 5: gdn_conv_kernel<5><<<grid, a->head_dim, 0, st>>>(p); break;
        case 6: gdn_conv_kernel<6><<<grid, a->head_dim, 0, st>>>(p); break;
        case 7: gdn_conv_kernel<7><<<grid, a->head_dim, 0, st>>>(p); break;
        default: gdn_conv_kernel<8><<<grid, a->head_dim, 0, st>>>(p); break;
    }
    return cuda_status(cudaGetLastError(), "gdn_conv launch");
}

extern "C" int sqmix_head_norm(const sqmix_head_norm_args *a, sqmix_stream_t stream) {
    SQMIX_CHECK_ARG(a != nullptr, "head_norm: null args");
    SQMIX_CHECK_ARG(a->x && a->out, "head_norm: null pointer argument");
    SQMIX_CHECK_ARG(float_dtype(a->x_dtype), "head_norm: x dtype %d", a->x_dtype);
    SQMIX_CHECK_ARG(!a->z || float_dtype(a->z_dtype), "head_norm: z dtype %d", a->z_dtype);
    SQMIX_CHECK_ARG(a->n_tokens >= 1 && a->n_heads >= 1 && a->head_dim >= 1, "head_norm: shape");
    SQMIX_CHECK_ARG(a->eps >= 0.f, "head_norm: eps must be >= 0");
    NormParams p;
    p.x = a->x;
    p.x_dtype = a->x_dtype;
    p.x_st = a->x_stride_tok;
    p.x_sh = a->x_stride_head;
    p.w = a->weight;
    p.w_sh = a->weight_stride_head;
    p.z = a->z;
    p.z_dtype = a->z_dtype;
    p.z_st = a->z_stride_tok;
    p.z_sh = a->z_stride_head;
    p.T = a->n_tokens;
    p.H = a->n_heads;
    p.d = a->head_dim;
    p.eps = a->eps;
    p.out = a->out;
    p.o_st = a->out_stride_tok;
    p.o_sh = a->out_stride_head;
    const int64_t rows = static_cast<int64_t>(a->n_tokens) * a->n_heads;
    SQMIX_CHECK_ARG(rows <= 8LL * 0x7fffffff, "head_norm: too many rows");
    head_norm_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p);
    return cuda_status(cudaGetLastError(), "head_norm launch");
}
