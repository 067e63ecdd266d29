// gdn.cu -- gated delta net recurrence (decode / short verify batches) and state copies.
//
// Replaces ggml_gated_delta_net (src/model/gdn.rs:489-500; recurrence at gdn.rs:9-24)
// together with the state plumbing around it:
//   * the plane select of the MTP rollback (get_rows, gdn.rs:445-463) is the `sel`
//     index read on the device at kernel start (no copy);
//   * the snapshot write-back (ggml_cpy of graph.rs:884-912, which ggml-cuda fuses
//     into the op) is done in place: slot s <- state after T - s tokens.
//
// Each value column j of a head evolves independently:
//     S'      = exp(g) S
//     delta_j = beta (v_j - sum_i S'_ij k_i)
//     S_ij    = S'_ij + k_i delta_j
//     o_j     = (sum_i S'_ij q_i + delta_j (k . q)) / sqrt(128)
// so one warp owns one column (128 f32 = 4 per lane, a single 16-byte load and
// store per plane), the whole 2 MiB state of a layer streams through HBM once in
// and n_snap times out, and no inter-warp communication is needed.
#include <math.h>

#include "common.cuh"

namespace sqmix {

struct GdnParams {
    const void *q;
    const void *k;
    const void *v;
    int dtype;
    int64_t qk_st, v_st, qk_sseq, v_sseq;
    const float *g;
    const float *beta;
    float *state;
    int n_planes;
    const int32_t *sel;
    int n_seqs, T, h_k, h_v, n_snap;
    float l2_eps;
    float *out;
    int plane0;   // input plane when sel is NULL
    int T_all;    // tokens per sequence in g, beta and out
    int64_t tok0; // first token of this launch within the sequence
    int state_ready;  // read the input state before waiting on the preceding kernel
    int h_v_off;      // layer index of value head 0 (value-head sharding)
    const float *dt_bias, *ssm_a;  // gate epilogue (ssm_a NULL: g, beta as given)
};

__device__ __forceinline__ float4 load4(const void *p, int64_t i, int dtype) {
    if (dtype == SQMIX_F32) return *reinterpret_cast<const float4 *>(static_cast<const float *>(p) + i);
    if (dtype == SQMIX_BF16) {
        const uint2 r = *reinterpret_cast<const uint2 *>(static_cast<const __nv_bfloat16 *>(p) + i);
        const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162 *>(&r.x);
        const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162 *>(&r.y);
        return make_float4(__low2float(a), __high2float(a), __low2float(b), __high2float(b));
    }
    const uint2 r = *reinterpret_cast<const uint2 *>(static_cast<const __half *>(p) + i);
    const __half2 a = *reinterpret_cast<const __half2 *>(&r.x);
    const __half2 b = *reinterpret_cast<const __half2 *>(&r.y);
    return make_float4(__low2float(a), __high2float(a), __low2float(b), __high2float(b));
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
    return x;
}

// L2 norm as gdn.rs:133-142 builds it: rms_norm(x, eps/n) then scale 1/sqrt(n).
__device__ __forceinline__ float4 l2norm4(float4 x, float eps) {
    const float ss = warp_sum(x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w);
    const float mean = ss / 128.0f;
    const float s = 1.0f / sqrtf(mean + eps / 128.0f);
    const float s2 = 1.0f / sqrtf(128.0f);
    return make_float4(x.x * s * s2, x.y * s * s2, x.z * s * s2, x.w * s * s2);
}

// grid: (n_seqs * h_v * 128 / JW / 8), block 256: warp -> (seq, head, JW consecutive
// value columns).  q, k, their norms and k.q are shared by the warp's columns; each
// lane keeps keys 4*lane..4*lane+3 of every column, so a warp has JW 16-byte loads
// in flight per lane (more columns per warp where there is enough work to spread).
// 8 columns (large batches): at most 64 registers, so 4 blocks (32 warps) per SM keep
// more state loads in flight (80 registers and 3 blocks measured 4.5 % slower for a
// 64-sequence batch; no spills at 64).  4 columns carry no minimum (0): bounding them
// measured 8 % slower for a single sequence, whose launch is latency bound.
template <int JW>
__global__ void __launch_bounds__(256, JW == 8 ? 4 : 0) gdn_recurrent_kernel(GdnParams p) {
    const int lane = threadIdx.x & 31;
    const int64_t wid = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
    constexpr int kGroups = 128 / JW;
    const int j0 = static_cast<int>(wid % kGroups) * JW;
    const int64_t hs = wid / kGroups;
    const int h = static_cast<int>(hs % p.h_v);
    const int64_t seq = hs / p.h_v;
    if (seq >= p.n_seqs) return;
    const int hk = (p.h_v_off + h) % p.h_k;
    // launched with programmatic stream serialisation: the launch overlaps the tail of
    // the kernel before it, whose results everything after griddepcontrol.wait may
    // use; with state_ready the caller guarantees that kernel writes neither the state
    // nor sel, so the state is read before the wait
    if (!p.state_ready) asm volatile("griddepcontrol.wait;" ::: "memory");

    int plane = p.sel ? p.sel[seq] : p.plane0;
    plane = min(max(plane, 0), p.n_planes - 1);
    const int64_t plane_elems = static_cast<int64_t>(p.h_v) * 128 * 128;
    float *st_seq = p.state + seq * p.n_planes * plane_elems;
    const int64_t col_off = (static_cast<int64_t>(h) * 128 + j0) * 128 + 4 * lane;  // column j0
    float4 S[JW];
#pragma unroll
    for (int c = 0; c < JW; ++c)
        S[c] = *reinterpret_cast<const float4 *>(st_seq + plane * plane_elems + col_off + c * 128);
    if (p.state_ready) asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" :::);

    const float inv_sqrt_d = 1.0f / sqrtf(128.0f);
    for (int t = 0; t < p.T; ++t) {
        const int64_t tt = p.tok0 + t;
        const int64_t qk_off = seq * p.qk_sseq + tt * p.qk_st + static_cast<int64_t>(hk) * 128 + 4 * lane;
        float4 kk = load4(p.k, qk_off, p.dtype);
        float4 qq = load4(p.q, qk_off, p.dtype);
        if (p.l2_eps > 0.f) {
            kk = l2norm4(kk, p.l2_eps);
            qq = l2norm4(qq, p.l2_eps);
        }
        const int64_t gb = (seq * p.T_all + tt) * p.h_v + h;
        float gl = p.g[gb], bt = p.beta[gb];
        gdn_gates(gl, bt, p.dt_bias, p.ssm_a, p.h_v_off + h);
        const float decay = expf(gl);
        const int64_t v_off = seq * p.v_sseq + tt * p.v_st + static_cast<int64_t>(h) * 128 + j0;
        float vj[JW];
#pragma unroll
        for (int c = 0; c < JW; ++c) vj[c] = load_act(p.v, v_off + c, p.dtype);
        float skv[JW], sq[JW];
#pragma unroll
        for (int c = 0; c < JW; ++c) {
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
            for (int c = 0; c < JW; ++c) {
                skv[c] += __shfl_xor_sync(0xffffffffu, skv[c], off);
                sq[c] += __shfl_xor_sync(0xffffffffu, sq[c], off);
            }
            kq += __shfl_xor_sync(0xffffffffu, kq, off);
        }
        float o[JW];
#pragma unroll
        for (int c = 0; c < JW; ++c) {
            const float delta = (vj[c] - skv[c]) * bt;
            S[c].x = fmaf(kk.x, delta, S[c].x);
            S[c].y = fmaf(kk.y, delta, S[c].y);
            S[c].z = fmaf(kk.z, delta, S[c].z);
            S[c].w = fmaf(kk.w, delta, S[c].w);
            o[c] = fmaf(delta, kq, sq[c]) * inv_sqrt_d;
        }
        if (lane == 0) {
            float *orow = p.out + ((seq * p.T_all + tt) * p.h_v + h) * 128 + j0;
#pragma unroll
            for (int c = 0; c < JW; ++c) orow[c] = o[c];
        }
        const int slot = p.T - 1 - t;
        if (slot < p.n_snap) {
#pragma unroll
            for (int c = 0; c < JW; ++c)
                *reinterpret_cast<float4 *>(st_seq + slot * plane_elems + col_off + c * 128) = S[c];
        }
    }
}

__global__ void copy_f32x4_kernel(float4 *dst, const float4 *src, int64_t n4) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        dst[i] = src[i];
}

}  // namespace sqmix

namespace sqmix {
int gdn_launch_recurrent(const sqmix_gdn_args *a, int plane_in, int64_t tok_off, int n_tok, int n_snap,
                         bool state_ready, cudaStream_t st) {
    GdnParams p;
    p.state_ready = state_ready ? 1 : 0;
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
    p.state = a->state;
    p.n_planes = a->n_planes;
    p.sel = plane_in < 0 ? a->sel : nullptr;
    p.plane0 = plane_in < 0 ? 0 : plane_in;
    p.n_seqs = a->n_seqs;
    p.T = n_tok;
    p.T_all = a->n_tokens;
    p.tok0 = tok_off;
    p.h_k = a->h_k;
    p.h_v = a->h_v;
    p.n_snap = n_snap;
    p.l2_eps = a->l2_eps;
    p.out = a->out;
    p.h_v_off = a->h_v_offset;
    p.dt_bias = a->dt_bias;
    p.ssm_a = a->ssm_a;
    // columns per warp: 8 once that still leaves two waves of resident warps, else 4.
    // Measured on B200 (32 value heads, per layer): 4 columns beat 1 and 2 at every
    // batch from 1 to 32 (batch 8: 7.7 us against 13.5 with 1), 8 wins from batch 64.
    const int64_t cols = static_cast<int64_t>(a->n_seqs) * a->h_v * 128;
    const int64_t resident = static_cast<int64_t>(sqmix_device_sm_count(-1)) * 64;
    const int jw = cols / 8 >= 2 * resident ? 8 : 4;
    const int64_t warps = cols / jw;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(warps / 8));
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e;
    if (jw == 8)
        e = cudaLaunchKernelEx(&cfg, gdn_recurrent_kernel<8>, p);
    else
        e = cudaLaunchKernelEx(&cfg, gdn_recurrent_kernel<4>, p);
    return cuda_status(e, "gdn recurrent launch");
}
}  // namespace sqmix

using namespace sqmix;

extern "C" int sqmix_gdn_decode(const sqmix_gdn_args *a, sqmix_stream_t stream) {
    SQMIX_CHECK_ARG(a != nullptr, "gdn_decode: null args");
    SQMIX_CHECK_ARG(a->q && a->k && a->v && a->g && a->beta && a->state && a->out,
                    "gdn_decode: null pointer argument");
    SQMIX_CHECK_ARG(a->dtype == SQMIX_F32 || a->dtype == SQMIX_F16 || a->dtype == SQMIX_BF16,
                    "gdn_decode: dtype %d", a->dtype);
    SQMIX_CHECK_ARG(a->h_k >= 1 && a->h_v >= 1 && a->h_v_offset >= 0, "gdn_decode: h_k=%d h_v=%d h_v_offset=%d",
                    a->h_k, a->h_v, a->h_v_offset);
    SQMIX_CHECK_ARG(a->n_seqs >= 1 && a->n_tokens >= 1, "gdn_decode: n_seqs=%d T=%d", a->n_seqs,
                    a->n_tokens);
    SQMIX_CHECK_ARG(a->n_planes >= 1, "gdn_decode: n_planes=%d", a->n_planes);
    SQMIX_CHECK_ARG(a->n_snap >= 1 && a->n_snap <= a->n_tokens && a->n_snap <= a->n_planes,
                    "gdn_decode: n_snap=%d must be in [1, min(T=%d, n_planes=%d)]", a->n_snap,
                    a->n_tokens, a->n_planes);
    SQMIX_CHECK_ARG(a->qk_stride_tok >= (int64_t)a->h_k * 128 && a->v_stride_tok >= (int64_t)a->h_v * 128,
                    "gdn_decode: token strides too small");
    SQMIX_CHECK_ARG(a->qk_stride_tok % 4 == 0 && a->qk_stride_seq % 4 == 0,
                    "gdn_decode: q/k strides must be multiples of 4 elements");
    SQMIX_CHECK_ARG((reinterpret_cast<uintptr_t>(a->state) & 15) == 0, "gdn_decode: state alignment");
    {
        // q/k are read 4 elements per lane (16 bytes for f32, 8 for bf16/f16)
        const uintptr_t align = a->dtype == SQMIX_F32 ? 15 : 7;
        SQMIX_CHECK_ARG(((reinterpret_cast<uintptr_t>(a->q) | reinterpret_cast<uintptr_t>(a->k)) & align) == 0,
                        "gdn_decode: q/k base pointers must be %d-byte aligned", (int)align + 1);
    }
    SQMIX_CHECK_ARG((a->flags & ~SQMIX_GDN_STATE_READY) == 0, "gdn_decode: unknown flags 0x%x", a->flags);
    return gdn_launch_recurrent(a, -1, 0, a->n_tokens, a->n_snap, (a->flags & SQMIX_GDN_STATE_READY) != 0,
                                reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int sqmix_gdn_state_copy(float *dst, const float *src, int64_t plane_elems, int32_t n_planes,
                                    sqmix_stream_t stream) {
    SQMIX_CHECK_ARG(dst && src, "gdn_state_copy: null pointer");
    SQMIX_CHECK_ARG(plane_elems > 0 && plane_elems % 4 == 0 && n_planes >= 1,
                    "gdn_state_copy: plane_elems=%lld n_planes=%d", (long long)plane_elems, n_planes);
    SQMIX_CHECK_ARG(((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15) == 0,
                    "gdn_state_copy: 16-byte alignment required");
    const int64_t n4 = plane_elems * n_planes / 4;
    int blocks = static_cast<int>((n4 + 255) / 256);
    if (blocks > 4 * sqmix_device_sm_count(-1)) blocks = 4 * sqmix_device_sm_count(-1);
    copy_f32x4_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<float4 *>(dst), reinterpret_cast<const float4 *>(src), n4);
    return cuda_status(cudaGetLastError(), "gdn_state_copy launch");
}
