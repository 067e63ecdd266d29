// mul_mat.cu -- the mixer projections at decode: ggml_mul_mat(w, x) as sqwen builds
// them (QG / K / V, src/model/attn.rs:127-129; W_o, attn.rs:285; qkv / z / beta / alpha,
// src/model/gdn.rs:264-276; out, gdn.rs:577):
//     y[t][o] = sum_i W[o][i] x[t][i],   o < n_out, i < n_in, t < n_tokens,
// W being ggml's [n_in, n_out] tensor (n_out contiguous rows of n_in values) in a GGUF
// block format: q8_0, q4_K, q6_K (the types of a Q4_K_M model's projection weights), or
// f32 / f16 / bf16.  Dequantised weights times x are summed in f32.  (ggml's CUDA
// backend quantises x to q8_1 for its quantised dot products; this path does not.)
//
// At decode a projection is a stream of its weight bytes.  One CTA per SM walks a
// contiguous range of row tiles; a tile (one shared-memory slot) holds up to 8
// consecutive rows -- contiguous bytes of the tensor -- brought in by a 1-D bulk copy
// (TMA, no multicast) on an mbarrier ring.  The ring is filled before the grid-
// dependency wait: the weights are model constants, only x comes from the kernel
// before.  Warp w takes row w of a tile; lane l takes the 32-value sub-block l % 8 of the
// row's 256-value units l / 8, l / 8 + 4, ..., dequantises it from shared memory into
// registers and multiplies it with the staged tokens (f32 in shared memory, 32-value
// sub-blocks padded to 36 floats so that the 8 lanes of a unit read 8 different bank
// groups).  q4_K's min term uses the per-sub-block sums of x.  The warp then reduces
// its lanes by shuffles.  A call handles up to kMaxPassTokens tokens per stream of W.
#include <math.h>

#include "common.cuh"
#include "sqmix.h"

namespace sqmix {
namespace {

constexpr int kMmWarps = 8;
constexpr int kMmThreads = kMmWarps * 32;
constexpr int kMaxIn = 4096;          // n_in limit (the model's 2048 and 4096)
constexpr int kMaxPassTokens = 4;     // tokens per stream of W
constexpr int kSubPad = 36;           // floats per staged 32-value sub-block
constexpr int kRingBudget = 96 * 1024;
constexpr int kMaxStages = 8;
constexpr int kSlotMax = 32 * 1024;   // bytes of one slot (<= 8 rows)

struct MmParams {
    const uint8_t *w;
    int w_type;
    int64_t row_bytes;
    int n_in, n_out;
    const void *x;
    int x_dtype;
    int64_t x_stride;
    int n_tok;  // tokens of this pass (<= NT)
    float *y;
    int64_t y_stride;
    uint32_t *status;
    int rows_per_slot, n_stages, slot_bytes;
};

__device__ __forceinline__ float f16_at(const uint8_t *p) {
    return __half2float(*reinterpret_cast<const __half *>(p));
}

// 32 bytes from a 2-byte aligned shared-memory address as 8 words
__device__ __forceinline__ void ld32b(const uint8_t *p, uint32_t (&w)[8]) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    if ((a & 3) == 0) {
        const uint32_t *q = reinterpret_cast<const uint32_t *>(p);
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = q[i];
    } else {
        const uint32_t *q = reinterpret_cast<const uint32_t *>(p - 2);
        uint32_t r[9];
#pragma unroll
        for (int i = 0; i < 9; ++i) r[i] = q[i];
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = __byte_perm(r[i], r[i + 1], 0x5432);
    }
}

// Unit (256 values) bytes per format; 0: unsupported.
__host__ __device__ constexpr int unit_bytes(int t) {
    return t == SQMIX_Q4_K ? 144 : t == SQMIX_Q6_K ? 210 : t == SQMIX_Q8_0 ? 272 : t == SQMIX_F32 ? 1024
           : (t == SQMIX_F16 || t == SQMIX_BF16) ? 512 : 0;
}

// The 32 values of sub-block j (0..7) of one 256-value unit at `u` (shared memory).
// For q4_K the min term is returned separately: value = v[l] - mterm.
template <int WT>
__device__ __forceinline__ void dequant_sub(const uint8_t *u, int j, float (&v)[32], float &mterm) {
    mterm = 0.f;
    if constexpr (WT == SQMIX_Q4_K) {
        const float d = f16_at(u), dmin = f16_at(u + 2);
        const uint8_t *s = u + 4;
        int sc, m;
        if (j < 4) {
            sc = s[j] & 63;
            m = s[j + 4] & 63;
        } else {
            sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
            m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
        }
        const float ds = d * static_cast<float>(sc);
        mterm = dmin * static_cast<float>(m);
        const uint4 *q4 = reinterpret_cast<const uint4 *>(u + 16 + 32 * (j >> 1));
        const uint4 a = q4[0], b = q4[1];
        const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        const int sh = 4 * (j & 1);
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int e = 0; e < 4; ++e) v[4 * i + e] = ds * static_cast<float>((w[i] >> (8 * e + sh)) & 0xF);
    } else if constexpr (WT == SQMIX_Q6_K) {
        const int half = j >> 2, k = j & 3;
        uint32_t ql[8], qh[8];
        ld32b(u + 64 * half + 32 * (k & 1), ql);
        ld32b(u + 128 + 32 * half, qh);
        const int8_t *sc = reinterpret_cast<const int8_t *>(u + 192 + 8 * half + 2 * k);
        const float d = f16_at(u + 208);
        const float d0 = d * static_cast<float>(sc[0]), d1 = d * static_cast<float>(sc[1]);
        const int lsh = 4 * (k >> 1), hsh = 2 * k;
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int lo = (ql[i] >> (8 * e + lsh)) & 0xF;
                const int hi = (qh[i] >> (8 * e + hsh)) & 3;
                const float q = static_cast<float>((lo | (hi << 4)) - 32);
                v[4 * i + e] = (i < 4 ? d0 : d1) * q;
            }
    } else if constexpr (WT == SQMIX_Q8_0) {
        const uint8_t *b = u + 34 * j;
        const float d = f16_at(b);
        uint32_t w[8];
        ld32b(b + 2, w);
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int e = 0; e < 4; ++e) v[4 * i + e] = d * static_cast<float>(static_cast<int8_t>((w[i] >> (8 * e)) & 0xFF));
    } else if constexpr (WT == SQMIX_F32) {
        const float4 *f = reinterpret_cast<const float4 *>(u + 128 * j);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 x = f[i];
            v[4 * i] = x.x;
            v[4 * i + 1] = x.y;
            v[4 * i + 2] = x.z;
            v[4 * i + 3] = x.w;
        }
    } else {  // f16 / bf16
        const uint4 *h = reinterpret_cast<const uint4 *>(u + 64 * j);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint4 x = h[i];
            const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                float2 f;
                if constexpr (WT == SQMIX_BF16)
                    f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w[e]));
                else
                    f = __half22float2(*reinterpret_cast<const __half2 *>(&w[e]));
                v[8 * i + 2 * e] = f.x;
                v[8 * i + 2 * e + 1] = f.y;
            }
        }
    }
}

template <int WT, int NT>
__global__ void __launch_bounds__(kMmThreads, 1) mul_mat_kernel(MmParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int ring_bytes = p.n_stages * p.slot_bytes;
    const int n_sub = p.n_in / 32;
    float *xs = reinterpret_cast<float *>(smem + ring_bytes);  // [NT][n_sub][kSubPad]
    float *xsum = xs + NT * n_sub * kSubPad;                   // [NT][n_sub]
    uint64_t *full_bar = reinterpret_cast<uint64_t *>(xsum + NT * n_sub);
    uint64_t *empty_bar = full_bar + kMaxStages;
    int *rel_cnt = reinterpret_cast<int *>(empty_bar + kMaxStages);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    const int n_tiles_all = (p.n_out + p.rows_per_slot - 1) / p.rows_per_slot;
    const int tile0 = static_cast<int>((static_cast<int64_t>(blockIdx.x) * n_tiles_all) / gridDim.x);
    const int tile1 = static_cast<int>((static_cast<int64_t>(blockIdx.x + 1) * n_tiles_all) / gridDim.x);
    const int n_tiles = tile1 - tile0;
    if (threadIdx.x == 0) {
        for (int s = 0; s < p.n_stages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], kMmWarps);
            rel_cnt[s] = 0;
        }
        fence_mbar_init();
    }
    __syncthreads();
    auto issue = [&](int it) {  // tile tile0 + it into slot it % n_stages
        const int s = it % p.n_stages;
        const int row0 = (tile0 + it) * p.rows_per_slot;
        const int rows = min(p.rows_per_slot, p.n_out - row0);
        const uint32_t bytes = static_cast<uint32_t>(rows * p.row_bytes);
        mbar_arrive_expect_tx(&full_bar[s], bytes);
        bulk_g2s(smem + s * p.slot_bytes, p.w + static_cast<int64_t>(row0) * p.row_bytes, bytes, &full_bar[s]);
    };
    // the weights are constants of the model: stream them before the dependency wait
    if (threadIdx.x == 0)
        for (int it = 0; it < n_tiles && it < p.n_stages; ++it) issue(it);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" :::);

    // tokens -> xs (padded sub-blocks) and their sub-block sums: a warp takes 32
    // consecutive values (one sub-block) per step, coalesced, with the loads of
    // kXBatch steps in flight together, and sums each sub-block by shuffles
    constexpr int kXBatch = 8;
    const int n_x = NT * p.n_in;  // a multiple of 256: every step is warp-uniform
    for (int base0 = warp * 32; base0 < n_x; base0 += kMmThreads * kXBatch) {
        float v[kXBatch];
#pragma unroll
        for (int b = 0; b < kXBatch; ++b) {
            const int idx = base0 + b * kMmThreads + lane;
            const int t = idx / p.n_in, i = idx - t * p.n_in;
            v[b] = idx < n_x && t < p.n_tok ? load_act(p.x, static_cast<int64_t>(t) * p.x_stride + i, p.x_dtype) : 0.f;
        }
#pragma unroll
        for (int b = 0; b < kXBatch; ++b) {
            const int idx = base0 + b * kMmThreads + lane;
            if (base0 + b * kMmThreads < n_x) {
                const int t = idx / p.n_in, i = idx - t * p.n_in;
                xs[(t * n_sub + (i >> 5)) * kSubPad + (i & 31)] = v[b];
                float sum = v[b];
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
                if (lane == 0) xsum[t * n_sub + (i >> 5)] = sum;
            }
        }
    }
    __syncthreads();

    const int n_units = p.n_in / 256;
    const int j = lane & 7;
    bool ok = true;
    for (int it = 0; it < n_tiles; ++it) {
        const int s = it % p.n_stages;
        if (!mbar_wait(&full_bar[s], (it / p.n_stages) & 1)) ok = false;
        if (__any_sync(0xffffffffu, !ok)) break;
        const int row = (tile0 + it) * p.rows_per_slot + warp;
        if (warp < p.rows_per_slot && row < p.n_out) {
            const uint8_t *wr = smem + s * p.slot_bytes + warp * p.row_bytes;
            float acc[NT];
#pragma unroll
            for (int t = 0; t < NT; ++t) acc[t] = 0.f;
            for (int un = lane >> 3; un < n_units; un += 4) {
                float v[32], mterm;
                dequant_sub<WT>(wr + un * unit_bytes(WT), j, v, mterm);
                const int sb = 8 * un + j;
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    const float4 *xv = reinterpret_cast<const float4 *>(xs + (t * n_sub + sb) * kSubPad);
                    float a = 0.f;
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const float4 x = xv[q];
                        a = fmaf(v[4 * q], x.x, a);
                        a = fmaf(v[4 * q + 1], x.y, a);
                        a = fmaf(v[4 * q + 2], x.z, a);
                        a = fmaf(v[4 * q + 3], x.w, a);
                    }
                    if constexpr (WT == SQMIX_Q4_K) a = fmaf(-mterm, xsum[t * n_sub + sb], a);
                    acc[t] += a;
                }
            }
#pragma unroll
            for (int t = 0; t < NT; ++t)
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], off);
            if (lane == 0)
#pragma unroll
                for (int t = 0; t < NT; ++t)
                    if (t < p.n_tok) p.y[static_cast<int64_t>(t) * p.y_stride + row] = acc[t];
        }
        // release the slot; the warp that releases it last refills it
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(&empty_bar[s]);
            if (atomicAdd(&rel_cnt[s], 1) == kMmWarps - 1) {
                rel_cnt[s] = 0;
                if (it + p.n_stages < n_tiles) {
                    // every warp has arrived: this wait returns at once
                    if (mbar_wait(&empty_bar[s], (it / p.n_stages) & 1))
                        issue(it + p.n_stages);
                    else
                        ok = false;
                }
            }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    if (__syncthreads_or(!ok)) {
        if (threadIdx.x == 0 && p.status) atomicOr(p.status, 1u);
        // never leave with a bulk copy still writing into shared memory: wait (bounded)
        // for the copies of the last slots
        if (threadIdx.x == 0) {
            const int first = n_tiles > p.n_stages ? n_tiles - p.n_stages : 0;
            for (int it = first; it < n_tiles; ++it)
                if (!mbar_wait(&full_bar[it % p.n_stages], (it / p.n_stages) & 1)) break;
        }
    }
}

template <int WT, int NT>
int launch_mm(const MmParams &p, int grid, size_t smem, cudaStream_t st) {
    auto kernel = mul_mat_kernel<WT, NT>;
    static std::atomic<uint64_t> attr_devices{0};
    {
        const cudaError_t e = set_smem_once(attr_devices, kernel, 227 * 1024);
        if (e != cudaSuccess) return cuda_status(e, "mul_mat smem attribute");
    }
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kMmThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_status(cudaLaunchKernelEx(&cfg, kernel, p), "mul_mat launch");
}

template <int NT>
int launch_mm_type(const MmParams &p, int grid, size_t smem, cudaStream_t st) {
    switch (p.w_type) {
        case SQMIX_Q4_K: return launch_mm<SQMIX_Q4_K, NT>(p, grid, smem, st);
        case SQMIX_Q6_K: return launch_mm<SQMIX_Q6_K, NT>(p, grid, smem, st);
        case SQMIX_Q8_0: return launch_mm<SQMIX_Q8_0, NT>(p, grid, smem, st);
        case SQMIX_F32: return launch_mm<SQMIX_F32, NT>(p, grid, smem, st);
        case SQMIX_F16: return launch_mm<SQMIX_F16, NT>(p, grid, smem, st);
        default: return launch_mm<SQMIX_BF16, NT>(p, grid, smem, st);
    }
}

}  // namespace
}  // namespace sqmix

using namespace sqmix;

extern "C" int64_t sqmix_mul_mat_row_bytes(int32_t w_type, int64_t n_in) {
    const int ub = unit_bytes(w_type);
    if (ub == 0 || n_in <= 0 || n_in % 256 != 0) return 0;
    return n_in / 256 * ub;
}

extern "C" int sqmix_mul_mat(const sqmix_mul_mat_args *a, sqmix_stream_t stream) {
    SQMIX_CHECK_ARG(a != nullptr, "mul_mat: null args");
    SQMIX_CHECK_ARG(a->w && a->x && a->y, "mul_mat: null pointer argument");
    SQMIX_CHECK_ARG(unit_bytes(a->w_type) != 0, "mul_mat: weight type %d (q8_0, q4_K, q6_K, f32, f16, bf16)",
                    a->w_type);
    SQMIX_CHECK_ARG(a->n_in >= 256 && a->n_in <= kMaxIn && a->n_in % 256 == 0,
                    "mul_mat: n_in=%lld must be a multiple of 256 in [256, %d]", (long long)a->n_in, kMaxIn);
    SQMIX_CHECK_ARG(a->n_out >= 1 && a->n_out <= (1 << 24), "mul_mat: n_out=%lld", (long long)a->n_out);
    SQMIX_CHECK_ARG(a->n_tokens >= 1, "mul_mat: n_tokens=%d", a->n_tokens);
    SQMIX_CHECK_ARG(a->x_dtype == SQMIX_F32 || a->x_dtype == SQMIX_F16 || a->x_dtype == SQMIX_BF16,
                    "mul_mat: x dtype %d", a->x_dtype);
    const int64_t rb = sqmix_mul_mat_row_bytes(a->w_type, a->n_in);
    SQMIX_CHECK_ARG(a->w_row_bytes == rb, "mul_mat: w_row_bytes=%lld, rows must be contiguous (%lld bytes)",
                    (long long)a->w_row_bytes, (long long)rb);
    // rows reach shared memory by 1-D bulk copies: 16-byte multiples (q6_K: n_in % 2048 == 0)
    SQMIX_CHECK_ARG(rb % 16 == 0, "mul_mat: a row of %lld bytes is not a multiple of 16 (q6_K needs n_in %% 2048 == 0)",
                    (long long)rb);
    SQMIX_CHECK_ARG((reinterpret_cast<uintptr_t>(a->w) & 15) == 0, "mul_mat: w must be 16-byte aligned");
    SQMIX_CHECK_ARG(a->x_stride >= a->n_in && a->y_stride >= a->n_out, "mul_mat: token strides too small");
    MmParams p;
    p.w = static_cast<const uint8_t *>(a->w);
    p.w_type = a->w_type;
    p.row_bytes = rb;
    p.n_in = static_cast<int>(a->n_in);
    p.n_out = static_cast<int>(a->n_out);
    p.x_dtype = a->x_dtype;
    p.x_stride = a->x_stride;
    p.y_stride = a->y_stride;
    p.status = a->status;
    p.rows_per_slot = static_cast<int>(std::min<int64_t>(kMmWarps, std::max<int64_t>(1, kSlotMax / rb)));
    p.slot_bytes = static_cast<int>((p.rows_per_slot * rb + 127) / 128 * 128);
    p.n_stages = std::max(2, std::min(kMaxStages, kRingBudget / p.slot_bytes));
    const int n_tiles = (p.n_out + p.rows_per_slot - 1) / p.rows_per_slot;
    const int grid = std::min(n_tiles, sqmix_device_sm_count(-1));
    if (grid <= 0) return cuda_status(cudaErrorInvalidDevice, "mul_mat device");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int elt = a->x_dtype == SQMIX_F32 ? 4 : 2;
    for (int t0 = 0; t0 < a->n_tokens; t0 += kMaxPassTokens) {
        const int nt = std::min(kMaxPassTokens, a->n_tokens - t0);
        p.x = static_cast<const uint8_t *>(a->x) + static_cast<int64_t>(t0) * a->x_stride * elt;
        p.y = a->y + static_cast<int64_t>(t0) * a->y_stride;
        p.n_tok = nt;
        const int NT = nt <= 1 ? 1 : nt <= 2 ? 2 : 4;
        const size_t smem = static_cast<size_t>(p.n_stages) * p.slot_bytes +
                            static_cast<size_t>(NT) * (p.n_in / 32) * (kSubPad + 1) * sizeof(float) +
                            2 * kMaxStages * sizeof(uint64_t) + kMaxStages * sizeof(int) + 16;
        int rc;
        if (NT == 1)
            rc = launch_mm_type<1>(p, grid, smem, st);
        else if (NT == 2)
            rc = launch_mm_type<2>(p, grid, smem, st);
        else
            rc = launch_mm_type<4>(p, grid, smem, st);
        if (rc != SQMIX_OK) return rc;
    }
    return SQMIX_OK;
}
