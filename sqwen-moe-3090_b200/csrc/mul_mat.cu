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
    int sstride;  // bytes between rows in a slot (tensor-core path: padded against bank conflicts)
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

// ---- quantised weights on the tensor cores ---------------------------------------
// The quantised formats go through mma.m16n8k16 (f16 operands, f32 accumulators): a
// tile is 16 weight rows (the M of the MMA); the 8 warps split the 256-value units of
// the contraction (warp w: units w, w + 8, ...), each warp moving on to the next tile
// as soon as it is done (a slot is refilled by the warp that releases it last), and the
// partial sums of a group of kTcGroup tiles are reduced through shared memory in a
// fixed order.  The A operand holds exact small integers read straight from the
// GGUF bytes: q4_K nibbles and q6_K 6-bit values masked into f16 words as subnormals
// (value q * 2^-24; high q4_K nibbles carry an extra x16), q8_0 bytes through
// 0x6400 | (q + 128) - 1152.  The K order inside a 16-value slice follows the bytes:
// lane c's 32-bit word holds values 4c .. 4c + 3, k-pairs (2c, 2c + 1) = values (4c,
// 4c + 2) and (2c + 8, 2c + 9) = (4c + 1, 4c + 3); the B operand (x) uses the same
// order.  x is split as x = hi + lo in f16, two MMAs per product, so every product and
// sum is exact to f32 rounding (|x| < 65504).  Each (row, scale block) result is scaled
// in f32: q4_K by d sc 2^24 (2^20 for high nibbles) per 32 values, minus dmin m sum(x);
// q6_K by d sc 2^24 per 16 values, minus 32 d sc sum(x); q8_0 by d per 32 values.  The
// 4 lanes of a row group compute a quarter of a unit's scales each and pass them round
// by shuffles.
constexpr int kTcRows = 16;

__device__ __forceinline__ uint32_t nib_lo(uint32_t w) { return w & 0x000F000Fu; }
__device__ __forceinline__ uint32_t nib_hi(uint32_t w) { return w & 0x00F000F0u; }
// 32-bit word at a 2-byte aligned shared-memory address
__device__ __forceinline__ uint32_t ld_u32_2a(const uint8_t *p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    if ((a & 3) == 0) return *reinterpret_cast<const uint32_t *>(p);
    const uint32_t *q = reinterpret_cast<const uint32_t *>(p - 2);
    return __byte_perm(q[0], q[1], 0x5432);
}
// int8 bytes (b0, b2) / (b1, b3) of w as exact f16 pairs
__device__ __forceinline__ uint32_t i8_pair(uint32_t wx, uint32_t sel) {
    const __half2 h = u32_as_h2(__byte_perm(wx, 0x64646464u, sel));
    return h2_as_u32(__hsub2(h, __float2half2_rn(1152.0f)));
}

constexpr int kTcGroup = 4;  // tiles whose partial sums are reduced together

template <int WT, int NT>
__global__ void __launch_bounds__(kMmThreads, 2) mul_mat_tc_kernel(MmParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int ring_bytes = p.n_stages * p.slot_bytes;
    const int n_units = p.n_in / 256;
    const int n_sl = p.n_in / 16;                                       // 16-value slices
    uint4 *bfrag = reinterpret_cast<uint4 *>(smem + ring_bytes);        // [n_sl][NT][4 lanes c]
    float *xs16 = reinterpret_cast<float *>(bfrag + n_sl * NT * 4);     // [NT][n_sl] slice sums
    float4 *red = reinterpret_cast<float4 *>(xs16 + NT * n_sl);         // [kTcGroup][8 warps][32 lanes]
    uint64_t *full_bar = reinterpret_cast<uint64_t *>(red + kTcGroup * kMmWarps * 32);
    uint64_t *empty_bar = full_bar + kMaxStages;
    int *rel_cnt = reinterpret_cast<int *>(empty_bar + kMaxStages);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, c = lane & 3;

    const int n_tiles_all = (p.n_out + kTcRows - 1) / kTcRows;
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
    // one bulk copy per row: rows land sstride bytes apart, sstride / 4 = 4 mod 8, so the
    // 8 row groups g of a fragment load hit 8 different groups of 4 banks
    auto issue = [&](int it) {
        const int s = it % p.n_stages;
        const int row0 = (tile0 + it) * kTcRows;
        const int rows = min(kTcRows, p.n_out - row0);
        mbar_arrive_expect_tx(&full_bar[s], static_cast<uint32_t>(rows * p.row_bytes));
        for (int r = 0; r < rows; ++r)
            bulk_g2s(smem + s * p.slot_bytes + r * p.sstride, p.w + static_cast<int64_t>(row0 + r) * p.row_bytes,
                     static_cast<uint32_t>(p.row_bytes), &full_bar[s]);
    };
    // the weights are constants of the model: stream them before the dependency wait
    if (threadIdx.x == 0)
        for (int it = 0; it < n_tiles && it < p.n_stages; ++it) issue(it);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" :::);

    // x -> B fragments (f16 hi / lo pairs in the K order above) and 16-value slice sums;
    // entry idx = (slice, token, lane c) covers x values 16 slice + 4 c .. + 3, the loads
    // of kXBatch strides in flight together (the entry count is a multiple of 64, so a
    // warp's 32 entries are all in range or all out)
    constexpr int kXBatch = 4;
    const int n_ent = n_sl * NT * 4;
    for (int base = threadIdx.x; base < n_ent; base += kMmThreads * kXBatch) {
        float v[kXBatch][4];
#pragma unroll
        for (int bb = 0; bb < kXBatch; ++bb) {
            const int idx = base + bb * kMmThreads;
            const int t = (idx >> 2) % NT, sl = (idx >> 2) / NT, cc = idx & 3;
#pragma unroll
            for (int e = 0; e < 4; ++e)
                v[bb][e] = idx < n_ent && t < p.n_tok
                               ? load_act(p.x, static_cast<int64_t>(t) * p.x_stride + 16 * sl + 4 * cc + e, p.x_dtype)
                               : 0.f;
        }
#pragma unroll
        for (int bb = 0; bb < kXBatch; ++bb) {
            const int idx = base + bb * kMmThreads;
            if ((idx & ~31) < n_ent) {  // the warp's first entry: warps are wholly in or out
                const int t = (idx >> 2) % NT, sl = (idx >> 2) / NT, cc = idx & 3;
                __half hv[4], lv[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    hv[e] = __float2half_rn(v[bb][e]);
                    lv[e] = __float2half_rn(v[bb][e] - __half2float(hv[e]));
                }
                bfrag[idx] = make_uint4(h2_as_u32(__halves2half2(hv[0], hv[2])), h2_as_u32(__halves2half2(hv[1], hv[3])),
                                        h2_as_u32(__halves2half2(lv[0], lv[2])), h2_as_u32(__halves2half2(lv[1], lv[3])));
                float sum = (v[bb][0] + v[bb][1]) + (v[bb][2] + v[bb][3]);  // lanes c of a slice are consecutive
                sum += __shfl_xor_sync(0xffffffffu, sum, 1);
                sum += __shfl_xor_sync(0xffffffffu, sum, 2);
                if (cc == 0) xs16[t * n_sl + sl] = sum;
            }
        }
    }
    __syncthreads();

    // this lane's B fragment of slice sl (zero for token columns g >= NT)
    auto bload = [&](int sl, uint32_t (&bh)[2], uint32_t (&bl)[2]) {
        if (g < NT) {
            const uint4 b = bfrag[(sl * NT + g) * 4 + c];
            bh[0] = b.x;
            bh[1] = b.y;
            bl[0] = b.z;
            bl[1] = b.w;
        } else {
            bh[0] = bh[1] = bl[0] = bl[1] = 0u;
        }
    };
    // sum of x over slices [sl0, sl0 + n) for the token columns 2c, 2c + 1
    auto xsum2 = [&](int sl0, int n, float &s0, float &s1) {
        s0 = s1 = 0.f;
        for (int i = 0; i < n; ++i) {
            if (2 * c < NT) s0 += xs16[(2 * c) * n_sl + sl0 + i];
            if (2 * c + 1 < NT) s1 += xs16[(2 * c + 1) * n_sl + sl0 + i];
        }
    };

    bool ok = true;
    for (int gb = 0; gb < n_tiles && ok; gb += kTcGroup) {
        const int ge = min(n_tiles, gb + kTcGroup);
        for (int it = gb; it < ge; ++it) {
            const int s = it % p.n_stages;
            if (!mbar_wait(&full_bar[s], (it / p.n_stages) & 1)) ok = false;
            if (__any_sync(0xffffffffu, !ok)) {
                ok = false;
                break;
            }
            const uint8_t *rg = smem + s * p.slot_bytes + g * p.sstride;
            const uint8_t *rg8 = rg + 8 * p.sstride;
            float y[4] = {0.f, 0.f, 0.f, 0.f};
            for (int u = warp; u < n_units; u += kMmWarps) {
                if constexpr (WT == SQMIX_Q4_K) {
                    // lane c: (d sc 2^24 or 2^20, dmin m) of sub-blocks 2c, 2c + 1 of rows g, g + 8
                    float2 fs[2][2];
#pragma unroll
                    for (int rr = 0; rr < 2; ++rr) {
                        const uint8_t *b = (rr ? rg8 : rg) + u * 144;
                        const float d = f16_at(b), dmin = f16_at(b + 2);
                        const uint8_t *sb = b + 4;
#pragma unroll
                        for (int q = 0; q < 2; ++q) {
                            const int j = 2 * c + q;
                            int sc, m;
                            if (j < 4) {
                                sc = sb[j] & 63;
                                m = sb[j + 4] & 63;
                            } else {
                                sc = (sb[j + 4] & 0xF) | ((sb[j - 4] >> 6) << 4);
                                m = (sb[j + 4] >> 4) | ((sb[j] >> 6) << 4);
                            }
                            fs[rr][q] = make_float2(d * static_cast<float>(sc) * (q ? 1048576.0f : 16777216.0f),
                                                    dmin * static_cast<float>(m));
                        }
                    }
#pragma unroll
                    for (int k = 0; k < 4; ++k) {  // 32 bytes: sub-blocks 2k (low nibbles), 2k + 1 (high)
                        float a0[4] = {0.f, 0.f, 0.f, 0.f}, a1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const int off = u * 144 + 16 + 32 * k + 16 * h + 4 * c;
                            const uint32_t w0 = *reinterpret_cast<const uint32_t *>(rg + off);
                            const uint32_t w1 = *reinterpret_cast<const uint32_t *>(rg8 + off);
                            const uint32_t alo[4] = {nib_lo(w0), nib_lo(w1), nib_lo(w0 >> 8), nib_lo(w1 >> 8)};
                            const uint32_t ahi[4] = {nib_hi(w0), nib_hi(w1), nib_hi(w0 >> 8), nib_hi(w1 >> 8)};
                            uint32_t bh[2], bl[2];
                            bload(2 * (8 * u + 2 * k) + h, bh, bl);
                            mma_f16_16816(a0, alo, bh[0], bh[1], a0);
                            mma_f16_16816(a0, alo, bl[0], bl[1], a0);
                            bload(2 * (8 * u + 2 * k + 1) + h, bh, bl);
                            mma_f16_16816(a1, ahi, bh[0], bh[1], a1);
                            mma_f16_16816(a1, ahi, bl[0], bl[1], a1);
                        }
#pragma unroll
                        for (int sbk = 0; sbk < 2; ++sbk) {  // sub-block 2k + sbk: lane 4 g' + k holds it
                            const int sub = 8 * u + 2 * k + sbk;
                            const float *a = sbk ? a1 : a0;
                            const int src = 4 * g + k;
                            const float f0x = __shfl_sync(0xffffffffu, fs[0][sbk].x, src);
                            const float f0y = __shfl_sync(0xffffffffu, fs[0][sbk].y, src);
                            const float f1x = __shfl_sync(0xffffffffu, fs[1][sbk].x, src);
                            const float f1y = __shfl_sync(0xffffffffu, fs[1][sbk].y, src);
                            float x0, x1;
                            xsum2(2 * sub, 2, x0, x1);
                            y[0] = fmaf(f0x, a[0], fmaf(-f0y, x0, y[0]));
                            y[1] = fmaf(f0x, a[1], fmaf(-f0y, x1, y[1]));
                            y[2] = fmaf(f1x, a[2], fmaf(-f1y, x0, y[2]));
                            y[3] = fmaf(f1x, a[3], fmaf(-f1y, x1, y[3]));
                        }
                    }
                } else if constexpr (WT == SQMIX_Q6_K) {
                    // lane c: d sc of slices 4c .. 4c + 3 of rows g, g + 8
                    float ds[2][4];
#pragma unroll
                    for (int rr = 0; rr < 2; ++rr) {
                        const uint8_t *b = (rr ? rg8 : rg) + u * 210;
                        const float d = f16_at(b + 208);
#pragma unroll
                        for (int q = 0; q < 4; ++q) ds[rr][q] = d * static_cast<float>(static_cast<int8_t>(b[192 + 4 * c + q]));
                    }
#pragma unroll 4
                    for (int q = 0; q < 16; ++q) {  // 16-value slice q of the unit: one scale
                        const int hh = q >> 3, k = (q >> 1) & 3, h = q & 1;
                        const int offl = u * 210 + 64 * hh + 32 * (k & 1) + 16 * h + 4 * c;
                        const int offh = u * 210 + 128 + 32 * hh + 16 * h + 4 * c;
                        const uint32_t l0 = ld_u32_2a(rg + offl) >> (4 * (k >> 1));
                        const uint32_t l1 = ld_u32_2a(rg8 + offl) >> (4 * (k >> 1));
                        const uint32_t h0 = ld_u32_2a(rg + offh) >> (2 * k), h1 = ld_u32_2a(rg8 + offh) >> (2 * k);
                        const uint32_t av[4] = {(l0 & 0x000F000Fu) | ((h0 & 0x00030003u) << 4),
                                                (l1 & 0x000F000Fu) | ((h1 & 0x00030003u) << 4),
                                                ((l0 >> 8) & 0x000F000Fu) | (((h0 >> 8) & 0x00030003u) << 4),
                                                ((l1 >> 8) & 0x000F000Fu) | (((h1 >> 8) & 0x00030003u) << 4)};
                        float a[4] = {0.f, 0.f, 0.f, 0.f};
                        uint32_t bh[2], bl[2];
                        bload(16 * u + q, bh, bl);
                        mma_f16_16816(a, av, bh[0], bh[1], a);
                        mma_f16_16816(a, av, bl[0], bl[1], a);
                        const int src = 4 * g + (q >> 2);
                        const float d0 = __shfl_sync(0xffffffffu, ds[0][q & 3], src);
                        const float d1 = __shfl_sync(0xffffffffu, ds[1][q & 3], src);
                        float x0, x1;
                        xsum2(16 * u + q, 1, x0, x1);
                        y[0] = fmaf(d0 * 16777216.0f, a[0], fmaf(-32.0f * d0, x0, y[0]));
                        y[1] = fmaf(d0 * 16777216.0f, a[1], fmaf(-32.0f * d0, x1, y[1]));
                        y[2] = fmaf(d1 * 16777216.0f, a[2], fmaf(-32.0f * d1, x0, y[2]));
                        y[3] = fmaf(d1 * 16777216.0f, a[3], fmaf(-32.0f * d1, x1, y[3]));
                    }
                } else {  // q8_0
                    // lane c: d of blocks 2c, 2c + 1 of rows g, g + 8
                    float dd[2][2];
#pragma unroll
                    for (int rr = 0; rr < 2; ++rr)
#pragma unroll
                        for (int q = 0; q < 2; ++q) dd[rr][q] = f16_at((rr ? rg8 : rg) + u * 272 + 34 * (2 * c + q));
#pragma unroll 2
                    for (int j = 0; j < 8; ++j) {  // block j of the unit: 32 values, one d
                        float a[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const int off = u * 272 + 34 * j + 2 + 16 * h + 4 * c;
                            const uint32_t w0 = ld_u32_2a(rg + off) ^ 0x80808080u;
                            const uint32_t w1 = ld_u32_2a(rg8 + off) ^ 0x80808080u;
                            const uint32_t av[4] = {i8_pair(w0, 0x4240u), i8_pair(w1, 0x4240u), i8_pair(w0, 0x4341u),
                                                    i8_pair(w1, 0x4341u)};
                            uint32_t bh[2], bl[2];
                            bload(2 * (8 * u + j) + h, bh, bl);
                            mma_f16_16816(a, av, bh[0], bh[1], a);
                            mma_f16_16816(a, av, bl[0], bl[1], a);
                        }
                        const int src = 4 * g + (j >> 1);
                        const float d0 = __shfl_sync(0xffffffffu, dd[0][j & 1], src);
                        const float d1 = __shfl_sync(0xffffffffu, dd[1][j & 1], src);
                        y[0] = fmaf(d0, a[0], y[0]);
                        y[1] = fmaf(d0, a[1], y[1]);
                        y[2] = fmaf(d1, a[2], y[2]);
                        y[3] = fmaf(d1, a[3], y[3]);
                    }
                }
            }
            red[((it - gb) * kMmWarps + warp) * 32 + lane] = make_float4(y[0], y[1], y[2], y[3]);
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
            ok = false;
            break;
        }
        // the group's outputs (tile, row r, token n): lane 4 (r % 8) + n / 2, register 2 (r / 8) + n % 2
        for (int o = threadIdx.x; o < (ge - gb) * kTcRows * NT; o += kMmThreads) {
            const int tl = o / (kTcRows * NT), rem = o % (kTcRows * NT), r = rem / NT, n = rem % NT;
            const int ln = 4 * (r & 7) + (n >> 1), reg = 2 * (r >> 3) + (n & 1);
            float acc = 0.f;
#pragma unroll
            for (int wv = 0; wv < kMmWarps; ++wv) {
                const float4 q4 = red[(tl * kMmWarps + wv) * 32 + ln];
                acc += reg == 0 ? q4.x : reg == 1 ? q4.y : reg == 2 ? q4.z : q4.w;
            }
            const int row = (tile0 + gb + tl) * kTcRows + r;
            if (row < p.n_out && n < p.n_tok) p.y[static_cast<int64_t>(n) * p.y_stride + row] = acc;
        }
        __syncthreads();  // the partial sums' space is reused by the next group
    }
    if (!ok) {
        if (threadIdx.x == 0 && p.status) atomicOr(p.status, 1u);
        // never leave with a bulk copy still writing into shared memory
        if (threadIdx.x == 0) {
            const int first = n_tiles > p.n_stages ? n_tiles - p.n_stages : 0;
            for (int it = first; it < n_tiles; ++it)
                if (!mbar_wait(&full_bar[it % p.n_stages], (it / p.n_stages) & 1)) break;
        }
    }
}

template <int WT, int NT>
int launch_mm_tc(const MmParams &p, int grid, size_t smem, cudaStream_t st) {
    auto kernel = mul_mat_tc_kernel<WT, NT>;
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
int launch_mm_tc_type(const MmParams &p, int grid, size_t smem, cudaStream_t st) {
    switch (p.w_type) {
        case SQMIX_Q4_K: return launch_mm_tc<SQMIX_Q4_K, NT>(p, grid, smem, st);
        case SQMIX_Q6_K: return launch_mm_tc<SQMIX_Q6_K, NT>(p, grid, smem, st);
        default: return launch_mm_tc<SQMIX_Q8_0, NT>(p, grid, smem, st);
    }
}

template <int NT>
int launch_mm_type(const MmParams &p, int grid, size_t smem, cudaStream_t st) {
    switch (p.w_type) {
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
    const bool tc = a->w_type == SQMIX_Q4_K || a->w_type == SQMIX_Q6_K || a->w_type == SQMIX_Q8_0;
    p.rows_per_slot = tc ? kTcRows : static_cast<int>(std::min<int64_t>(kMmWarps, std::max<int64_t>(1, kSlotMax / rb)));
    p.sstride = static_cast<int>(tc && (rb / 4) % 8 == 0 ? rb + 16 : rb);
    p.slot_bytes = static_cast<int>((p.rows_per_slot * static_cast<int64_t>(p.sstride) + 127) / 128 * 128);
    p.n_stages = std::max(2, std::min(kMaxStages, kRingBudget / p.slot_bytes));
    const int n_tiles = (p.n_out + p.rows_per_slot - 1) / p.rows_per_slot;
    const int grid = std::min(n_tiles, sqmix_device_sm_count(-1));
    if (grid <= 0) return cuda_status(cudaErrorInvalidDevice, "mul_mat device");
    constexpr size_t kSmemMax = 227 * 1024;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int elt = a->x_dtype == SQMIX_F32 ? 4 : 2;
    for (int t0 = 0; t0 < a->n_tokens; t0 += kMaxPassTokens) {
        const int nt = std::min(kMaxPassTokens, a->n_tokens - t0);
        p.x = static_cast<const uint8_t *>(a->x) + static_cast<int64_t>(t0) * a->x_stride * elt;
        p.y = a->y + static_cast<int64_t>(t0) * a->y_stride;
        p.n_tok = nt;
        const int NT = nt <= 1 ? 1 : nt <= 2 ? 2 : 4;
        int rc;
        if (tc) {
            // B fragments, slice sums, the cross-warp partial sums of a group of tiles
            const size_t extra = static_cast<size_t>(p.n_in) * NT * 4 + static_cast<size_t>(NT) * (p.n_in / 16) * 4 +
                                 static_cast<size_t>(kTcGroup) * kMmWarps * 32 * 16 +
                                 2 * kMaxStages * sizeof(uint64_t) + kMaxStages * sizeof(int) + 16;
            // two CTAs per SM when the ring of at least 2 slots allows (more warps to hide
            // the latency of the dequant / MMA chains), else one
            MmParams q = p;
            constexpr size_t kSmemHalf = 113 * 1024 - 1024;
            const size_t budget = extra + 2 * static_cast<size_t>(q.slot_bytes) <= kSmemHalf ? kSmemHalf : kSmemMax;
            q.n_stages = static_cast<int>(std::min<size_t>(q.n_stages, (budget - extra) / q.slot_bytes));
            if (q.n_stages < 2) return cuda_status(cudaErrorInvalidValue, "mul_mat shared memory");
            const size_t smem = static_cast<size_t>(q.n_stages) * q.slot_bytes + extra;
            const int grid_tc = std::min(n_tiles, (budget == kSmemHalf ? 2 : 1) * sqmix_device_sm_count(-1));
            if (NT == 1)
                rc = launch_mm_tc_type<1>(q, grid_tc, smem, st);
            else if (NT == 2)
                rc = launch_mm_tc_type<2>(q, grid_tc, smem, st);
            else
                rc = launch_mm_tc_type<4>(q, grid_tc, smem, st);
        } else {
            const size_t smem = static_cast<size_t>(p.n_stages) * p.slot_bytes +
                                static_cast<size_t>(NT) * (p.n_in / 32) * (kSubPad + 1) * sizeof(float) +
                                2 * kMaxStages * sizeof(uint64_t) + kMaxStages * sizeof(int) + 16;
            if (NT == 1)
                rc = launch_mm_type<1>(p, grid, smem, st);
            else if (NT == 2)
                rc = launch_mm_type<2>(p, grid, smem, st);
            else
                rc = launch_mm_type<4>(p, grid, smem, st);
        }
        if (rc != SQMIX_OK) return rc;
    }
    return SQMIX_OK;
}
