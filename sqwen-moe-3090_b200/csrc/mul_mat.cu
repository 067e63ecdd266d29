// mul_mat.cu -- the mixer projections at decode: ggml_mul_mat(w, x) as sqwen builds
// them (QG / K / V, src/model/attn.rs:127-129; W_o, attn.rs:285; qkv / z / beta / alpha,
// src/model/gdn.rs:264-276; out, gdn.rs:577):
//     y[t][o] = sum_i W[o][i] x[t][i],   o < n_out, i < n_in, t < n_tokens,
// W being ggml's [n_in, n_out] tensor (n_out contiguous rows of n_in values) in a GGUF
// block format: q8_0, q4_K, q6_K (the types of a Q4_K_M model's projection weights), or
// f32 / f16 / bf16.  Dequantised weights times x are summed in f32.  (ggml's CUDA
// backend quantises x to q8_1 for its quantised dot products; this path does not.)
//
// At decode a projection is a stream of its weight bytes.  A launch serves a group of
// projections of the same x (a layer's QG / K / V, or qkv / z / beta / alpha): their
// row tiles form one list, and each CTA walks a contiguous range of it, so the fixed
// cost of a launch (the wait on the kernel before, staging x) is paid once per group.
// Tiles reach shared memory by bulk copies (TMA, no multicast) on an mbarrier ring that
// is filled before the grid-dependency wait: the weights are model constants, only x
// comes from the kernel before.  Quantised tiles go through the tensor cores, f32 / f16
// / bf16 tiles through FMAs, in the same kernel.  A pass serves up to kMaxPassTokens
// tokens per stream of W.
#include <math.h>

#include "common.cuh"
#include "sqmix.h"

namespace sqmix {
// the prefill form (mul_mat_gemm.cu) for a validated group; its 128 x 128 output tiles
// (0: x not usable by the form)
int mul_mat_gemm_launch(const sqmix_mul_mat_args *args, int n, cudaStream_t st);
int mul_mat_gemm_tiles(const sqmix_mul_mat_args *args, int n);

namespace {

// A CTA has W = 8 warps (two CTAs per SM) or, for 16 or more units per row, W = 16 (one
// CTA per SM, one unit per warp); either way at most 128 registers a thread.
constexpr int kMmRegThreads = 512;    // threads per SM the registers are budgeted for
constexpr int kMaxIn = 4096;          // n_in limit (the model's 2048 and 4096)
constexpr int kMaxPassTokens = 4;     // tokens per stream of W
// The tensor-core GEMM form (mul_mat_gemm.cu) takes n_tokens >= kGemmTokens, >= 48 when
// its tiles fill at least 48 CTAs, >= 16 when at least 96 (measured crossovers against
// ceil(n_tokens / 4) passes of the decode form: the GEMM's time hardly depends on the
// batch below 128 tokens, the decode form's grows with every 4)
constexpr int kGemmTokens = 128;
constexpr int kGemmMinTokens = 16;
__host__ constexpr int gemm_min_tiles(int n_tokens) { return n_tokens >= 48 ? 48 : 96; }
constexpr int kMaxStages = 8;
constexpr int kFloatSlot = 16 * 1024; // slot bytes of a launch of float-typed weights only
constexpr int kMaxSeg = SQMIX_MUL_MAT_MAX_GROUP;

// one projection of a launch
struct MmSeg {
    const uint8_t *w;
    float *y;          // this pass's first token
    int64_t y_stride;
    int w_type;
    int row_bytes;
    int sstride;       // quantised: bytes between row pairs in a slot; float: between rows
    int rows;          // rows per tile: 16 for the quantised formats
    int n_out;
    int tile0;         // first tile of the projection in the launch's tile list
};

struct MmParams {
    MmSeg seg[kMaxSeg];
    int n_seg, n_tiles;
    int n_in;
    const void *x;
    int x_dtype;
    int64_t x_stride;
    int n_tok;         // tokens of this pass (<= NT)
    int has_float;     // x is also staged in f32 for float-typed rows
    uint32_t *status;
    int n_stages, slot_bytes;
};

// the projection that tile t of the launch belongs to
__device__ __forceinline__ int seg_of(const MmParams &p, int t) {
    int s = 0;
    while (s + 1 < p.n_seg && t >= p.seg[s + 1].tile0) ++s;
    return s;
}

__device__ __forceinline__ float f16_at(const uint8_t *p) {
    return __half2float(*reinterpret_cast<const __half *>(p));
}

// The block formats that go through the tensor cores.
__host__ __device__ constexpr bool quant_type(int t) { return t == SQMIX_Q4_K || t == SQMIX_Q6_K || t == SQMIX_Q8_0; }

// Unit (256 values) bytes per format; 0: unsupported.
__host__ __device__ constexpr int unit_bytes(int t) {
    return t == SQMIX_Q4_K ? 144 : t == SQMIX_Q6_K ? 210 : t == SQMIX_Q8_0 ? 272 : t == SQMIX_F32 ? 1024
           : (t == SQMIX_F16 || t == SQMIX_BF16) ? 512 : 0;
}

// ---- the tiles ---------------------------------------------------------------------
// q8_0 / q4_K / q6_K tiles go through mma.m16n8k16 (f16 operands, f32 accumulators): a
// tile is 16 weight rows of one projection (the M of the MMA), brought in as 8 bulk
// copies of two consecutive rows each, the pairs sstride = 2 row_bytes + 16 bytes apart
// in the slot (sstride / 4 = 4 mod 8).  MMA row g is the pair's first row, MMA row g + 8
// its second: the 8 row groups of a fragment load then hit 8 different groups of 4
// banks.  A float-typed tile holds as many rows as fit the slot, in one copy
// (unit_float).  The 8 warps split the
// 256-value units of the contraction (warp w: units w, w + 8, ...), each warp moving on
// to the next tile as soon as it is done (a slot is refilled by the warp that releases
// it last), and the partial sums of a group of kTcGroup tiles are reduced through
// shared memory in a fixed order.
//
// The A operand holds exact small integers read straight from the GGUF bytes: q4_K
// nibbles and q6_K 6-bit values masked into f16 words as subnormals (value q 2^-24;
// high q4_K nibbles carry an extra x16), q8_0 bytes through 0x6400 | (q + 128) - 1152.
// The K order inside a 16-value slice follows the bytes: lane c's 32-bit word holds
// values 4c .. 4c + 3, k-pairs (2c, 2c + 1) = values (4c, 4c + 2) and (2c + 8, 2c + 9) =
// (4c + 1, 4c + 3); the B operand uses the same order.  x is split as x = hi + lo in
// f16, and the two halves are two columns of B (column 2t: token t's hi, 2t + 1: its
// lo), so one MMA serves 4 tokens and lane c of a row group ends with token c's sum in
// (d0 + d1, d2 + d3) for rows g, g + 8: every product and sum is exact to f32 rounding
// (|x| < 65504).  Each (row, scale block) result is scaled in f32: q4_K by d sc 2^24
// (2^20 for high nibbles) per 32 values, minus dmin m sum(x); q6_K by d sc 2^24 per 16
// values, minus 32 d sc sum(x); q8_0 by d per 32 values.  A warp decodes a unit's scales
// once into its table (the 4 lanes of a row group a quarter each) and reads them back as
// broadcasts.
constexpr int kTcRows = 16;
constexpr int kTcGroup = 4;   // tiles whose partial sums are reduced together
constexpr int kTabStride = 36; // floats per row group g of a warp's scale table (g at 4-bank offsets)

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
// d = A B (+ 0): a pure function of its operands, free for the scheduler to move
__device__ __forceinline__ void mma_f16_zero(float (&d)[4], const uint32_t (&a)[4], uint2 b) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b.x), "r"(b.y), "f"(0.f));
}
// d += A B
__device__ __forceinline__ void mma_f16_acc(float (&d)[4], const uint32_t (&a)[4], uint2 b) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b.x), "r"(b.y));
}
// B fragment of 16-value slice sl for lane (g, c): column g = token g / 2, hi (g even) or
// lo (g odd); columns of absent tokens are zero
template <int NT>
__device__ __forceinline__ uint2 bfrag_at(const uint2 *bf, int sl, int g, int c) {
    return g < 2 * NT ? bf[(sl * 2 * NT + g) * 4 + c] : make_uint2(0u, 0u);
}

// One 256-value unit u of rows g, g + 8 (rg, rg8: the rows in the slot), token c of this
// lane: y0 / y1 += the unit's dot products.  tab: the warp's scale table, [8 row groups g]
// [kTabStride] floats, entry e of row group g holding row g's and row g + 8's scales.
template <int NT>
__device__ __forceinline__ void unit_q4k(const uint8_t *rg, const uint8_t *rg8, int u, int g, int c,
                                         const uint2 *bf, const float *xs32, int xs32_st, float *tab, float &y0,
                                         float &y1) {
    __syncwarp();  // the previous unit's table reads are done
    // lane (g, c) decodes row g + 8 (c / 2), sub-blocks 4 (c % 2) .. + 3: the 12 scale bytes
    // as three words (a unit starts 16-byte aligned in the slot), four 6-bit scales / mins
    // per word; entry j = (d sc 2^24 or 2^20, dmin m) of row g, then of row g + 8
    {
        const int rh = c >> 1;
        const uint8_t *b = (rh ? rg8 : rg) + u * 144;
        const float d = f16_at(b), dmin = f16_at(b + 2);
        const uint32_t s0 = *reinterpret_cast<const uint32_t *>(b + 4);
        const uint32_t s1 = *reinterpret_cast<const uint32_t *>(b + 8);
        const uint32_t s2 = *reinterpret_cast<const uint32_t *>(b + 12);
        const bool upper = c & 1;
        const uint32_t sc4 = upper ? (s2 & 0x0F0F0F0Fu) | ((s0 >> 2) & 0x30303030u) : s0 & 0x3F3F3F3Fu;
        const uint32_t m4 = upper ? ((s2 >> 4) & 0x0F0F0F0Fu) | ((s1 >> 2) & 0x30303030u) : s1 & 0x3F3F3F3Fu;
        const float dl = d * 16777216.0f, dh = d * 1048576.0f;
        float *e = tab + g * kTabStride + 16 * (c & 1) + 2 * rh;
#pragma unroll
        for (int q = 0; q < 4; ++q)
            *reinterpret_cast<float2 *>(e + 4 * q) =
                make_float2((q & 1 ? dh : dl) * static_cast<float>((sc4 >> (8 * q)) & 0xFF),
                            dmin * static_cast<float>((m4 >> (8 * q)) & 0xFF));
    }
    // this lane's token c: the unit's 32-value sums of x
    float xj[8];
    if (c < NT) {
        const float4 *xp = reinterpret_cast<const float4 *>(xs32 + c * xs32_st + 8 * u);
        const float4 x0 = xp[0], x1 = xp[1];
        xj[0] = x0.x, xj[1] = x0.y, xj[2] = x0.z, xj[3] = x0.w, xj[4] = x1.x, xj[5] = x1.y, xj[6] = x1.z, xj[7] = x1.w;
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) xj[j] = 0.f;
    }
    // two halves of the unit: the MMAs of a half do not need the table, so the first
    // half's overlap the table's stores; the __syncwarp before the first epilogue makes
    // the table visible
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        float acc[4][4];  // sub-blocks 4 half + 0 .. 3
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {  // 32 bytes: sub-blocks 2k (low nibbles), 2k + 1 (high)
            const int k = 2 * half + kk;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int off = u * 144 + 16 + 32 * k + 16 * h + 4 * c;
                const uint32_t w0 = *reinterpret_cast<const uint32_t *>(rg + off);
                const uint32_t w1 = *reinterpret_cast<const uint32_t *>(rg8 + off);
                const uint32_t w0s = w0 >> 8, w1s = w1 >> 8;
                const uint32_t alo[4] = {nib_lo(w0), nib_lo(w1), nib_lo(w0s), nib_lo(w1s)};
                const uint32_t ahi[4] = {nib_hi(w0), nib_hi(w1), nib_hi(w0s), nib_hi(w1s)};
                const uint2 bl = bfrag_at<NT>(bf, 2 * (8 * u + 2 * k) + h, g, c);
                const uint2 bh = bfrag_at<NT>(bf, 2 * (8 * u + 2 * k + 1) + h, g, c);
                if (h == 0) {
                    mma_f16_zero(acc[2 * kk], alo, bl);
                    mma_f16_zero(acc[2 * kk + 1], ahi, bh);
                } else {
                    mma_f16_acc(acc[2 * kk], alo, bl);
                    mma_f16_acc(acc[2 * kk + 1], ahi, bh);
                }
            }
        }
        if (half == 0) __syncwarp();
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
            const int j = 4 * half + jj;
            const float4 f = *reinterpret_cast<const float4 *>(tab + g * kTabStride + 4 * j);
            y0 = fmaf(f.x, acc[jj][0] + acc[jj][1], fmaf(-f.y, xj[j], y0));
            y1 = fmaf(f.z, acc[jj][2] + acc[jj][3], fmaf(-f.w, xj[j], y1));
        }
    }
}

template <int NT>
__device__ __forceinline__ void unit_q6k(const uint8_t *rg, const uint8_t *rg8, int u, int g, int c,
                                         const uint2 *bf, const float *xs16, int xs16_st, float *tab, float &y0,
                                         float &y1) {
    __syncwarp();
    // lane c: d sc of slices 4c .. 4c + 3; entry q = (row g, row g + 8)
    {
        const uint8_t *b0 = rg + u * 210, *b1 = rg8 + u * 210;
        const float d0 = f16_at(b0 + 208), d1 = f16_at(b1 + 208);
#pragma unroll
        for (int q = 0; q < 4; ++q)
            *reinterpret_cast<float2 *>(tab + g * kTabStride + 2 * (4 * c + q)) =
                make_float2(d0 * static_cast<float>(static_cast<int8_t>(b0[192 + 4 * c + q])),
                            d1 * static_cast<float>(static_cast<int8_t>(b1[192 + 4 * c + q])));
    }
    __syncwarp();
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
        float a[4];
        mma_f16_zero(a, av, bfrag_at<NT>(bf, 16 * u + q, g, c));
        const float2 dd = *reinterpret_cast<const float2 *>(tab + g * kTabStride + 2 * q);
        const float d0 = dd.x, d1 = dd.y;
        const float xq = c < NT ? xs16[c * xs16_st + 16 * u + q] : 0.f;
        y0 = fmaf(d0 * 16777216.0f, a[0] + a[1], fmaf(-32.0f * d0, xq, y0));
        y1 = fmaf(d1 * 16777216.0f, a[2] + a[3], fmaf(-32.0f * d1, xq, y1));
    }
}

template <int NT>
__device__ __forceinline__ void unit_q8_0(const uint8_t *rg, const uint8_t *rg8, int u, int g, int c,
                                          const uint2 *bf, float *tab, float &y0, float &y1) {
    __syncwarp();
    // lane c: d of blocks 2c, 2c + 1; entry j = (row g, row g + 8)
#pragma unroll
    for (int q = 0; q < 2; ++q)
        *reinterpret_cast<float2 *>(tab + g * kTabStride + 2 * (2 * c + q)) =
            make_float2(f16_at(rg + u * 272 + 34 * (2 * c + q)), f16_at(rg8 + u * 272 + 34 * (2 * c + q)));
    __syncwarp();
#pragma unroll 2
    for (int j = 0; j < 8; ++j) {  // block j of the unit: 32 values, one d
        float a[4];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int off = u * 272 + 34 * j + 2 + 16 * h + 4 * c;
            const uint32_t w0 = ld_u32_2a(rg + off) ^ 0x80808080u;
            const uint32_t w1 = ld_u32_2a(rg8 + off) ^ 0x80808080u;
            const uint32_t av[4] = {i8_pair(w0, 0x4240u), i8_pair(w1, 0x4240u), i8_pair(w0, 0x4341u),
                                    i8_pair(w1, 0x4341u)};
            const uint2 b = bfrag_at<NT>(bf, 2 * (8 * u + j) + h, g, c);
            if (h == 0)
                mma_f16_zero(a, av, b);
            else
                mma_f16_acc(a, av, b);
        }
        const float2 dd = *reinterpret_cast<const float2 *>(tab + g * kTabStride + 2 * j);
        y0 = fmaf(dd.x, a[0] + a[1], y0);
        y1 = fmaf(dd.y, a[2] + a[3], y1);
    }
}

// f32 / f16 / bf16 rows (the 32-row beta / alpha): FMAs in f32.  Lane l takes values
// 256 u + 8 l .. + 7 of each of the tile's rows against x in f32 (xf: [NT][n_in]); each
// (row, token) sum is reduced over the warp by shuffles, and lane (g, c) keeps rows g,
// g + 8 of token c, as the tensor-core units leave them.
template <int NT>
__device__ __forceinline__ void unit_float(const uint8_t *slot, int sstride, int rows, int wt, int u, int lane,
                                           const float *xf, int n_in, int g, int c, float &y0, float &y1) {
    float xv[NT][8];
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        const float4 *xp = reinterpret_cast<const float4 *>(xf + t * n_in + 256 * u + 8 * lane);
        const float4 a = xp[0], b = xp[1];
        xv[t][0] = a.x, xv[t][1] = a.y, xv[t][2] = a.z, xv[t][3] = a.w;
        xv[t][4] = b.x, xv[t][5] = b.y, xv[t][6] = b.z, xv[t][7] = b.w;
    }
    for (int r = 0; r < rows; ++r) {
        float w[8];
        if (wt == SQMIX_F32) {
            const float4 *wp = reinterpret_cast<const float4 *>(slot + r * sstride + u * 1024 + 32 * lane);
            const float4 a = wp[0], b = wp[1];
            w[0] = a.x, w[1] = a.y, w[2] = a.z, w[3] = a.w, w[4] = b.x, w[5] = b.y, w[6] = b.z, w[7] = b.w;
        } else {
            const uint4 h = *reinterpret_cast<const uint4 *>(slot + r * sstride + u * 512 + 16 * lane);
            const uint32_t hw[4] = {h.x, h.y, h.z, h.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 f = wt == SQMIX_BF16 ? __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&hw[e]))
                                                  : __half22float2(*reinterpret_cast<const __half2 *>(&hw[e]));
                w[2 * e] = f.x;
                w[2 * e + 1] = f.y;
            }
        }
        float mine = 0.f;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            float a = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) a = fmaf(w[i], xv[t][i], a);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
            if (t == 0 || c == t) mine = a;
        }
        if (r == g) y0 += mine;
        if (r == g + 8) y1 += mine;
    }
}

// shared memory of mul_mat_tc_kernel after its ring
__host__ __device__ constexpr size_t tc_extra_bytes(int nt, int w, int n_in, bool has_float) {
    return static_cast<size_t>(n_in / 16) * 2 * nt * 4 * 8 +                 // B fragments
           (has_float ? static_cast<size_t>(nt) * n_in * 4 : 0) +             // x in f32
           static_cast<size_t>(nt) * (n_in / 16 + 4) * 4 +                    // 16-value sums
           static_cast<size_t>(nt) * (n_in / 32 + 4) * 4 +                    // 32-value sums
           static_cast<size_t>(w) * 8 * kTabStride * 4 +                      // scale tables
           static_cast<size_t>(kTcGroup) * w * 32 * 8 +                       // partial sums
           2 * kMaxStages * sizeof(uint64_t) + kMaxStages * sizeof(int) + 16;  // barriers
}

template <int NT, int W>
__global__ void __launch_bounds__(W * 32, kMmRegThreads / (W * 32)) mul_mat_kernel(const __grid_constant__ MmParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int ring_bytes = p.n_stages * p.slot_bytes;
    const int n_units = p.n_in / 256;
    const int n_sl = p.n_in / 16, n_sub = p.n_in / 32;
    const int xs16_st = n_sl + 4, xs32_st = n_sub + 4;  // token rows 4 banks apart, 16-byte aligned
    uint2 *bf = reinterpret_cast<uint2 *>(smem + ring_bytes);                  // [n_sl][2 NT][4 lanes c]
    float *xf = reinterpret_cast<float *>(bf + n_sl * 2 * NT * 4);            // [NT][n_in] if has_float
    float *xs16 = xf + (p.has_float ? NT * p.n_in : 0);                        // [NT][xs16_st]
    float *xs32 = xs16 + NT * xs16_st;                                         // [NT][xs32_st]
    float *tab_all = xs32 + NT * xs32_st;                                      // [8 warps][8][kTabStride]
    float2 *red = reinterpret_cast<float2 *>(tab_all + W * 8 * kTabStride);   // [kTcGroup][W][32]
    uint64_t *full_bar = reinterpret_cast<uint64_t *>(red + kTcGroup * W * 32);
    uint64_t *empty_bar = full_bar + kMaxStages;
    int *rel_cnt = reinterpret_cast<int *>(empty_bar + kMaxStages);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, c = lane & 3;
    float *tab = tab_all + warp * 8 * kTabStride;

    const int tile0 = static_cast<int>((static_cast<int64_t>(blockIdx.x) * p.n_tiles) / gridDim.x);
    const int tile1 = static_cast<int>((static_cast<int64_t>(blockIdx.x + 1) * p.n_tiles) / gridDim.x);
    const int n_tiles = tile1 - tile0;
    if (threadIdx.x == 0) {
        for (int s = 0; s < p.n_stages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], W);
            rel_cnt[s] = 0;
        }
        fence_mbar_init();
    }
    __syncthreads();
    // quantised tiles: one bulk copy per row pair, the lanes of one warp issuing them
    // together; float tiles: one copy
    auto issue = [&](int it) {
        const int s = it % p.n_stages;
        const MmSeg &sg = p.seg[seg_of(p, tile0 + it)];
        const int row0 = (tile0 + it - sg.tile0) * sg.rows;
        const int rows = min(sg.rows, sg.n_out - row0);
        if (lane == 0) mbar_arrive_expect_tx(&full_bar[s], static_cast<uint32_t>(rows * sg.row_bytes));
        __syncwarp();
        const uint8_t *src = sg.w + static_cast<int64_t>(row0) * sg.row_bytes;
        if (!quant_type(sg.w_type)) {
            if (lane == 0) bulk_g2s(smem + s * p.slot_bytes, src, static_cast<uint32_t>(rows * sg.row_bytes), &full_bar[s]);
        } else if (2 * lane < rows) {
            const int nr = min(2, rows - 2 * lane);
            bulk_g2s(smem + s * p.slot_bytes + lane * sg.sstride, src + static_cast<int64_t>(2 * lane) * sg.row_bytes,
                     static_cast<uint32_t>(nr * sg.row_bytes), &full_bar[s]);
        }
    };
    // the weights are constants of the model: stream them before the dependency wait
    if (warp == 0)
        for (int it = 0; it < n_tiles && it < p.n_stages; ++it) issue(it);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" :::);

    // f32 x rows 16-byte aligned: 4 values per load
    const bool x_vec = p.x_dtype == SQMIX_F32 &&
                       ((reinterpret_cast<uintptr_t>(p.x) | static_cast<uintptr_t>(p.x_stride * 4)) & 15) == 0;
    // x -> the B fragments and slice sums of this warp's units (no other warp reads them):
    // entry (slice l of unit u, token t, lane c) covers x values 16 (16 u + l) + 4 c .. + 3
    for (int u = warp; u < n_units; u += W) {
        constexpr int kE = 2 * NT;  // 64 NT entries per unit
        float v[kE][4];
#pragma unroll
        for (int e = 0; e < kE; ++e) {
            const int idx = e * 32 + lane;
            const int t = (idx >> 2) % NT, sl = 16 * u + (idx >> 2) / NT;
            const int64_t i0 = static_cast<int64_t>(t) * p.x_stride + 16 * sl + 4 * c;
            if (t >= p.n_tok) {
                v[e][0] = v[e][1] = v[e][2] = v[e][3] = 0.f;
            } else if (x_vec) {
                const float4 xv = *reinterpret_cast<const float4 *>(static_cast<const float *>(p.x) + i0);
                v[e][0] = xv.x, v[e][1] = xv.y, v[e][2] = xv.z, v[e][3] = xv.w;
            } else {
#pragma unroll
                for (int q = 0; q < 4; ++q) v[e][q] = load_act(p.x, i0 + q, p.x_dtype);
            }
        }
#pragma unroll
        for (int e = 0; e < kE; ++e) {
            const int idx = e * 32 + lane;
            const int t = (idx >> 2) % NT, sl = 16 * u + (idx >> 2) / NT;
            __half hv[4], lv[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                hv[q] = __float2half_rn(v[e][q]);
                lv[q] = __float2half_rn(v[e][q] - __half2float(hv[q]));
            }
            bf[(sl * 2 * NT + 2 * t) * 4 + c] =
                make_uint2(h2_as_u32(__halves2half2(hv[0], hv[2])), h2_as_u32(__halves2half2(hv[1], hv[3])));
            bf[(sl * 2 * NT + 2 * t + 1) * 4 + c] =
                make_uint2(h2_as_u32(__halves2half2(lv[0], lv[2])), h2_as_u32(__halves2half2(lv[1], lv[3])));
            float sum = (v[e][0] + v[e][1]) + (v[e][2] + v[e][3]);  // lanes c of a slice are consecutive
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            if (c == 0) xs16[t * xs16_st + sl] = sum;
        }
        __syncwarp();
        if (lane < 8 * NT) {
            const int t = lane >> 3, j = lane & 7;
            const float *s16 = xs16 + t * xs16_st + 16 * u + 2 * j;
            xs32[t * xs32_st + 8 * u + j] = s16[0] + s16[1];
        }
        if (p.has_float)  // f32 x for float-typed rows: lane l keeps values 256 u + 8 l .. + 7
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                float4 *dst = reinterpret_cast<float4 *>(xf + t * p.n_in + 256 * u + 8 * lane);
                const int64_t i0 = static_cast<int64_t>(t) * p.x_stride + 256 * u + 8 * lane;
                if (t >= p.n_tok) {
                    dst[0] = dst[1] = make_float4(0.f, 0.f, 0.f, 0.f);
                } else if (x_vec) {
                    const float4 *src = reinterpret_cast<const float4 *>(static_cast<const float *>(p.x) + i0);
                    dst[0] = src[0];
                    dst[1] = src[1];
                } else {
                    dst[0] = make_float4(load_act(p.x, i0, p.x_dtype), load_act(p.x, i0 + 1, p.x_dtype),
                                         load_act(p.x, i0 + 2, p.x_dtype), load_act(p.x, i0 + 3, p.x_dtype));
                    dst[1] = make_float4(load_act(p.x, i0 + 4, p.x_dtype), load_act(p.x, i0 + 5, p.x_dtype),
                                         load_act(p.x, i0 + 6, p.x_dtype), load_act(p.x, i0 + 7, p.x_dtype));
                }
            }
    }
    __syncwarp();

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
            const MmSeg &sg = p.seg[seg_of(p, tile0 + it)];
            const uint8_t *rg = smem + s * p.slot_bytes + g * sg.sstride;  // tile row 2g: MMA row g
            const uint8_t *rg8 = rg + sg.row_bytes;                           // tile row 2g + 1: MMA row g + 8
            const int wt = sg.w_type;
            float y0 = 0.f, y1 = 0.f;
            for (int u = warp; u < n_units; u += W) {
                if (wt == SQMIX_Q4_K)
                    unit_q4k<NT>(rg, rg8, u, g, c, bf, xs32, xs32_st, tab, y0, y1);
                else if (wt == SQMIX_Q6_K)
                    unit_q6k<NT>(rg, rg8, u, g, c, bf, xs16, xs16_st, tab, y0, y1);
                else if (wt == SQMIX_Q8_0)
                    unit_q8_0<NT>(rg, rg8, u, g, c, bf, tab, y0, y1);
                else
                    unit_float<NT>(smem + s * p.slot_bytes, sg.sstride, min(sg.rows, sg.n_out - (tile0 + it - sg.tile0) * sg.rows),
                                   wt, u, lane, xf, p.n_in, g, c, y0, y1);
            }
            red[((it - gb) * W + warp) * 32 + lane] = make_float2(y0, y1);
            // release the slot; the warp that releases it last refills it
            __syncwarp();
            int last = 0;
            if (lane == 0) {
                mbar_arrive(&empty_bar[s]);
                last = atomicAdd(&rel_cnt[s], 1) == W - 1;
                if (last) rel_cnt[s] = 0;
            }
            last = __shfl_sync(0xffffffffu, last, 0);
            if (last && it + p.n_stages < n_tiles) {
                // every warp has arrived: this wait returns at once
                int e_ok = 1;
                if (lane == 0) e_ok = mbar_wait(&empty_bar[s], (it / p.n_stages) & 1);
                if (__shfl_sync(0xffffffffu, e_ok, 0))
                    issue(it + p.n_stages);
                else
                    ok = false;
            }
        }
        if (__syncthreads_or(!ok)) {
            ok = false;
            break;
        }
        // the group's outputs (tile, MMA row r, token n): lane 4 (r % 8) + n, component r / 8;
        // MMA row r is tile row 2 (r % 8) + r / 8 of a quantised tile, row r of a float tile
        for (int o = threadIdx.x; o < (ge - gb) * kTcRows * NT; o += W * 32) {
            const int tl = o / (kTcRows * NT), rem = o % (kTcRows * NT), r = rem / NT, n = rem % NT;
            const int ln = 4 * (r & 7) + n;
            float acc = 0.f;
#pragma unroll
            for (int wv = 0; wv < W; ++wv) {
                const float2 q2 = red[(tl * W + wv) * 32 + ln];
                acc += r < 8 ? q2.x : q2.y;
            }
            const int t = tile0 + gb + tl;
            const MmSeg &sg = p.seg[seg_of(p, t)];
            const int tr = quant_type(sg.w_type) ? 2 * (r & 7) + (r >> 3) : r;
            const int row = (t - sg.tile0) * sg.rows + tr;
            if (r < sg.rows && row < sg.n_out && n < p.n_tok) sg.y[static_cast<int64_t>(n) * sg.y_stride + row] = acc;
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

template <typename K>
int launch_pdl(K kernel, std::atomic<uint64_t> &attr_devices, const MmParams &p, int grid, int threads, size_t smem,
               cudaStream_t st) {
    {
        const cudaError_t e = set_smem_once(attr_devices, kernel, 227 * 1024);
        if (e != cudaSuccess) return cuda_status(e, "mul_mat smem attribute");
    }
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_status(cudaLaunchKernelEx(&cfg, kernel, p), "mul_mat launch");
}

template <int NT, int W>
int launch_mm(const MmParams &p, int grid, size_t smem, cudaStream_t st) {
    static std::atomic<uint64_t> attr_devices{0};
    return launch_pdl(mul_mat_kernel<NT, W>, attr_devices, p, grid, W * 32, smem, st);
}

template <int W>
int launch_mm_nt(int NT, const MmParams &p, int grid, size_t smem, cudaStream_t st) {
    return NT == 1 ? launch_mm<1, W>(p, grid, smem, st)
           : NT == 2 ? launch_mm<2, W>(p, grid, smem, st)
                     : launch_mm<4, W>(p, grid, smem, st);
}

int64_t row_bytes_of(int32_t w_type, int64_t n_in) {
    const int ub = unit_bytes(w_type);
    if (ub == 0 || n_in <= 0 || n_in % 256 != 0) return 0;
    return n_in / 256 * ub;
}

int check_entry(const sqmix_mul_mat_args *a, int i) {
    SQMIX_CHECK_ARG(a->w && a->x && a->y, "mul_mat[%d]: null pointer argument", i);
    SQMIX_CHECK_ARG(unit_bytes(a->w_type) != 0, "mul_mat[%d]: weight type %d (q8_0, q4_K, q6_K, f32, f16, bf16)", i,
                    a->w_type);
    SQMIX_CHECK_ARG(a->n_in >= 256 && a->n_in <= kMaxIn && a->n_in % 256 == 0,
                    "mul_mat[%d]: n_in=%lld must be a multiple of 256 in [256, %d]", i, (long long)a->n_in, kMaxIn);
    SQMIX_CHECK_ARG(a->n_out >= 1 && a->n_out <= (1 << 24), "mul_mat[%d]: n_out=%lld", i, (long long)a->n_out);
    SQMIX_CHECK_ARG(a->n_tokens >= 1, "mul_mat[%d]: n_tokens=%d", i, a->n_tokens);
    SQMIX_CHECK_ARG(a->x_dtype == SQMIX_F32 || a->x_dtype == SQMIX_F16 || a->x_dtype == SQMIX_BF16,
                    "mul_mat[%d]: x dtype %d", i, a->x_dtype);
    const int64_t rb = row_bytes_of(a->w_type, a->n_in);
    SQMIX_CHECK_ARG(a->w_row_bytes == rb, "mul_mat[%d]: w_row_bytes=%lld, rows must be contiguous (%lld bytes)", i,
                    (long long)a->w_row_bytes, (long long)rb);
    // rows reach shared memory by 1-D bulk copies: 16-byte multiples (q6_K: n_in % 2048 == 0)
    SQMIX_CHECK_ARG(rb % 16 == 0,
                    "mul_mat[%d]: a row of %lld bytes is not a multiple of 16 (q6_K needs n_in %% 2048 == 0)", i,
                    (long long)rb);
    SQMIX_CHECK_ARG((reinterpret_cast<uintptr_t>(a->w) & 15) == 0, "mul_mat[%d]: w must be 16-byte aligned", i);
    SQMIX_CHECK_ARG(a->x_stride >= a->n_in && a->y_stride >= a->n_out, "mul_mat[%d]: token strides too small", i);
    return SQMIX_OK;
}

}  // namespace
}  // namespace sqmix

using namespace sqmix;

extern "C" int64_t sqmix_mul_mat_row_bytes(int32_t w_type, int64_t n_in) { return row_bytes_of(w_type, n_in); }

extern "C" int sqmix_mul_mat_group(const sqmix_mul_mat_args *args, int32_t n, sqmix_stream_t stream) {
    SQMIX_CHECK_ARG(args != nullptr, "mul_mat: null args");
    SQMIX_CHECK_ARG(n >= 1 && n <= SQMIX_MUL_MAT_MAX_GROUP, "mul_mat_group: n=%d must be in [1, %d]", n,
                    SQMIX_MUL_MAT_MAX_GROUP);
    for (int i = 0; i < n; ++i) {
        const int rc = check_entry(&args[i], i);
        if (rc != SQMIX_OK) return rc;
    }
    const sqmix_mul_mat_args &a0 = args[0];
    for (int i = 1; i < n; ++i)
        SQMIX_CHECK_ARG(args[i].x == a0.x && args[i].x_dtype == a0.x_dtype && args[i].x_stride == a0.x_stride &&
                            args[i].n_tokens == a0.n_tokens && args[i].n_in == a0.n_in,
                        "mul_mat_group: entry %d does not share x (pointer, dtype, stride, n_tokens, n_in) with entry 0",
                        i);
    if (a0.n_tokens >= kGemmMinTokens) {  // the GEMM form needs x rows 16-byte aligned (tiles 0 otherwise)
        const int tiles = mul_mat_gemm_tiles(args, n);
        if (tiles > 0 && (a0.n_tokens >= kGemmTokens || tiles >= gemm_min_tiles(a0.n_tokens)))
            return mul_mat_gemm_launch(args, n, reinterpret_cast<cudaStream_t>(stream));
    }
    // the launch's tile list: the projections in call order, 16-row tiles for the
    // quantised formats, float-typed rows as many as fit the slot (up to 16)
    MmParams p = {};
    int max_sstride = 0;
    int64_t max_float_rb = 0;
    for (int i = 0; i < n; ++i) {
        const int64_t rb = row_bytes_of(args[i].w_type, args[i].n_in);
        if (quant_type(args[i].w_type))
            max_sstride = std::max(max_sstride, static_cast<int>(2 * rb + 16));
        else
            max_float_rb = std::max(max_float_rb, rb);
    }
    p.slot_bytes = static_cast<int>(std::max<int64_t>(max_sstride > 0 ? kTcRows / 2 * max_sstride : kFloatSlot, max_float_rb));
    p.slot_bytes = (p.slot_bytes + 127) / 128 * 128;
    for (int i = 0; i < n; ++i) {
        const int64_t rb = row_bytes_of(args[i].w_type, args[i].n_in);
        MmSeg &sg = p.seg[p.n_seg];
        sg.w = static_cast<const uint8_t *>(args[i].w);
        sg.y_stride = args[i].y_stride;
        sg.w_type = args[i].w_type;
        sg.row_bytes = static_cast<int>(rb);
        sg.n_out = static_cast<int>(args[i].n_out);
        sg.tile0 = p.n_tiles;
        if (quant_type(sg.w_type)) {
            sg.rows = kTcRows;
            sg.sstride = static_cast<int>(2 * rb + 16);  // rb / 4 is 0 or 4 mod 8: sstride / 4 is 4 mod 8
        } else {
            sg.rows = static_cast<int>(std::min<int64_t>(kTcRows, p.slot_bytes / rb));
            sg.sstride = sg.row_bytes;
            p.has_float = 1;
        }
        p.n_tiles += (sg.n_out + sg.rows - 1) / sg.rows;
        ++p.n_seg;
    }
    const int sms = sqmix_device_sm_count(-1);
    if (sms <= 0) return cuda_status(cudaErrorInvalidDevice, "mul_mat device");
    p.n_in = static_cast<int>(a0.n_in);
    p.x_dtype = a0.x_dtype;
    p.x_stride = a0.x_stride;
    p.status = a0.status;
    // 16 warps (one per unit) for rows of 16 or more units when a ring of 2 slots fits
    // beside the rest, else 8; as many CTAs per SM as the registers allow and leave room
    // for a ring of at least 2 slots
    auto smem_budget = [](int ctas) { return static_cast<size_t>(228 * 1024 / ctas - 1024); };
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int elt = a0.x_dtype == SQMIX_F32 ? 4 : 2;
    for (int t0 = 0; t0 < a0.n_tokens; t0 += kMaxPassTokens) {
        const int nt = std::min(kMaxPassTokens, a0.n_tokens - t0);
        const int NT = nt <= 1 ? 1 : nt <= 2 ? 2 : 4;
        MmParams q = p;
        q.x = static_cast<const uint8_t *>(a0.x) + static_cast<int64_t>(t0) * a0.x_stride * elt;
        q.n_tok = nt;
        for (int s = 0; s < q.n_seg; ++s) q.seg[s].y = args[s].y + static_cast<int64_t>(t0) * q.seg[s].y_stride;
        const int W = q.n_in / 256 >= 16 &&
                              tc_extra_bytes(NT, 16, q.n_in, q.has_float != 0) + 2 * static_cast<size_t>(q.slot_bytes) <=
                                  227 * 1024
                          ? 16
                          : 8;
        const size_t extra = tc_extra_bytes(NT, W, q.n_in, q.has_float != 0);
        int ctas = kMmRegThreads / (W * 32);
        while (ctas > 1 && extra + 2 * static_cast<size_t>(q.slot_bytes) > smem_budget(ctas)) --ctas;
        const size_t budget = std::min<size_t>(smem_budget(ctas), 227 * 1024);
        if (extra + 2 * static_cast<size_t>(q.slot_bytes) > budget)
            return cuda_status(cudaErrorInvalidValue, "mul_mat shared memory");
        q.n_stages = static_cast<int>(std::min<size_t>(kMaxStages, (budget - extra) / q.slot_bytes));
        const size_t smem = static_cast<size_t>(q.n_stages) * q.slot_bytes + extra;
        const int grid = std::min(q.n_tiles, ctas * sms);
        const int rc = W == 16 ? launch_mm_nt<16>(NT, q, grid, smem, st) : launch_mm_nt<8>(NT, q, grid, smem, st);
        if (rc != SQMIX_OK) return rc;
    }
    return SQMIX_OK;
}

extern "C" int sqmix_mul_mat(const sqmix_mul_mat_args *a, sqmix_stream_t stream) {
    SQMIX_CHECK_ARG(a != nullptr, "mul_mat: null args");
    return sqmix_mul_mat_group(a, 1, stream);
}
