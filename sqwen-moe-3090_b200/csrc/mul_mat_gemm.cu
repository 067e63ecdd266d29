// mul_mat_gemm.cu -- the mixer projections at prefill (n_tokens >= 128, or fewer with
// enough output tiles; mul_mat.cu decides): ggml_mul_mat(w, x) as a tensor-core GEMM,
//     Y[t][o] = sum_i W[o][i] x[t][i].
//
// An item is a 128 x 128 tile of Y (128 weight rows of one projection x 128 tokens); the
// CTAs (one per SM, grid = min(items, SMs)) walk the items.  tcgen05.mma with the
// dequantised weights as the A operand in TENSOR memory and x as the B operand straight
// from its tensor-map boxes in 128-byte-swizzled shared memory, an f32 accumulator in
// tensor memory.  The contraction runs in stages of 64 values:
//   warp 1, lane 0: brings the stage's x boxes (128 tokens x 64 values) into the x ring
//     by tensor-map loads (no multicast; tokens beyond n_tokens read as zeros);
//   warps 4-11 (producers): dequantise the stage's 128 x 64 weight values (warp w: rows
//     32 (w % 4) .., values 32 ((w - 4) / 4) ..; thread = row) as ggml does (q4_K
//     d sc q - dmin m, q6_K d sc (q - 32), q8_0 d q, float rows as they are) in f32 and
//     store them into the stage's tensor-memory columns (tcgen05.st);
//   warp 0, lane 0: waits for both halves of a stage, issues its MMAs (f32 x:
//     .kind::tf32, M 128 x N 128 x K 8; f16 / bf16 x: .kind::f16 with the weights
//     rounded to x's type, K 16) and commits them to the stage's empty barrier, which
//     frees the weight columns and the x slot;
//   warps 0-3 (epilogue): after the item's last commit read the accumulator (thread =
//     weight row, 32 tokens per tensor-memory load) and store Y.
// Shared memory holds only x and the barriers; the weights never pass through it.
// Precision: the tensor cores read tf32 operands (10-bit mantissa) for f32 x -- each
// weight and x value truncated to tf32 -- or f16 / bf16 ones; sums in f32.  The decode
// form (mul_mat.cu) keeps f32-exact sums for <= 4 tokens per weight stream.  x rows must
// be 16-byte aligned (the tensor map); the host sends other x to the decode form.
#include <math.h>

#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "sqmix.h"
#include "tc.cuh"

namespace sqmix {
namespace {

constexpr int kGM = 128;            // weight rows per item (MMA M)
constexpr int kGN = 128;            // tokens per item (MMA N)
constexpr int kGK = 64;             // contraction values per stage
constexpr int kGStages = 4;         // stages in flight (weight columns and x slots)
constexpr int kGWDepth = 2;         // weight boxes in flight
constexpr int kGWarps = 12;
constexpr int kGThreads = kGWarps * 32;
constexpr int kGProdWarp0 = 4;
constexpr int kGProdWarps = 8;
constexpr int kGMaxSeg = SQMIX_MUL_MAT_MAX_GROUP;
constexpr int kGXSlot = kGN * kGK * 4;   // 32 KB: one stage of x (f32: two 16 KB boxes; 16-bit: one)
constexpr int kGWBoxMax = 272;          // bytes of a weight row in one weight box (q8_0's unit)
constexpr int kGWSlot = kGM * kGWBoxMax;  // one weight box of 128 rows
constexpr int kGWOff = kGStages * kGXSlot;
constexpr int kGBarOff = kGWOff + kGWDepth * kGWSlot;
constexpr int kGSmem = kGBarOff + 256 + 1024;  // + slack for the 1024-byte alignment of the rings
// tensor memory: the accumulator (128 columns), then kGStages stages of 64 weight columns
constexpr uint32_t kGTmemCols = 512;
constexpr uint32_t kGAcol0 = kGN;

struct GemmSeg {
    CUtensorMap wmap;  // the weight rows in boxes of 128 rows (one unit of 256 values, or one stage of float rows)
    const uint8_t *w;
    float *y;
    int64_t y_stride;
    int w_type;
    int row_bytes;
    int n_out;
    int item0;    // first item of the projection
    int m_tiles;  // ceil(n_out / kGM)
    int box_rows; // rows of a weight box: min(kGM, n_out)
};

struct GemmParams {
    CUtensorMap xmap;  // x as [n_tok][n_in], boxes of 128 bytes x 128 tokens, 128-byte swizzle
    GemmSeg seg[kGMaxSeg];
    int n_seg, n_items;
    int n_in, n_tok, t_tiles;
    int x_dtype;
    uint32_t *status;
};

__device__ __forceinline__ float f16_bits(uint32_t h) { return __half2float(__ushort_as_half(static_cast<unsigned short>(h))); }
// An integer 0 <= q < 2^23 (the low bits of w selected by mask after a shift) as a float,
// exactly, on the integer and FMA pipes: 2^23 + q has q as its mantissa.
__device__ __forceinline__ float small_int_f32(uint32_t bits) { return __uint_as_float(0x4B000000u | bits) - 8388608.0f; }

// Raw weight words of 32 consecutive values k0 .. k0 + 31 (k0 % 32 == 0) of a row:
//   q4_K: [0..3] the unit's 16-byte header, [4..11] the 32 nibble bytes;
//   q6_K: [0..8] ql and [9..17] qh as the aligned words covering them, [18] the word
//         holding d, [19] the word holding the two int8 scales;
//   q8_0: [0..8] the aligned words covering the 32 int8, [9] the word holding d;
//   f32:  [0..31]; f16 / bf16: [0..15].
// A weight box: 128 rows x wbox_bytes(type) bytes, covering `spb` stages of 64 values
// (a 256-value unit of the block formats -- q6_K's unit at its 16-byte-aligned start
// below -- or one stage of float rows)
__host__ __device__ constexpr int wbox_bytes(int t) {
    return t == SQMIX_Q4_K ? 144 : t == SQMIX_Q6_K ? 224 : t == SQMIX_Q8_0 ? 272 : t == SQMIX_F32 ? 256 : 128;
}
__host__ __device__ constexpr int wbox_stages(int t) { return t == SQMIX_F32 || t == SQMIX_F16 || t == SQMIX_BF16 ? 1 : 4; }

// The raw words of 32 consecutive values k0 .. k0 + 31 of a row whose current weight box
// starts at `rb` in shared memory
__device__ __forceinline__ const uint32_t *sm_word(const uint8_t *p) {
    return reinterpret_cast<const uint32_t *>(reinterpret_cast<uintptr_t>(p) & ~static_cast<uintptr_t>(3));
}
__device__ __forceinline__ void load_w32s(const uint8_t *rb, int wt, int k0, uint32_t (&r)[32]) {
    if (wt == SQMIX_Q4_K) {
        const int j = (k0 >> 5) & 7;
        const uint4 h = *reinterpret_cast<const uint4 *>(rb);
        const uint4 q0 = *reinterpret_cast<const uint4 *>(rb + 16 + 32 * (j >> 1));
        const uint4 q1 = *reinterpret_cast<const uint4 *>(rb + 32 + 32 * (j >> 1));
        r[0] = h.x, r[1] = h.y, r[2] = h.z, r[3] = h.w;
        r[4] = q0.x, r[5] = q0.y, r[6] = q0.z, r[7] = q0.w, r[8] = q1.x, r[9] = q1.y, r[10] = q1.z, r[11] = q1.w;
    } else if (wt == SQMIX_Q6_K) {
        const int u = k0 >> 8, i0 = k0 & 255, hh = i0 >> 7, kq = (i0 & 127) >> 5;
        const uint8_t *ub = rb + ((210 * u) & 15);  // the unit inside its 16-byte-aligned box
        const uint32_t *ql = sm_word(ub + 64 * hh + 32 * (kq & 1)), *qh = sm_word(ub + 128 + 32 * hh);
#pragma unroll
        for (int i = 0; i < 9; ++i) {
            r[i] = ql[i];
            r[9 + i] = qh[i];
        }
        r[18] = *sm_word(ub + 208);
        r[19] = *sm_word(ub + 192 + 8 * hh + 2 * kq);
    } else if (wt == SQMIX_Q8_0) {
        const uint8_t *bb = rb + 34 * ((k0 >> 5) & 7);
        const uint32_t *q = sm_word(bb + 2);
#pragma unroll
        for (int i = 0; i < 9; ++i) r[i] = q[i];
        r[9] = *sm_word(bb);
    } else if (wt == SQMIX_F32) {
        const uint4 *f = reinterpret_cast<const uint4 *>(rb + 4 * (k0 & 63));
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint4 a = f[i];
            r[4 * i] = a.x, r[4 * i + 1] = a.y, r[4 * i + 2] = a.z, r[4 * i + 3] = a.w;
        }
    } else {
        const uint4 *f = reinterpret_cast<const uint4 *>(rb + 2 * (k0 & 63));
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint4 a = f[i];
            r[4 * i] = a.x, r[4 * i + 1] = a.y, r[4 * i + 2] = a.z, r[4 * i + 3] = a.w;
        }
    }
}

// The raw words of load_w32s as 32 f32 values (K order), each computed as ggml
// dequantises it
__device__ __forceinline__ void conv_w32(const uint32_t (&r)[32], int wt, int k0, float (&v)[32]) {
    if (wt == SQMIX_Q4_K) {
        const int j = (k0 >> 5) & 7;
        const float d = f16_bits(r[0] & 0xFFFF), dmin = f16_bits(r[0] >> 16);
        const int sh = 8 * (j & 3);
        const uint32_t b0 = (r[1] >> sh) & 0xFF, b1 = (r[2] >> sh) & 0xFF, b2 = (r[3] >> sh) & 0xFF;
        const uint32_t sc = j < 4 ? b0 & 63 : (b2 & 0xF) | ((b0 >> 6) << 4);
        const uint32_t m = j < 4 ? b1 & 63 : (b2 >> 4) | ((b1 >> 6) << 4);
        const float d1 = d * static_cast<float>(sc), m1 = dmin * static_cast<float>(m);
        const int ns = 4 * (j & 1);
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int e = 0; e < 4; ++e) v[4 * i + e] = fmaf(d1, small_int_f32((r[4 + i] >> (8 * e + ns)) & 0xF), -m1);
    } else if (wt == SQMIX_Q6_K) {
        const int u = k0 >> 8, kq = (k0 & 127) >> 5;
        const bool mis = u & 1;
        const float d = f16_bits(mis ? r[18] >> 16 : r[18] & 0xFFFF);
        const int so = (2 * u + 2 * kq) & 3;  // byte offset of the scale pair in its word
        const float d0 = d * static_cast<float>(static_cast<int8_t>((r[19] >> (8 * so)) & 0xFF));
        const float d1 = d * static_cast<float>(static_cast<int8_t>((r[19] >> (8 * so + 8)) & 0xFF));
        const int lsh = 4 * (kq >> 1), hsh = 2 * kq;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t ql = mis ? __byte_perm(r[i], r[i + 1], 0x5432) : r[i];
            const uint32_t qh = mis ? __byte_perm(r[9 + i], r[10 + i], 0x5432) : r[9 + i];
#pragma unroll
            for (int e = 0; e < 4; ++e)
                v[4 * i + e] = (i < 4 ? d0 : d1) *
                               (small_int_f32(((ql >> (8 * e + lsh)) & 0xF) | (((qh >> (8 * e + hsh)) & 3) << 4)) - 32.0f);
        }
    } else if (wt == SQMIX_Q8_0) {
        const int b = k0 >> 5;
        const bool mis = !(b & 1);
        const float d = f16_bits((b & 1) ? r[9] >> 16 : r[9] & 0xFFFF);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t w = mis ? __byte_perm(r[i], r[i + 1], 0x5432) : r[i];
#pragma unroll
            for (int e = 0; e < 4; ++e) v[4 * i + e] = d * (small_int_f32(((w >> (8 * e)) & 0xFF) ^ 0x80) - 128.0f);
        }
    } else if (wt == SQMIX_F32) {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
    } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const float2 f = wt == SQMIX_F16 ? __half22float2(u32_as_h2(r[i]))
                                             : __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&r[i]));
            v[2 * i] = f.x;
            v[2 * i + 1] = f.y;
        }
    }
}

// 2-D tensor-map load of box (x0 = value, y0 = token) into shared memory (no multicast)
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x0, int y0, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x0), "r"(y0), "r"(smem_u32(bar))
        : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem] with tf32 operands; one thread
__device__ __forceinline__ void mma_ts_tf32(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// instruction descriptor of .kind::tf32: tf32 A and B, f32 accumulator, both K-major
__host__ __device__ constexpr uint32_t idesc_tf32_f32(int m, int n) {
    return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(m >> 4) << 24);
}

__global__ void __launch_bounds__(kGThreads, 1) mul_mat_gemm_kernel(const __grid_constant__ GemmParams p) {
    extern __shared__ uint8_t gsm_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(gsm_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t *ring_x = sm;           // kGStages slots of x boxes
    uint8_t *ring_w = sm + kGWOff;  // kGWDepth slots of weight boxes
    uint64_t *afull = reinterpret_cast<uint64_t *>(sm + kGBarOff);  // weight columns stored (producer warps)
    uint64_t *xfull = afull + kGStages;                              // x boxes landed (transaction bytes)
    uint64_t *sempty = xfull + kGStages;                             // the stage's MMAs are done
    uint64_t *done = sempty + kGStages;                              // an item's MMAs are done
    uint64_t *wfull = done + 1;                                      // weight boxes landed
    uint64_t *wempty = wfull + kGWDepth;                             // weight boxes converted (producer warps)
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(wempty + kGWDepth);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool f32x = p.x_dtype == SQMIX_F32;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kGStages; ++s) {
            mbar_init(&afull[s], kGProdWarps);
            mbar_init(&xfull[s], 1);
            mbar_init(&sempty[s], 1);
        }
        mbar_init(done, 1);
        for (int s = 0; s < kGWDepth; ++s) {
            mbar_init(&wfull[s], 1);
            mbar_init(&wempty[s], kGProdWarps);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0) tc::tmem_alloc(tmem_slot, kGTmemCols);
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem = *tmem_slot;
    const int n_k = p.n_in / kGK;
    // x comes from the kernel before; the weights are model constants
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" :::);

    bool ok = true;
    int done_phase = 0;
    int x_issued = 0;  // global stages whose x boxes were requested (warp 1, lane 0)
    int w_issued = 0;  // weight boxes requested (warp 2, lane 0)
    int wblk0 = 0;     // weight boxes of the items before this one (every thread counts them)
    for (int item = blockIdx.x; item < p.n_items; item += gridDim.x) {
        int si = 0;
        while (si + 1 < p.n_seg && item >= p.seg[si + 1].item0) ++si;
        const GemmSeg &sg = p.seg[si];
        const int rel = item - sg.item0;
        const int m0 = (rel / p.t_tiles) * kGM, t0 = (rel % p.t_tiles) * kGN;
        // stage counter continues across items: stage k of this item is ring use g0 + k
        const int g0 = ((item - blockIdx.x) / gridDim.x) * n_k;
        const int spb = wbox_stages(sg.w_type), wbytes = wbox_bytes(sg.w_type);
        if (warp >= kGProdWarp0) {
            const int q = warp & 3, h = (warp - kGProdWarp0) >> 2;
            const int r = 32 * q + lane;
            const uint32_t lane_base = static_cast<uint32_t>(32 * q) << 16;
            for (int kc = 0; kc < n_k; ++kc) {
                const int gs = g0 + kc, s = gs % kGStages;
                const int gb = wblk0 + kc / spb, ws = gb % kGWDepth;
                if (kc % spb == 0 && !*abort_flag && !mbar_wait(&wfull[ws], (gb / kGWDepth) & 1)) *abort_flag = 1;
                if (*abort_flag) break;
                float v[32];
                if (r < sg.box_rows) {
                    uint32_t raw[32];
                    load_w32s(ring_w + ws * kGWSlot + r * wbytes, sg.w_type, kc * kGK + 32 * h, raw);
                    conv_w32(raw, sg.w_type, kc * kGK + 32 * h, v);
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = 0.f;
                }
                if (kc % spb == spb - 1) {  // the box is converted: release it to the issuer
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&wempty[ws]);
                }
                if (gs >= kGStages && !*abort_flag && !mbar_wait(&sempty[s], ((gs / kGStages) - 1) & 1)) *abort_flag = 1;
                if (*abort_flag) break;
                tc::fence_after();
                const uint32_t col = tmem + lane_base + kGAcol0 + s * kGK;
                if (f32x) {
                    uint32_t o[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(v[i]);
                    tc::st32(col + 32 * h, o);
                } else {
                    uint32_t o[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        if (p.x_dtype == SQMIX_F16) {
                            o[i] = h2_as_u32(__floats2half2_rn(v[2 * i], v[2 * i + 1]));
                        } else {
                            const __nv_bfloat162 b2 = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
                            o[i] = *reinterpret_cast<const uint32_t *>(&b2);
                        }
                    }
                    tc::st16(col + 16 * h, o);
                }
                tc::wait_st();
                tc::fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&afull[s]);
            }
        } else if (warp == 0) {
            if (lane == 0) {
                const uint32_t idesc = f32x                      ? idesc_tf32_f32(kGM, kGN)
                                       : p.x_dtype == SQMIX_F16 ? tc::idesc_f16_f32(kGM, kGN, 0, 0)
                                                                : tc::idesc_bf16_f32(kGM, kGN, 0, 0);
                for (int kc = 0; kc < n_k; ++kc) {
                    const int gs = g0 + kc, s = gs % kGStages;
                    if (!*abort_flag && !mbar_wait(&afull[s], (gs / kGStages) & 1)) *abort_flag = 1;
                    if (!*abort_flag && !mbar_wait(&xfull[s], (gs / kGStages) & 1)) *abort_flag = 1;
                    if (*abort_flag) break;
                    tc::fence_after();
                    const uint32_t xs = smem_u32(ring_x + s * kGXSlot), a = tmem + kGAcol0 + s * kGK;
                    if (f32x) {  // K 8 per MMA: boxes of 32 values, 32 bytes per step
#pragma unroll
                        for (int kk = 0; kk < 8; ++kk)
                            mma_ts_tf32(tmem, a + 8 * kk, tc::desc_sw128(xs + (kk >> 2) * (kGN * 128) + (kk & 3) * 32, 16, 1024),
                                        idesc, (kc | kk) != 0 ? 1u : 0u);
                    } else {  // K 16 per MMA: one box of 64 values
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            tc::mma_ts(tmem, a + 8 * kk, tc::desc_sw128(xs + kk * 32, 16, 1024), idesc, (kc | kk) != 0 ? 1u : 0u);
                    }
                    tc::commit(&sempty[s]);
                }
                tc::commit(done);  // arrives when every MMA issued so far is complete
            }
            __syncwarp();
        } else if (warp == 1) {
            if (lane == 0) {
                const uint32_t xbytes = f32x ? 2 * kGN * 128 : kGN * 128;
                for (int kc = 0; kc < n_k; ++kc) {
                    const int gs = g0 + kc, s = gs % kGStages;
                    if (gs >= kGStages && !*abort_flag && !mbar_wait(&sempty[s], ((gs / kGStages) - 1) & 1)) *abort_flag = 1;
                    if (*abort_flag) break;
                    uint8_t *dst = ring_x + s * kGXSlot;
                    mbar_arrive_expect_tx(&xfull[s], xbytes);
                    tma_load_2d(dst, &p.xmap, kc * kGK, t0, &xfull[s]);
                    if (f32x) tma_load_2d(dst + kGN * 128, &p.xmap, kc * kGK + 32, t0, &xfull[s]);
                    x_issued = gs + 1;
                }
            }
            __syncwarp();
        }
        if (warp == 2) {
            if (lane == 0) {
                const int nb = n_k / spb;
                for (int b = 0; b < nb; ++b) {
                    const int gb = wblk0 + b, ws = gb % kGWDepth;
                    if (gb >= kGWDepth && !*abort_flag && !mbar_wait(&wempty[ws], ((gb / kGWDepth) - 1) & 1)) *abort_flag = 1;
                    if (*abort_flag) break;
                    // box column: the unit's 16-byte-aligned first byte (in elements of the map),
                    // or the stage's first value for float rows
                    int x0;
                    if (sg.w_type == SQMIX_Q4_K) x0 = 144 * b;
                    else if (sg.w_type == SQMIX_Q6_K) x0 = (210 * b) & ~15;
                    else if (sg.w_type == SQMIX_Q8_0) x0 = 136 * b;  // 16-bit elements
                    else x0 = 64 * b;
                    mbar_arrive_expect_tx(&wfull[ws], static_cast<uint32_t>(sg.box_rows * wbytes));
                    tma_load_2d(ring_w + ws * kGWSlot, &sg.wmap, x0, m0, &wfull[ws]);
                    w_issued = gb + 1;
                }
            }
            __syncwarp();
        }
        wblk0 += n_k / spb;
        // epilogue: warps 0-3 (tensor-memory lanes 32 warp ..)
        if (warp < 4) {
            if (!mbar_wait(done, done_phase & 1)) *abort_flag = 1;
            tc::fence_after();
            const int row = m0 + 32 * warp + lane;
            if (!*abort_flag) {
#pragma unroll 1
                for (int c0 = 0; c0 < kGN; c0 += 32) {
                    uint32_t v[32];
                    tc::ld32(tmem + (static_cast<uint32_t>(32 * warp) << 16) + c0, v);
                    if (row < sg.n_out)
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            const int t = t0 + c0 + i;
                            if (t < p.n_tok) sg.y[static_cast<int64_t>(t) * sg.y_stride + row] = __uint_as_float(v[i]);
                        }
                }
            }
            tc::fence_before();
        }
        ++done_phase;
        // the accumulator is free for the next item once the epilogue has read it
        __syncthreads();
        tc::fence_after();
        if (*abort_flag) {
            ok = false;
            break;
        }
    }
    if (!ok && threadIdx.x == 0 && p.status) atomicOr(p.status, 1u);
    if (!ok && warp == 2 && lane == 0)
        for (int g = w_issued > kGWDepth ? w_issued - kGWDepth : 0; g < w_issued; ++g)
            if (!mbar_wait(&wfull[g % kGWDepth], (g / kGWDepth) & 1)) break;
    if (!ok && warp == 1 && lane == 0) {
        // never exit with a tensor-map load still writing into shared memory: wait (bounded)
        // for the last requests (earlier ones were consumed before their slots were reused)
        for (int g = x_issued > kGStages ? x_issued - kGStages : 0; g < x_issued; ++g)
            if (!mbar_wait(&xfull[g % kGStages], (g / kGStages) & 1)) break;
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    if (warp == 0) tc::tmem_dealloc(tmem, kGTmemCols);
}

// cuTensorMapEncodeTiled from the driver (no link-time dependency on libcuda)
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    });
    return fn;
}

}  // namespace

// Output tiles (items) of the prefill GEMM for a validated group; 0 when the form cannot
// take this x (rows not 16-byte aligned, or no tensor-map encoder).
int mul_mat_gemm_tiles(const sqmix_mul_mat_args *args, int n) {
    const sqmix_mul_mat_args &a0 = args[0];
    const int64_t elt = a0.x_dtype == SQMIX_F32 ? 4 : 2;
    if (((reinterpret_cast<uintptr_t>(a0.x) | static_cast<uintptr_t>(a0.x_stride * elt)) & 15) != 0 || !tensor_map_encoder())
        return 0;
    int m = 0;
    for (int i = 0; i < n; ++i) m += static_cast<int>((args[i].n_out + kGM - 1) / kGM);
    return m * ((a0.n_tokens + kGN - 1) / kGN);
}

// Launches the prefill GEMM for a validated group (every entry sharing x, which
// mul_mat_gemm_tiles accepted).
int mul_mat_gemm_launch(const sqmix_mul_mat_args *args, int n, cudaStream_t st) {
    GemmParams p = {};
    const sqmix_mul_mat_args &a0 = args[0];
    p.n_in = static_cast<int>(a0.n_in);
    p.n_tok = a0.n_tokens;
    p.t_tiles = (a0.n_tokens + kGN - 1) / kGN;
    p.x_dtype = a0.x_dtype;
    p.status = a0.status;
    {
        const int64_t elt = a0.x_dtype == SQMIX_F32 ? 4 : 2;
        const PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
        if (!enc) return cuda_status(cudaErrorNotSupported, "mul_mat gemm tensor map encoder");
        // (the weight maps below use the same encoder)
        const cuuint64_t dims[2] = {static_cast<cuuint64_t>(a0.n_in), static_cast<cuuint64_t>(a0.n_tokens)};
        const cuuint64_t strides[1] = {static_cast<cuuint64_t>(a0.x_stride * elt)};
        const cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / elt), static_cast<cuuint32_t>(kGN)};
        const cuuint32_t es[2] = {1, 1};
        const CUtensorMapDataType dt = a0.x_dtype == SQMIX_F32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                       : a0.x_dtype == SQMIX_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                                 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
        if (enc(&p.xmap, dt, 2, const_cast<void *>(a0.x), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
            CUDA_SUCCESS)
            return cuda_status(cudaErrorInvalidValue, "mul_mat gemm tensor map of x");
    }
    const PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    for (int i = 0; i < n; ++i) {
        GemmSeg &sg = p.seg[p.n_seg++];
        {  // the weight rows as boxes of 128 rows x wbox_bytes (no swizzle; rows beyond n_out read as zeros)
            const int wt = args[i].w_type;
            const int64_t rb = args[i].w_row_bytes;
            CUtensorMapDataType dt;
            cuuint64_t dims[2];
            cuuint32_t box[2];
            if (wt == SQMIX_Q8_0) {
                dt = CU_TENSOR_MAP_DATA_TYPE_UINT16;
                dims[0] = static_cast<cuuint64_t>(rb / 2);
                box[0] = static_cast<cuuint32_t>(wbox_bytes(wt) / 2);
            } else if (wt == SQMIX_F32) {
                dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
                dims[0] = static_cast<cuuint64_t>(a0.n_in);
                box[0] = kGK;
            } else if (wt == SQMIX_F16 || wt == SQMIX_BF16) {
                dt = CU_TENSOR_MAP_DATA_TYPE_UINT16;
                dims[0] = static_cast<cuuint64_t>(a0.n_in);
                box[0] = kGK;
            } else {  // q4_K, q6_K as bytes
                dt = CU_TENSOR_MAP_DATA_TYPE_UINT8;
                dims[0] = static_cast<cuuint64_t>(rb);
                box[0] = static_cast<cuuint32_t>(wbox_bytes(wt));
            }
            dims[1] = static_cast<cuuint64_t>(args[i].n_out);
            box[1] = static_cast<cuuint32_t>(std::min<int64_t>(kGM, args[i].n_out));
            sg.box_rows = static_cast<int>(box[1]);
            const cuuint64_t strides[1] = {static_cast<cuuint64_t>(rb)};
            const cuuint32_t es[2] = {1, 1};
            if (enc(&sg.wmap, dt, 2, const_cast<void *>(args[i].w), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
                CUDA_SUCCESS)
                return cuda_status(cudaErrorInvalidValue, "mul_mat gemm tensor map of w");
        }
        sg.w = static_cast<const uint8_t *>(args[i].w);
        sg.y = args[i].y;
        sg.y_stride = args[i].y_stride;
        sg.w_type = args[i].w_type;
        sg.row_bytes = static_cast<int>(args[i].w_row_bytes);
        sg.n_out = static_cast<int>(args[i].n_out);
        sg.m_tiles = (sg.n_out + kGM - 1) / kGM;
        sg.item0 = p.n_items;
        p.n_items += sg.m_tiles * p.t_tiles;
    }
    const int sms = sqmix_device_sm_count(-1);
    if (sms <= 0) return cuda_status(cudaErrorInvalidDevice, "mul_mat device");
    static std::atomic<uint64_t> attr_devices{0};
    {
        const cudaError_t e = set_smem_once(attr_devices, mul_mat_gemm_kernel, kGSmem);
        if (e != cudaSuccess) return cuda_status(e, "mul_mat gemm smem attribute");
    }
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(std::min(p.n_items, sms));
    cfg.blockDim = dim3(kGThreads);
    cfg.dynamicSmemBytes = kGSmem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_status(cudaLaunchKernelEx(&cfg, mul_mat_gemm_kernel, p), "mul_mat gemm launch");
}

}  // namespace sqmix
