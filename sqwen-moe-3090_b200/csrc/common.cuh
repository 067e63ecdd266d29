// common.cuh -- shared device helpers for the sqmix kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "sqmix.h"

namespace sqmix {

// ----------------------------------------------------------------- errors ----
// Set by the C-ABI wrappers; read through sqmix_last_error().
void set_error(const char *fmt, ...);
int cuda_status(cudaError_t e, const char *what);

#define SQMIX_CHECK_ARG(cond, ...)          \
    do {                                    \
        if (!(cond)) {                      \
            ::sqmix::set_error(__VA_ARGS__); \
            return SQMIX_EINVAL;            \
        }                                   \
    } while (0)

// ------------------------------------------------------- element loading ----
__device__ __forceinline__ float load_act(const void *p, int64_t i, int dtype) {
    if (dtype == SQMIX_F32) return static_cast<const float *>(p)[i];
    if (dtype == SQMIX_BF16) return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
    return __half2float(static_cast<const __half *>(p)[i]);
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded device waits give up after this many nanoseconds and raise an error flag
// instead of hanging the GPU.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// --------------------------------------------------------------- mbarrier ----
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Returns false when the wait exceeded kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
    }
}

// 1-D bulk async copy global -> shared (TMA engine, no tensor map, no multicast).
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst_smem, const void *src_gmem, uint32_t bytes,
                                         uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// --------------------------------------------------------- tensor cores ------
// Legacy warp-level MMA (mma.sync) -- used where operands are produced in
// registers (in-register q4_0 dequant), see fa_decode.cu.
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                              uint32_t b1, const float (&c)[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%10,%11,%12,%13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]),
          "f"(c[2]), "f"(c[3]));
}

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t orv) {
    uint32_t r;
    // (a & mask) | orv
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(orv));
    return r;
}

__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) {
    return *reinterpret_cast<uint32_t *>(&h);
}
__device__ __forceinline__ __half2 u32_as_h2(uint32_t u) {
    return *reinterpret_cast<__half2 *>(&u);
}
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    return h2_as_u32(__floats2half2_rn(lo, hi));
}

// ---------------------------------------------------- tiled q4_0 layout ------
//
// The cache is a sequence of 16-token groups.  Group gr (tokens 16gr..16gr+15)
// holds one 2304-byte UNIT per KV head (head-minor): unit (gr, h) at byte
// (gr * 2 + h) * 2304.  A unit stores the 16 tokens x 8 blocks of that head:
// a 2048-byte nibble area (4 rows x 32 lanes x 16 bytes, row-major, so each lane's
// 16-byte load is conflict-free) followed by a 256-byte fp16 scale area.  The
// assignment of bytes to lanes follows the m16n8k16 fragment each lane consumes:
//
// K unit (QK^T, A = K tile with M = tokens):
//   nibble row i, lane L = 4g + c, word w (4 bytes at i*512 + L*16 + 4w):
//     token = g + 8*(i >> 1), block b = 4*(i & 1) + w, bytes qs_b[4c .. 4c+3]
//   scale area: token g + 8r, block b at 2048 + g*32 + r*16 + 2b
// V unit (PV, A = V^T tile with M = dims):
//   nibble row i, lane L = 4g + c, word w: block b = 2i + (w >> 1), m = w & 1,
//     beta = g + 8m; bytes = qs_b[beta] of tokens {2c, 2c+8, 2c+1, 2c+9}
//   scale area: block b, tokens {2c, 2c+1, 2c+8, 2c+9}[j] at 2048 + c*64 + 8b + 2j
//
constexpr int kUnitBytes = 2304;
constexpr int kUnitQsBytes = 2048;
constexpr int kGroupTokens = 16;
constexpr int kHeadsKV = 2;
constexpr int kGroupBytes = kUnitBytes * kHeadsKV;  // 4608 = 16 tokens * 288

// Byte offset (within the cache) of qs byte `j` (0..15) of block `b` (0..7) of
// token `t` (absolute), head `h`, for the K layout.
__host__ __device__ __forceinline__ int64_t k_qs_offset(int64_t t, int h, int b, int j) {
    const int64_t gr = t >> 4;
    const int tt = static_cast<int>(t & 15);
    const int g = tt & 7, r = tt >> 3;
    const int c = j >> 2, byte = j & 3;
    const int i = 2 * r + (b >> 2), w = b & 3;
    return (gr * kHeadsKV + h) * kUnitBytes + i * 512 + (4 * g + c) * 16 + 4 * w + byte;
}
__host__ __device__ __forceinline__ int64_t k_scale_offset(int64_t t, int h, int b) {
    const int64_t gr = t >> 4;
    const int tt = static_cast<int>(t & 15);
    const int g = tt & 7, r = tt >> 3;
    return (gr * kHeadsKV + h) * kUnitBytes + kUnitQsBytes + g * 32 + r * 16 + 2 * b;
}
// V layout: byte j (0..15) of block b of token t.
__host__ __device__ __forceinline__ int64_t v_qs_offset(int64_t t, int h, int b, int j) {
    const int64_t gr = t >> 4;
    const int tt = static_cast<int>(t & 15);
    // tokens {2c, 2c+8, 2c+1, 2c+9} -> byte position within the word
    const int hi8 = tt >> 3, lo = tt & 7;
    const int c = lo >> 1, odd = lo & 1;
    const int pos = odd * 2 + hi8;  // 2c -> 0, 2c+8 -> 1, 2c+1 -> 2, 2c+9 -> 3
    const int m = j >> 3, g = j & 7;
    const int i = b >> 1, w = ((b & 1) << 1) | m;
    return (gr * kHeadsKV + h) * kUnitBytes + i * 512 + (4 * g + c) * 16 + 4 * w + pos;
}
__host__ __device__ __forceinline__ int64_t v_scale_offset(int64_t t, int h, int b) {
    const int64_t gr = t >> 4;
    const int tt = static_cast<int>(t & 15);
    const int hi8 = tt >> 3, lo = tt & 7;
    const int c = lo >> 1, odd = lo & 1;
    const int jj = hi8 * 2 + odd;  // 2c -> 0, 2c+1 -> 1, 2c+8 -> 2, 2c+9 -> 3
    return (gr * kHeadsKV + h) * kUnitBytes + kUnitQsBytes + c * 64 + 8 * b + 2 * jj;
}

}  // namespace sqmix
