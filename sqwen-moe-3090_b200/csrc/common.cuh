// common.cuh -- shared device helpers for the sqmix kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "sqmix.h"

namespace sqmix {

// ----------------------------------------------------------------- errors ----
// Set by the C-ABI wrappers; read through sqmix_last_error().
void set_error(const char *fmt, ...);
int cuda_status(cudaError_t e, const char *what);

// Function attributes such as cudaFuncAttributeMaxDynamicSharedMemorySize are per
// device: a launcher records the devices it has set them on, one bit per ordinal.
// Returns the current device's bit (0 if it cannot be represented: set every time).
inline uint64_t current_device_bit() {
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d > 63) return 0;
    return 1ull << d;
}
// Sets a dynamic shared memory limit on `kernel` once per device (mask: the caller's
// per-kernel record).
template <typename K>
inline cudaError_t set_smem_once(std::atomic<uint64_t> &mask, K kernel, int bytes) {
    const uint64_t bit = current_device_bit();
    if (bit && (mask.load() & bit)) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) mask.fetch_or(bit);
    return e;
}

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

// ---------------------------------------------------------------- clusters ----
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// shared::cluster address of the variable at shared::cta address `addr` in CTA `rank`
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
// arrival (release at cluster scope) on an mbarrier given by shared::cluster address
__device__ __forceinline__ void mbar_arrive_cl(uint32_t bar_cl) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cl) : "memory");
}
// arrival with the default semantics (release at CTA scope) on an mbarrier given by
// shared::cluster address: the form the tensor-core pipelines of a CTA pair use for the
// per-stage handshakes (it does not wait for the thread's loads still in flight)
__device__ __forceinline__ void mbar_arrive_remote(uint32_t bar_cl) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar_cl) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cl(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// wait with acquire at cluster scope (arrivals from the peer CTA); false after kWaitLimitNs
__device__ __forceinline__ bool mbar_wait_cl(uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait_cl(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait_cl(bar, parity)) return true;
        if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
    }
}
__device__ __forceinline__ void st_cluster_v4(uint32_t addr_cl, int4 v) {
    asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr_cl), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w)
                 : "memory");
}
// every thread of both CTAs of the cluster (all warps converged)
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
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
// 2^x (MUFU approximation; 2^-inf = 0)
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    return h2_as_u32(__floats2half2_rn(lo, hi));
}

// ------------------------------------------------------- GDN gate epilogue ----
// beta = sigmoid(b) and g = softplus(alpha + dt_bias) * ssm_a (gdn.rs:268-287:
// ggml_sigmoid, ggml_add, ggml_softplus, ggml_mul); softplus(x) = log1p(e^x), x itself
// above 20 (e^x no longer changes 1 + e^x in f32 there).
__device__ __forceinline__ float gdn_softplus(float x) { return x > 20.0f ? x : log1pf(expf(x)); }
__device__ __forceinline__ void gdn_gates(float &g, float &beta, const float *dt_bias, const float *ssm_a, int hg) {
    if (!ssm_a) return;
    g = gdn_softplus(g + (dt_bias ? dt_bias[hg] : 0.0f)) * ssm_a[hg];
    beta = 1.0f / (1.0f + expf(-beta));
}

// ------------------------------------------------------------------ RoPE ----
// Angle of rotation pair i at text position `pos`: theta = pos * scale^i with the
// power built by repeated float multiplication (as ggml-cpu builds its rope cache,
// tests/attn_test.rs:173-193); cos/sin of that float angle are evaluated in double
// after a Cody-Waite reduction modulo 2*pi (2*pi split into a 34-bit head, exact for
// multiples k < 2^19, plus a double tail) and rounded to float.  The results are
// within an ulp of libm's cosf/sinf, and the reduction keeps positions ~1.7e5 on the
// fast path of sincos().
__device__ __forceinline__ float2 rope_cos_sin(int64_t pos, float theta_scale, int i) {
    float th = static_cast<float>(static_cast<int32_t>(pos));
    for (int k = 0; k < i; ++k) th = __fmul_rn(th, theta_scale);
    const double x = static_cast<double>(th);
    const double kq = rint(x * 0.15915494309189535);  // x / (2 pi)
    const double two_pi_hi = 6.2831853069365025;     // 2 pi truncated to 34 significant bits
    const double two_pi_lo = 2.430840202602477e-10;  // 2 pi - two_pi_hi
    const double r = __dsub_rn(__dsub_rn(x, kq * two_pi_hi), kq * two_pi_lo);
    double sd, cd;
    sincos(r, &sd, &cd);
    return make_float2(static_cast<float>(cd), static_cast<float>(sd));
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

// ------------------------------------------------------- q4_0 block store ---
// One element of a new K/V row: head h, dim `dim` of token row `base` (element
// offset of the head's first value) in `src`; K rows get the partial RoPE of
// attn.rs:183-204 (NEOX pairs (i, i + n_rot/2)) with cos/sin from `rope_tab`.
__device__ __forceinline__ float kv_row_elem(const void *src, int64_t base, int dim, int dtype,
                                             int rope_n_rot, const float2 *rope_tab) {
    float x = load_act(src, base + dim, dtype);
    if (dim < rope_n_rot) {
        const int half = rope_n_rot >> 1;
        const int i = dim < half ? dim : dim - half;
        const float partner = load_act(src, base + (dim < half ? dim + half : dim - half), dtype);
        const float2 cs = rope_tab[i];
        x = dim < half ? __fsub_rn(__fmul_rn(x, cs.x), __fmul_rn(partner, cs.y))   // x0 c - x1 s
                       : __fadd_rn(__fmul_rn(partner, cs.y), __fmul_rn(x, cs.x));  // x0 s + x1 c
    }
    return x;
}

// One warp quantises one 32-element block (lane j holds element j) of token `row`,
// head h, block b into the tiled cache.  quantize_row_q4_0 rounding: the signed value
// of largest magnitude (first index on ties) gives d = max / -8, id = 1/d (0 if d == 0),
// nibble = min(15, trunc(x * id + 8.5)), every step an IEEE single op (no contraction),
// d stored as fp16 (RNE).  Bit-exact with ggml's CPU reference for the same input.
__device__ __forceinline__ void q4_0_store_block(float x, int lane, uint8_t *cache, int64_t row, int h,
                                                 int b, bool is_v) {
    float amax = fabsf(x);
    float vmax = x;
    int idx = lane;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float oa = __shfl_xor_sync(0xffffffffu, amax, off);
        const float ov = __shfl_xor_sync(0xffffffffu, vmax, off);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, off);
        if (oa > amax || (oa == amax && oi < idx)) {
            amax = oa;
            vmax = ov;
            idx = oi;
        }
    }
    // A block whose every |x| is 0 keeps max = 0 (the reference starts from amax = max = 0).
    if (amax == 0.0f) vmax = 0.0f;
    const float d = __fdiv_rn(vmax, -8.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    int q = __float2int_rz(__fadd_rn(__fmul_rn(x, id), 8.5f));
    q = min(15, max(0, q));
    const int qhi = __shfl_down_sync(0xffffffffu, q, 16);
    if (lane < 16) {
        const uint8_t byte = static_cast<uint8_t>(q | (qhi << 4));
        cache[is_v ? v_qs_offset(row, h, b, lane) : k_qs_offset(row, h, b, lane)] = byte;
    }
    if (lane == 0)
        *reinterpret_cast<__half *>(cache + (is_v ? v_scale_offset(row, h, b) : k_scale_offset(row, h, b))) =
            __float2half_rn(d);
}

// N blocks at once (one per value of x[k], lane j holding element j of each), with the
// reductions of the blocks interleaved: the same rounding as q4_0_store_block.
// Blocks with live[k] false are skipped.
template <int N>
__device__ __forceinline__ void q4_0_store_blocks(const float (&x)[N], int lane, uint8_t *kcache, uint8_t *vcache,
                                                  const int64_t (&row)[N], const int (&h)[N], const int (&b)[N],
                                                  const bool (&is_v)[N], const bool (&live)[N]) {
    float amax[N], vmax[N];
    int idx[N];
#pragma unroll
    for (int k = 0; k < N; ++k) {
        amax[k] = fabsf(x[k]);
        vmax[k] = x[k];
        idx[k] = lane;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
        for (int k = 0; k < N; ++k) {
            const float oa = __shfl_xor_sync(0xffffffffu, amax[k], off);
            const float ov = __shfl_xor_sync(0xffffffffu, vmax[k], off);
            const int oi = __shfl_xor_sync(0xffffffffu, idx[k], off);
            if (oa > amax[k] || (oa == amax[k] && oi < idx[k])) {
                amax[k] = oa;
                vmax[k] = ov;
                idx[k] = oi;
            }
        }
    }
#pragma unroll
    for (int k = 0; k < N; ++k) {
        if (amax[k] == 0.0f) vmax[k] = 0.0f;
        const float d = __fdiv_rn(vmax[k], -8.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        int q = __float2int_rz(__fadd_rn(__fmul_rn(x[k], id), 8.5f));
        q = min(15, max(0, q));
        const int qhi = __shfl_down_sync(0xffffffffu, q, 16);
        if (!live[k]) continue;
        uint8_t *cache = is_v[k] ? vcache : kcache;
        if (lane < 16) {
            const uint8_t byte = static_cast<uint8_t>(q | (qhi << 4));
            cache[is_v[k] ? v_qs_offset(row[k], h[k], b[k], lane) : k_qs_offset(row[k], h[k], b[k], lane)] = byte;
        }
        if (lane == 0)
            *reinterpret_cast<__half *>(cache + (is_v[k] ? v_scale_offset(row[k], h[k], b[k])
                                                         : k_scale_offset(row[k], h[k], b[k]))) = __float2half_rn(d);
    }
}

}  // namespace sqmix
