// fa_decode.cu -- split-KV FlashAttention decode over the tiled q4_0 KV cache.
//
// Replaces ggml_flash_attn_ext (src/model/attn.rs:238-249; the op's contract is
// restated at src/backend/ffi.rs:363-377) for 1 or 2 query tokens (decode, MTP
// verify), plus the sigmoid output gate of attn.rs:282-283 (fused in the merge).
//
// Design (per CTA = one split of the key range):
//   * lane 0 of warp 0 streams 64-token tiles of K and V (18 KiB each) with 1-D
//     TMA bulk copies into a 4-stage shared-memory ring (mbarrier full/empty);
//   * warps 0..7 (warp w handles KV head w/4 and 16-token group w%4 of
//     each tile) dequantise q4_0 nibbles straight into mma.m16n8k16 A-fragments
//     (no dequantised tile is ever written to shared memory), compute
//     S^T = K Q^T with M = 16 tokens x N = 8 query heads (GQA packing: no padding
//     at n_q = 1), apply the per-block K scale in fp32, run an online softmax with
//     warp shuffles, transpose P with movmatrix, fold the per-block V scale into P
//     and accumulate O^T = V^T P^T;
//   * the 4 warps of a KV head merge through shared memory and the CTA writes one
//     (O, m, l) partial; fa_merge_kernel combines the splits (log-sum-exp merge),
//     applies sigmoid(gate) and writes out / lse.
// Keys are never read beyond min(n_kv, q_pos0 + n_q): the causal limit of
// graph.rs:553-559 is applied implicitly, so no mask tensor exists.
#include <math.h>

#include "common.cuh"

namespace sqmix {

constexpr int kFaStages = 4;
constexpr int kFaTileGroups = 4;                           // 64 tokens per stage
constexpr int kFaTileBytes = kFaTileGroups * kGroupBytes;  // 18432 per cache
constexpr int kFaConsumerWarps = 8;
constexpr int kFaThreads = kFaConsumerWarps * 32;
constexpr int kFaWsHeader = 256;  // error word + reserved

struct FaDecodeParams {
    const void *q;
    int q_dtype;
    int64_t q_st;
    int64_t q_sh;
    const uint8_t *k_cache;
    const uint8_t *v_cache;
    const int64_t *n_kv;
    const int64_t *q_pos0;
    int64_t capacity;  // rows in each cache: device-side n_kv is clamped to it
    float c;  // scale * log2(e)
    int rope_n_rot;
    float rope_theta_scale;
    int64_t rope_pos_offset;
    float *part_o;   // [splits][nq][16][256]
    float *part_ml;  // [splits][nq][16][2]
    uint32_t *err;
};

template <int NQ>
struct FaSmem {
    static constexpr int kStageBytes = 2 * kFaTileBytes;
    static constexpr int kRingBytes = kFaStages * kStageBytes;             // 147456
    static constexpr int kQBytes = NQ * 16 * 256 * 4;                       // f32 staging
    static constexpr int kRedOBytes = kFaConsumerWarps * NQ * 8 * 256 * 4;  // reuses the ring
    static_assert(kRedOBytes <= kRingBytes, "reduction buffer must fit in the ring");
    // n_q = 2 keeps the Q^T fragments in shared memory ([kvh][qi][b][s][lane] uint2):
    // in registers they push the kernel past 224 registers and into spills.
    static constexpr bool kQfSmem = NQ >= 2;
    static constexpr int kQfBytes = kQfSmem ? 2 * NQ * 8 * 2 * 32 * 8 : 0;
    static constexpr int kQfOffset = kRingBytes + kQBytes;
    static constexpr int kBarOffset = kQfOffset + kQfBytes;
    static constexpr int kRedMlOffset = kBarOffset + 128;
    static constexpr int kTotal = kRedMlOffset + kFaConsumerWarps * NQ * 8 * 2 * 4;
};

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Nibble-pair extraction.  With w = 4 bytes {b0, b1, b2, b3}:
//   lo(w)   = {b0 & 15, b2 & 15} - 8          (exact in f16)
//   hi16(w) = 16 * ({b0 >> 4, b2 >> 4} - 8)   (exact; the x16 is undone elsewhere)
__device__ __forceinline__ uint32_t nib_lo(uint32_t w) {
    const __half2 v = u32_as_h2(lop3_and_or(w, 0x000F000Fu, 0x64006400u));
    return h2_as_u32(__hsub2(v, __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408))));
}
__device__ __forceinline__ uint32_t nib_hi16(uint32_t w) {
    const __half2 v = u32_as_h2(lop3_and_or(w, 0x00F000F0u, 0x64006400u));
    return h2_as_u32(__hsub2(v, __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480))));
}

template <int NQ>
__global__ void __launch_bounds__(kFaThreads, 1) fa_decode_kernel(FaDecodeParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    using L = FaSmem<NQ>;
    uint8_t *ring = smem;
    float *q_s = reinterpret_cast<float *>(smem + L::kRingBytes);
    uint64_t *full_bar = reinterpret_cast<uint64_t *>(smem + L::kBarOffset);
    uint64_t *empty_bar = full_bar + kFaStages;
    float *red_ml = reinterpret_cast<float *>(smem + L::kRedMlOffset);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    // ---- work range: a contiguous run of 16-token groups ---------------------
    int64_t n_kv = *p.n_kv;
    if (n_kv > p.capacity) {
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(p.err, 8u);
        n_kv = p.capacity;
    }
    const int64_t q_pos0 = *p.q_pos0;
    int64_t n_keys = q_pos0 + NQ;  // causal: query NQ-1 sees keys <= q_pos0 + NQ - 1
    if (n_keys > n_kv) n_keys = n_kv;
    if (n_keys < 0) n_keys = 0;
    const int64_t n_groups = (n_keys + kGroupTokens - 1) / kGroupTokens;
    const int64_t g_begin = (static_cast<int64_t>(blockIdx.x) * n_groups) / gridDim.x;
    const int64_t g_end = (static_cast<int64_t>(blockIdx.x + 1) * n_groups) / gridDim.x;
    const int n_tiles = static_cast<int>((g_end - g_begin + kFaTileGroups - 1) / kFaTileGroups);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kFaStages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], kFaConsumerWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();

    // Lane 0 of warp 0 doubles as the TMA producer (a separate producer warp would
    // put 3 warps on one SM sub-partition and cap every thread at 168 registers).
    const bool producer = threadIdx.x == 0;
    auto issue = [&](int it) {
        const int s = it % kFaStages;
        const int64_t gr0 = g_begin + static_cast<int64_t>(it) * kFaTileGroups;
        int64_t ng = g_end - gr0;
        if (ng > kFaTileGroups) ng = kFaTileGroups;
        const uint32_t bytes = static_cast<uint32_t>(ng) * kGroupBytes;
        mbar_arrive_expect_tx(&full_bar[s], 2 * bytes);
        uint8_t *dst = ring + s * L::kStageBytes;
        bulk_g2s(dst, p.k_cache + gr0 * kGroupBytes, bytes, &full_bar[s]);
        bulk_g2s(dst + kFaTileBytes, p.v_cache + gr0 * kGroupBytes, bytes, &full_bar[s]);
    };
    if (producer)
        for (int it = 0; it < n_tiles && it < kFaStages; ++it) issue(it);

    // ================= consumers =================
    const int kvh = warp >> 2;  // KV head
    const int u = warp & 3;     // group within the tile
    const int g = lane >> 2;
    const int c = lane & 3;

    // ---- stage Q (f32) with RoPE, then build the B fragments ------------------
    for (int i = threadIdx.x; i < NQ * 16 * 256; i += kFaConsumerWarps * 32) {
        const int qi = i / (16 * 256);
        const int h = (i / 256) & 15;
        const int d = i & 255;
        q_s[i] = load_act(p.q, qi * p.q_st + h * p.q_sh + d, p.q_dtype);
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kFaConsumerWarps * 32));
    if (p.rope_n_rot > 0) {
        const int half = p.rope_n_rot >> 1;
        for (int i = threadIdx.x; i < NQ * 16 * half; i += kFaConsumerWarps * 32) {
            const int qi = i / (16 * half);
            const int h = (i / half) & 15;
            const int pi = i % half;
            float th = static_cast<float>(static_cast<int32_t>(q_pos0 + qi + p.rope_pos_offset));
            for (int k = 0; k < pi; ++k) th = __fmul_rn(th, p.rope_theta_scale);
            float sn, cs;
            sincosf(th, &sn, &cs);
            float *row = q_s + (qi * 16 + h) * 256;
            const float x0 = row[pi], x1 = row[pi + half];
            row[pi] = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
            row[pi + half] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
        }
        asm volatile("bar.sync 1, %0;" ::"n"(kFaConsumerWarps * 32));
    }
    // B fragment of Q^T for block b, k-slice s: k-slot kappa of slice s maps to
    // dim 32b + (kappa < 8 ? 4(kappa/2) + 2(kappa%2) : 16 + 4((kappa-8)/2) + 2(kappa%2)) + s;
    // lane (g, c) supplies head 8*kvh + g, k-slots {2c, 2c+1} and {2c+8, 2c+9}.
    constexpr int kQfN = L::kQfSmem ? 1 : NQ;  // register copy unused when in smem
    uint32_t qf[kQfN][8][2][2];
    uint2 *qf_s = reinterpret_cast<uint2 *>(smem + L::kQfOffset);
#pragma unroll
    for (int qi = 0; qi < NQ; ++qi) {
        const float *row = q_s + (qi * 16 + kvh * 8 + g) * 256;
#pragma unroll
        for (int b = 0; b < 8; ++b) {
#pragma unroll
            for (int s = 0; s < 2; ++s) {
                const int d0 = 32 * b + 4 * c + s;
                const uint32_t lo = pack_half2(row[d0], row[d0 + 2]);
                const uint32_t hi = pack_half2(row[d0 + 16] * 0.0625f, row[d0 + 18] * 0.0625f);
                if constexpr (L::kQfSmem) {
                    if (u == 0) qf_s[(((kvh * NQ + qi) * 8 + b) * 2 + s) * 32 + lane] = make_uint2(lo, hi);
                } else {
                    qf[qi][b][0 + s][0] = lo;
                    qf[qi][b][0 + s][1] = hi;
                }
            }
        }
    }
    if constexpr (L::kQfSmem) asm volatile("bar.sync 1, %0;" ::"n"(kFaConsumerWarps * 32));

    float o[NQ][8][2][4];
    float m_run[NQ][2], l_run[NQ][2];
#pragma unroll
    for (int qi = 0; qi < NQ; ++qi) {
        m_run[qi][0] = m_run[qi][1] = -INFINITY;
        l_run[qi][0] = l_run[qi][1] = 0.f;
#pragma unroll
        for (int b = 0; b < 8; ++b)
#pragma unroll
            for (int m = 0; m < 2; ++m)
#pragma unroll
                for (int r = 0; r < 4; ++r) o[qi][b][m][r] = 0.f;
    }
    const float zero4[4] = {0.f, 0.f, 0.f, 0.f};
    bool ok = true;

    for (int it = 0; it < n_tiles; ++it) {
        const int s = it % kFaStages;
        if (!mbar_wait(&full_bar[s], (it / kFaStages) & 1)) {
            ok = false;
            break;
        }
        const int64_t gr = g_begin + static_cast<int64_t>(it) * kFaTileGroups + u;
        const int64_t tok0 = gr * kGroupTokens;
        if (gr < g_end && tok0 < n_keys) {
            const uint8_t *kunit = ring + s * L::kStageBytes + (u * 2 + kvh) * kUnitBytes;
            const uint8_t *vunit = kunit + kFaTileBytes;

            // ---------------- S^T = K Q^T ----------------
            const uint4 *kq4 = reinterpret_cast<const uint4 *>(kunit);
            uint32_t kw[16];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint4 x = kq4[i * 32 + lane];
                kw[4 * i + 0] = x.x;
                kw[4 * i + 1] = x.y;
                kw[4 * i + 2] = x.z;
                kw[4 * i + 3] = x.w;
            }
            const uint4 *ksc = reinterpret_cast<const uint4 *>(kunit + kUnitQsBytes + g * 32);
            const uint4 kd0 = ksc[0], kd1 = ksc[1];
            const uint32_t kdl[4] = {kd0.x, kd0.y, kd0.z, kd0.w};
            const uint32_t kdh[4] = {kd1.x, kd1.y, kd1.z, kd1.w};

            float sc[NQ][4];
#pragma unroll
            for (int qi = 0; qi < NQ; ++qi)
#pragma unroll
                for (int r = 0; r < 4; ++r) sc[qi][r] = 0.f;
#pragma unroll
            for (int b = 0; b < 8; ++b) {
                const uint32_t wl = kw[(b >> 2) * 4 + (b & 3)];      // token g
                const uint32_t wh = kw[8 + (b >> 2) * 4 + (b & 3)];  // token g+8
                const uint32_t wl8 = wl >> 8, wh8 = wh >> 8;
                const uint32_t a0[4] = {nib_lo(wl), nib_lo(wh), nib_hi16(wl), nib_hi16(wh)};
                const uint32_t a1[4] = {nib_lo(wl8), nib_lo(wh8), nib_hi16(wl8), nib_hi16(wh8)};
                const __half2 dl2 = u32_as_h2(kdl[b >> 1]);
                const __half2 dh2 = u32_as_h2(kdh[b >> 1]);
                const float dl = (b & 1) ? __high2float(dl2) : __low2float(dl2);
                const float dh = (b & 1) ? __high2float(dh2) : __low2float(dh2);
#pragma unroll
                for (int qi = 0; qi < NQ; ++qi) {
                    uint32_t b00, b01, b10, b11;
                    if constexpr (L::kQfSmem) {
                        const uint2 *qb = qf_s + ((kvh * NQ + qi) * 8 + b) * 2 * 32 + lane;
                        const uint2 x0 = qb[0], x1 = qb[32];
                        b00 = x0.x;
                        b01 = x0.y;
                        b10 = x1.x;
                        b11 = x1.y;
                    } else {
                        b00 = qf[qi][b][0][0];
                        b01 = qf[qi][b][0][1];
                        b10 = qf[qi][b][1][0];
                        b11 = qf[qi][b][1][1];
                    }
                    float acc[4];
                    mma_f16_16816(acc, a0, b00, b01, zero4);
                    mma_f16_16816(acc, a1, b10, b11, acc);
                    sc[qi][0] = fmaf(dl, acc[0], sc[qi][0]);
                    sc[qi][1] = fmaf(dl, acc[1], sc[qi][1]);
                    sc[qi][2] = fmaf(dh, acc[2], sc[qi][2]);
                    sc[qi][3] = fmaf(dh, acc[3], sc[qi][3]);
                }
            }

            // ---------------- online softmax ----------------
            const int64_t t_lo = tok0 + g, t_hi = tok0 + g + 8;
            uint32_t pb[NQ][2];
#pragma unroll
            for (int qi = 0; qi < NQ; ++qi) {
                int64_t lim = q_pos0 + qi;  // inclusive
                if (lim > n_kv - 1) lim = n_kv - 1;
                const bool vlo = t_lo <= lim, vhi = t_hi <= lim;
                const float x0 = vlo ? sc[qi][0] : -INFINITY;
                const float x1 = vlo ? sc[qi][1] : -INFINITY;
                const float x2 = vhi ? sc[qi][2] : -INFINITY;
                const float x3 = vhi ? sc[qi][3] : -INFINITY;
                float mx0 = fmaxf(x0, x2), mx1 = fmaxf(x1, x3);
#pragma unroll
                for (int off = 4; off < 32; off <<= 1) {
                    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
                    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
                }
                const float mn0 = fmaxf(m_run[qi][0], mx0);
                const float mn1 = fmaxf(m_run[qi][1], mx1);
                const float al0 = (mn0 == m_run[qi][0]) ? 1.f : ex2((m_run[qi][0] - mn0) * p.c);
                const float al1 = (mn1 == m_run[qi][1]) ? 1.f : ex2((m_run[qi][1] - mn1) * p.c);
                const float p0 = vlo ? ex2((x0 - mn0) * p.c) : 0.f;
                const float p1 = vlo ? ex2((x1 - mn1) * p.c) : 0.f;
                const float p2 = vhi ? ex2((x2 - mn0) * p.c) : 0.f;
                const float p3 = vhi ? ex2((x3 - mn1) * p.c) : 0.f;
                l_run[qi][0] = fmaf(l_run[qi][0], al0, p0 + p2);
                l_run[qi][1] = fmaf(l_run[qi][1], al1, p1 + p3);
                m_run[qi][0] = mn0;
                m_run[qi][1] = mn1;
                if (__any_sync(0xffffffffu, al0 != 1.f || al1 != 1.f)) {
#pragma unroll
                    for (int b = 0; b < 8; ++b)
#pragma unroll
                        for (int m = 0; m < 2; ++m) {
                            o[qi][b][m][0] *= al0;
                            o[qi][b][m][1] *= al1;
                            o[qi][b][m][2] *= al0;
                            o[qi][b][m][3] *= al1;
                        }
                }
                // P^T as the B operand: transpose the two 8x8 halves of the C fragment.
                pb[qi][0] = movmatrix_trans(pack_half2(p0, p1));
                pb[qi][1] = movmatrix_trans(pack_half2(p2, p3));
            }

            // ---------------- O^T += V^T P'^T ----------------
            const uint4 *vq4 = reinterpret_cast<const uint4 *>(vunit);
            uint32_t vw[16];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint4 x = vq4[i * 32 + lane];
                vw[4 * i + 0] = x.x;
                vw[4 * i + 1] = x.y;
                vw[4 * i + 2] = x.z;
                vw[4 * i + 3] = x.w;
            }
            const uint4 *vsc = reinterpret_cast<const uint4 *>(vunit + kUnitQsBytes + c * 64);
            uint32_t vd[16];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint4 x = vsc[i];
                vd[4 * i + 0] = x.x;
                vd[4 * i + 1] = x.y;
                vd[4 * i + 2] = x.z;
                vd[4 * i + 3] = x.w;
            }
#pragma unroll
            for (int b = 0; b < 8; ++b) {
                const __half2 s0 = u32_as_h2(vd[2 * b]);      // tokens 2c, 2c+1
                const __half2 s1 = u32_as_h2(vd[2 * b + 1]);  // tokens 2c+8, 2c+9
                uint32_t pbs[NQ][2];
#pragma unroll
                for (int qi = 0; qi < NQ; ++qi) {
                    pbs[qi][0] = h2_as_u32(__hmul2(u32_as_h2(pb[qi][0]), s0));
                    pbs[qi][1] = h2_as_u32(__hmul2(u32_as_h2(pb[qi][1]), s1));
                }
#pragma unroll
                for (int m = 0; m < 2; ++m) {
                    const uint32_t w = vw[2 * b + m];
                    const uint32_t w8 = w >> 8;
                    const uint32_t a[4] = {nib_lo(w), nib_hi16(w), nib_lo(w8), nib_hi16(w8)};
#pragma unroll
                    for (int qi = 0; qi < NQ; ++qi)
                        mma_f16_16816(o[qi][b][m], a, pbs[qi][0], pbs[qi][1], o[qi][b][m]);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[s]);
        if (producer && it + kFaStages < n_tiles) {
            // Refill this stage once all 8 warps have released it.
            if (!mbar_wait(&empty_bar[s], (it / kFaStages) & 1)) {
                ok = false;
                break;
            }
            issue(it + kFaStages);
        }
    }
    if (!ok) {
        if (lane == 0) atomicOr(p.err, 4u);
        // Never leave the CTA with a bulk copy still writing into shared memory.
        if (producer) {
            const int first = n_tiles > kFaStages ? n_tiles - kFaStages : 0;
            for (int it = first; it < n_tiles; ++it)
                if (!mbar_wait(&full_bar[it % kFaStages], (it / kFaStages) & 1)) break;
        }
    }

    // ---- finish l over the 8 token rows of the fragment ------------------------
#pragma unroll
    for (int qi = 0; qi < NQ; ++qi)
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int off = 4; off < 32; off <<= 1)
                l_run[qi][j] += __shfl_xor_sync(0xffffffffu, l_run[qi][j], off);

    __syncthreads();  // ring is free: every issued tile has been consumed
    // red_o[warp][qi][head8][256]
    float *red_o = reinterpret_cast<float *>(ring);
#pragma unroll
    for (int qi = 0; qi < NQ; ++qi) {
        float *base = red_o + (static_cast<size_t>(warp) * NQ + qi) * 8 * 256;
#pragma unroll
        for (int b = 0; b < 8; ++b)
#pragma unroll
            for (int m = 0; m < 2; ++m) {
                const int d_lo = 32 * b + 8 * m + g;
                const int d_hi = d_lo + 16;
                base[(2 * c) * 256 + d_lo] = o[qi][b][m][0];
                base[(2 * c + 1) * 256 + d_lo] = o[qi][b][m][1];
                base[(2 * c) * 256 + d_hi] = o[qi][b][m][2] * 0.0625f;
                base[(2 * c + 1) * 256 + d_hi] = o[qi][b][m][3] * 0.0625f;
            }
        if (g == 0) {
            float *ml = red_ml + ((warp * NQ + qi) * 8) * 2;
            ml[(2 * c) * 2 + 0] = m_run[qi][0];
            ml[(2 * c) * 2 + 1] = l_run[qi][0];
            ml[(2 * c + 1) * 2 + 0] = m_run[qi][1];
            ml[(2 * c + 1) * 2 + 1] = l_run[qi][1];
        }
    }
    __syncthreads();

    // ---- combine the 4 warps of each KV head, write this split's partial ------
    float *po = p.part_o + static_cast<size_t>(blockIdx.x) * NQ * 16 * 256;
    float *pml = p.part_ml + static_cast<size_t>(blockIdx.x) * NQ * 16 * 2;
    for (int i = threadIdx.x; i < NQ * 2 * 8 * 256; i += kFaConsumerWarps * 32) {
        const int d = i & 255;
        const int h8 = (i >> 8) & 7;
        const int kh = (i >> 11) & 1;
        const int qi = i >> 12;
        float M = -INFINITY;
#pragma unroll
        for (int w4 = 0; w4 < 4; ++w4) M = fmaxf(M, red_ml[(((kh * 4 + w4) * NQ + qi) * 8 + h8) * 2]);
        float acc = 0.f, lsum = 0.f;
#pragma unroll
        for (int w4 = 0; w4 < 4; ++w4) {
            const int wv = kh * 4 + w4;
            const float mw = red_ml[((wv * NQ + qi) * 8 + h8) * 2];
            const float wgt = (mw == -INFINITY) ? 0.f : ex2((mw - M) * p.c);
            acc = fmaf(red_o[((static_cast<size_t>(wv) * NQ + qi) * 8 + h8) * 256 + d], wgt, acc);
            lsum = fmaf(red_ml[((wv * NQ + qi) * 8 + h8) * 2 + 1], wgt, lsum);
        }
        const int head = kh * 8 + h8;
        po[(qi * 16 + head) * 256 + d] = acc;
        if (d == 0) {
            pml[(qi * 16 + head) * 2 + 0] = M;
            pml[(qi * 16 + head) * 2 + 1] = lsum;
        }
    }
}

// out[row][d] = sigmoid(gate) * sum_s O_s exp2((m_s - M) c) / sum_s l_s exp2((m_s - M) c)
struct FaMergeParams {
    const float *part_o;
    const float *part_ml;
    int n_splits;
    int n_rows;  // n_q * 16
    const void *gate;
    int gate_dtype;
    int64_t g_st;
    int64_t g_sh;
    float c;
    float scale;
    float *out;
    float *lse;
};

__global__ void __launch_bounds__(64) fa_merge_kernel(FaMergeParams p) {
    extern __shared__ float wts[];  // [n_splits]
    __shared__ float s_M, s_L;
    const int row = blockIdx.x;
    const int d = blockIdx.y * 64 + threadIdx.x;
    if (threadIdx.x < 32) {
        float M = -INFINITY;
        for (int sidx = threadIdx.x; sidx < p.n_splits; sidx += 32)
            M = fmaxf(M, p.part_ml[(static_cast<size_t>(sidx) * p.n_rows + row) * 2]);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
        float Ls = 0.f;
        for (int sidx = threadIdx.x; sidx < p.n_splits; sidx += 32) {
            const float mw = p.part_ml[(static_cast<size_t>(sidx) * p.n_rows + row) * 2];
            const float w = (mw == -INFINITY) ? 0.f : ex2((mw - M) * p.c);
            wts[sidx] = w;
            Ls = fmaf(p.part_ml[(static_cast<size_t>(sidx) * p.n_rows + row) * 2 + 1], w, Ls);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) Ls += __shfl_xor_sync(0xffffffffu, Ls, off);
        if (threadIdx.x == 0) {
            s_M = M;
            s_L = Ls;
        }
    }
    __syncthreads();
    float acc0 = 0.f, acc1 = 0.f;
    int sidx = 0;
    for (; sidx + 1 < p.n_splits; sidx += 2) {
        acc0 = fmaf(p.part_o[(static_cast<size_t>(sidx) * p.n_rows + row) * 256 + d], wts[sidx], acc0);
        acc1 = fmaf(p.part_o[(static_cast<size_t>(sidx + 1) * p.n_rows + row) * 256 + d], wts[sidx + 1],
                    acc1);
    }
    if (sidx < p.n_splits)
        acc0 = fmaf(p.part_o[(static_cast<size_t>(sidx) * p.n_rows + row) * 256 + d], wts[sidx], acc0);
    const float Lsum = s_L;
    float y = Lsum > 0.f ? (acc0 + acc1) / Lsum : 0.f;
    if (p.gate) {
        const int qi = row >> 4, h = row & 15;
        const float gv = load_act(p.gate, qi * p.g_st + h * p.g_sh + d, p.gate_dtype);
        y *= 1.0f / (1.0f + expf(-gv));
    }
    p.out[static_cast<size_t>(row) * 256 + d] = y;
    if (p.lse && blockIdx.y == 0 && threadIdx.x == 0)
        p.lse[row] = Lsum > 0.f ? s_M * p.scale + logf(Lsum) : -INFINITY;
}

// Merge of normalised partials across GPUs: O = sum_p O_p e^(lse_p - L).
__global__ void __launch_bounds__(256) merge_lse_kernel(int n_parts, int n_rows, const float *o_parts,
                                                         const float *lse_parts, const float *gate,
                                                         float *out, float *lse_out) {
    const int row = blockIdx.x;
    const int d = threadIdx.x;
    float M = -INFINITY;
    for (int i = 0; i < n_parts; ++i) M = fmaxf(M, lse_parts[static_cast<size_t>(i) * n_rows + row]);
    float Ls = 0.f, acc = 0.f;
    for (int i = 0; i < n_parts; ++i) {
        const float l = lse_parts[static_cast<size_t>(i) * n_rows + row];
        const float w = (l == -INFINITY) ? 0.f : expf(l - M);
        Ls += w;
        acc = fmaf(o_parts[(static_cast<size_t>(i) * n_rows + row) * 256 + d], w, acc);
    }
    float y = Ls > 0.f ? acc / Ls : 0.f;
    if (gate) y *= 1.0f / (1.0f + expf(-gate[static_cast<size_t>(row) * 256 + d]));
    out[static_cast<size_t>(row) * 256 + d] = y;
    if (lse_out && d == 0) lse_out[row] = Ls > 0.f ? M + logf(Ls) : -INFINITY;
}

}  // namespace sqmix

using namespace sqmix;

static size_t fa_ws_layout(int32_t n_splits, int32_t n_q, size_t *off_ml, size_t *off_o) {
    const size_t ml = static_cast<size_t>(n_splits) * n_q * 16 * 2 * sizeof(float);
    const size_t ob = static_cast<size_t>(n_splits) * n_q * 16 * 256 * sizeof(float);
    *off_ml = kFaWsHeader;
    *off_o = kFaWsHeader + ((ml + 255) / 256) * 256;
    return *off_o + ob;
}

extern "C" size_t sqmix_fa_workspace_bytes(int32_t n_splits, int32_t n_q) {
    if (n_splits <= 0) n_splits = sqmix_device_sm_count(-1);
    if (n_q < 1) n_q = 1;
    size_t a, b;
    return fa_ws_layout(n_splits, n_q, &a, &b);
}

template <int NQ>
static int launch_fa(const sqmix_fa_args *a, int n_splits, cudaStream_t st) {
    static bool attr_set = false;
    using L = FaSmem<NQ>;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(fa_decode_kernel<NQ>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal);
        if (e != cudaSuccess) return cuda_status(e, "fa_decode smem attribute");
        attr_set = true;
    }
    size_t off_ml, off_o;
    fa_ws_layout(n_splits, NQ, &off_ml, &off_o);
    uint8_t *ws = static_cast<uint8_t *>(a->workspace);
    FaDecodeParams p;
    p.q = a->q;
    p.q_dtype = a->q_dtype;
    p.q_st = a->q_stride_tok;
    p.q_sh = a->q_stride_head;
    p.k_cache = static_cast<const uint8_t *>(a->k_cache);
    p.v_cache = static_cast<const uint8_t *>(a->v_cache);
    p.n_kv = a->n_kv;
    p.q_pos0 = a->q_pos0;
    p.capacity = a->capacity;
    p.c = a->scale * 1.4426950408889634f;
    p.rope_n_rot = a->rope_n_rot;
    p.rope_pos_offset = a->rope_pos_offset;
    p.rope_theta_scale =
        a->rope_n_rot > 0 ? powf(a->rope_freq_base, -2.0f / static_cast<float>(a->rope_n_rot)) : 1.0f;
    p.part_o = reinterpret_cast<float *>(ws + off_o);
    p.part_ml = reinterpret_cast<float *>(ws + off_ml);
    p.err = reinterpret_cast<uint32_t *>(ws);
    fa_decode_kernel<NQ><<<n_splits, kFaThreads, L::kTotal, st>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_status(e, "fa_decode launch");

    FaMergeParams mp;
    mp.part_o = p.part_o;
    mp.part_ml = p.part_ml;
    mp.n_splits = n_splits;
    mp.n_rows = NQ * 16;
    mp.gate = a->gate;
    mp.gate_dtype = a->gate_dtype;
    mp.g_st = a->gate_stride_tok;
    mp.g_sh = a->gate_stride_head;
    mp.c = p.c;
    mp.scale = a->scale;
    mp.out = a->out;
    mp.lse = a->lse;
    dim3 grid(NQ * 16, 4);
    fa_merge_kernel<<<grid, 64, n_splits * sizeof(float), st>>>(mp);
    return cuda_status(cudaGetLastError(), "fa_merge launch");
}

extern "C" int sqmix_fa_decode(const sqmix_fa_args *a, sqmix_stream_t stream) {
    SQMIX_CHECK_ARG(a != nullptr, "fa_decode: null args");
    SQMIX_CHECK_ARG(a->q && a->k_cache && a->v_cache && a->n_kv && a->q_pos0 && a->out &&
                        a->workspace,
                    "fa_decode: null pointer argument");
    SQMIX_CHECK_ARG(a->n_q == 1 || a->n_q == 2, "fa_decode: n_q=%d (supported: 1, 2)", a->n_q);
    SQMIX_CHECK_ARG(a->q_dtype == SQMIX_F32 || a->q_dtype == SQMIX_F16 || a->q_dtype == SQMIX_BF16,
                    "fa_decode: q dtype %d", a->q_dtype);
    SQMIX_CHECK_ARG(!a->gate || a->gate_dtype == SQMIX_F32 || a->gate_dtype == SQMIX_F16 ||
                        a->gate_dtype == SQMIX_BF16,
                    "fa_decode: gate dtype %d", a->gate_dtype);
    SQMIX_CHECK_ARG(a->capacity > 0 && a->capacity % SQMIX_KV_PAD == 0, "fa_decode: capacity");
    SQMIX_CHECK_ARG((reinterpret_cast<uintptr_t>(a->k_cache) & 15) == 0 &&
                        (reinterpret_cast<uintptr_t>(a->v_cache) & 15) == 0,
                    "fa_decode: caches must be 16-byte aligned");
    SQMIX_CHECK_ARG(a->scale > 0.f, "fa_decode: scale must be positive");
    SQMIX_CHECK_ARG(a->rope_n_rot >= 0 && a->rope_n_rot <= 256 && a->rope_n_rot % 2 == 0 &&
                        (a->rope_n_rot == 0 || a->rope_freq_base > 0.f),
                    "fa_decode: rope parameters");
    int n_splits = a->n_splits > 0 ? a->n_splits : sqmix_device_sm_count(-1);
    SQMIX_CHECK_ARG(n_splits >= 1 && n_splits <= 4096, "fa_decode: n_splits=%d", n_splits);
    const size_t need = sqmix_fa_workspace_bytes(n_splits, a->n_q);
    if (a->workspace_bytes < need) {
        set_error("fa_decode: workspace %zu bytes < %zu needed", a->workspace_bytes, need);
        return SQMIX_ENOSPC;
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    return a->n_q == 1 ? launch_fa<1>(a, n_splits, st) : launch_fa<2>(a, n_splits, st);
}

extern "C" int sqmix_attn_merge_lse(int32_t n_parts, int32_t n_rows, const float *o_parts,
                                    const float *lse_parts, const float *gate, float *out,
                                    float *lse_out, sqmix_stream_t stream) {
    SQMIX_CHECK_ARG(n_parts >= 1 && n_rows >= 1, "merge_lse: n_parts=%d n_rows=%d", n_parts, n_rows);
    SQMIX_CHECK_ARG(o_parts && lse_parts && out, "merge_lse: null pointer");
    merge_lse_kernel<<<n_rows, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        n_parts, n_rows, o_parts, lse_parts, gate, out, lse_out);
    return cuda_status(cudaGetLastError(), "merge_lse launch");
}
