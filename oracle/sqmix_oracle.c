/*
 * sqmix_oracle.c -- CPU restatement of the ggml nodes on sqwen's attention-mixer path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity oracle and the timed CPU
 * baseline.  Only tests/, __graft_entry__.smoke() and bench.py's CPU legs may load
 * it; the CUDA library never links or calls it.
 *
 * The reference (sqwen, a Rust crate) does not contain this arithmetic: it calls an
 * un-vendored ggml / ggml-cpu / ggml-cuda (llama.cpp, pinned in
 * src/backend/ffi.rs:1 as commit ed7ac35e1, "0.7.0-dev build 1218" in README.md:104).
 * Each routine below restates the published behaviour of one node, citing the
 * reference file:line that fixes it.
 *
 * Parity pins:
 *   - q4_0 quantize/dequantize: PINNED bit-exactly against gguf-py 0.19.0
 *     (gguf/quants.py class Q4_0), a numpy restatement of ggml's
 *     quantize_row_q4_0 that ships in this image (fixtures in tests/golden/).
 *   - RoPE, attention and the gated delta rule: pinned only by the reference's
 *     own restatements and invariants (tests/attn_test.rs:148-359,
 *     tests/gdn_test.rs:186-378, tests/gdn_prod_dim_test.rs:245-326).  There are no
 *     golden vectors for these nodes anywhere in the reference: parity with ggml's
 *     exact FA/GDN rounding is UNPINNED.
 *
 * Build: oracle/Makefile (gcc -O2 -fopenmp -ffp-contract=off; contraction must stay
 * off so x*id + 8.5f rounds twice, exactly as quantize_row_q4_0 does).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define QK4_0 32

/* ---------------------------------------------------------------- fp16 ---- */

/* IEEE binary16 <- binary32, round-to-nearest-even (what ggml's
 * GGML_FP32_TO_FP16 / F16C and numpy's astype(float16) both do). */
uint16_t oracle_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t absx = x & 0x7fffffffu;
    if (absx >= 0x7f800000u) { /* inf or nan */
        return (uint16_t)(sign | 0x7c00u | (absx > 0x7f800000u ? 0x200u : 0u));
    }
    if (absx >= 0x477ff000u) { /* rounds to >= 65520 -> inf */
        return (uint16_t)(sign | 0x7c00u);
    }
    if (absx < 0x38800000u) { /* result is subnormal (or zero) in fp16 */
        if (absx < 0x33000000u) return (uint16_t)sign; /* < 2^-25: rounds to 0 */
        uint32_t mant = (absx & 0x7fffffu) | 0x800000u;
        int e = (int)(absx >> 23);                    /* biased exp, 102..112 */
        int shift = 126 - e;                          /* 14..24 */
        uint32_t q = mant >> shift;
        uint32_t rem = mant & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    /* normal */
    uint32_t e = (absx >> 23) - 127 + 15;
    uint32_t mant = absx & 0x7fffffu;
    uint32_t q = (e << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++; /* may carry into exp */
    return (uint16_t)(sign | q);
}

float oracle_f16_to_f32(uint16_t h) {
    /* tests/kernel_verify.rs:253-268 and tests/attn_test.rs:231-255 decode the same way */
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu;
    uint32_t m = h & 0x3ffu;
    uint32_t x;
    if (e == 0) {
        if (m == 0) {
            x = sign;
        } else { /* subnormal: normalise */
            int sh = 0;
            while (!(m & 0x400u)) { m <<= 1; sh++; }
            m &= 0x3ffu;
            x = sign | ((uint32_t)(127 - 15 + 1 - sh) << 23) | (m << 13);
        }
    } else if (e == 31) {
        x = sign | 0x7f800000u | (m << 13);
    } else {
        x = sign | ((e - 15 + 127) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

/* ---------------------------------------------------------------- q4_0 ---- */

/*
 * One 32-element block -> 18 bytes {fp16 d; u8 qs[16]}.
 * Restates ggml quantize_row_q4_0_ref, whose observable behaviour the reference
 * documents at tests/attn_test.rs:781-833 (d = max/-8 of the signed value of largest
 * magnitude; grid [-8d, 7d]) and tests/kernel_verify.rs:270-292 (element j in the
 * low nibble of qs[j], element j+16 in the high nibble).  Ties on |x| keep the first
 * index (strict '<' compare), id = 1/d from the UNROUNDED d (0 when d == 0), the
 * nibble is min(15, trunc(x*id + 8.5f)), and d is stored as fp16 (RNE).
 */
static void quantize_block_q4_0(const float *x, uint8_t *blk) {
    float amax = 0.0f, max = 0.0f;
    for (int j = 0; j < QK4_0; j++) {
        const float v = x[j];
        if (amax < fabsf(v)) {
            amax = fabsf(v);
            max = v;
        }
    }
    const float d = max / -8;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    const uint16_t dh = oracle_f32_to_f16(d);
    blk[0] = (uint8_t)(dh & 0xff);
    blk[1] = (uint8_t)(dh >> 8);
    for (int j = 0; j < QK4_0 / 2; j++) {
        const float x0 = x[j] * id;
        const float x1 = x[QK4_0 / 2 + j] * id;
        int q0 = (int)(x0 + 8.5f); /* C conversion truncates toward zero */
        int q1 = (int)(x1 + 8.5f);
        if (q0 > 15) q0 = 15;
        if (q1 > 15) q1 = 15;
        if (q0 < 0) q0 = 0;
        if (q1 < 0) q1 = 0;
        blk[2 + j] = (uint8_t)(q0 | (q1 << 4));
    }
}

/* ggml_quantize_chunk(GGML_TYPE_Q4_0, ...) as called at tests/attn_test.rs:210-229. */
void oracle_q4_0_quantize_rows(const float *x, int64_t nrows, int64_t n_per_row, uint8_t *out) {
    const int64_t nb = n_per_row / QK4_0;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < nrows; r++) {
        for (int64_t b = 0; b < nb; b++) {
            quantize_block_q4_0(x + r * n_per_row + b * QK4_0, out + (r * nb + b) * 18);
        }
    }
}

/* dequantize_row_q4_0: tests/kernel_verify.rs:270-292, tests/attn_test.rs:257-276. */
void oracle_q4_0_dequantize_rows(const uint8_t *in, int64_t nrows, int64_t n_per_row, float *out) {
    const int64_t nb = n_per_row / QK4_0;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < nrows; r++) {
        for (int64_t b = 0; b < nb; b++) {
            const uint8_t *blk = in + (r * nb + b) * 18;
            const float d = oracle_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
            float *y = out + r * n_per_row + b * QK4_0;
            for (int j = 0; j < QK4_0 / 2; j++) {
                y[j] = (float)((blk[2 + j] & 0x0f) - 8) * d;
                y[j + QK4_0 / 2] = (float)((blk[2 + j] >> 4) - 8) * d;
            }
        }
    }
}

/* ---------------------------------------------------------------- rope ---- */

/*
 * ggml_rope_multi, mode IMROPE (attn.rs:183-204), restated after the reference's own
 * restatement tests/attn_test.rs:148-208: theta starts at the position of the
 * matching stream and is multiplied by theta_scale = base^(-2/n_rot) once per pair
 * (repeated multiplication, not pow); pair i rotates dims (i, i + n_rot/2).  The
 * stream of pair i is picked by its sector (i mod sum(sections)).  x is
 * [n_tokens][n_head][head_dim] (dim fastest), pos is i32 [4*n_tokens] laid out
 * t/h/w/e (graph.rs:457-467 writes the same absolute position into all four).
 */
void oracle_rope_imrope(float *x, int64_t n_tokens, int64_t n_head, int64_t head_dim,
                        const int32_t *pos, const int32_t sections[4], float freq_base,
                        int32_t n_rot) {
    const int n_dims = n_rot;
    const float theta_scale = powf(freq_base, -2.0f / (float)n_dims);
    const int sect_dims = sections[0] + sections[1] + sections[2] + sections[3];
    float *cache = (float *)malloc(sizeof(float) * (size_t)n_dims);
    for (int64_t t = 0; t < n_tokens; t++) {
        float th_t = (float)pos[t];
        float th_h = (float)pos[t + n_tokens];
        float th_w = (float)pos[t + 2 * n_tokens];
        float th_e = (float)pos[t + 3 * n_tokens];
        for (int i0 = 0; i0 < n_dims; i0 += 2) {
            const int sector = (i0 / 2) % sect_dims;
            float theta;
            if (sector % 3 == 1 && sector < 3 * sections[1]) theta = th_h;
            else if (sector % 3 == 2 && sector < 3 * sections[2]) theta = th_w;
            else if (sector % 3 == 0 && sector < 3 * sections[0]) theta = th_t;
            else theta = th_e;
            cache[i0] = cosf(theta);
            cache[i0 + 1] = sinf(theta);
            th_t *= theta_scale;
            th_w *= theta_scale;
            th_h *= theta_scale;
            th_e *= theta_scale;
        }
        for (int64_t h = 0; h < n_head; h++) {
            float *a = x + (t * n_head + h) * head_dim;
            for (int i0 = 0; i0 < n_dims; i0 += 2) {
                const int ic = i0 / 2;
                const float c = cache[i0], s = cache[i0 + 1];
                const float x0 = a[ic];
                const float x1 = a[ic + n_dims / 2];
                a[ic] = x0 * c - x1 * s;
                a[ic + n_dims / 2] = x0 * s + x1 * c;
            }
        }
    }
    free(cache);
}

/* Text-only positions (graph.rs:457-467): all four streams equal p0 + t. */
void oracle_rope_text(float *x, int64_t n_tokens, int64_t n_head, int64_t head_dim,
                      int64_t pos0, float freq_base, int32_t n_rot) {
    int32_t *pos = (int32_t *)malloc(sizeof(int32_t) * 4 * (size_t)n_tokens);
    for (int s = 0; s < 4; s++)
        for (int64_t t = 0; t < n_tokens; t++) pos[s * n_tokens + t] = (int32_t)(pos0 + t);
    /* Sections only choose which stream a pair reads; with equal streams any split
     * summing to n_rot/2 gives the same angles.  qwen35moe uses [11,11,10,0]
     * (tests/gdn_prod_dim_test.rs:35-37). */
    int32_t sec[4] = {n_rot / 2, 0, 0, 0};
    oracle_rope_imrope(x, n_tokens, n_head, head_dim, pos, sec, freq_base, n_rot);
    free(pos);
}

/* ----------------------------------------------------------- attention ---- */

/*
 * ggml_flash_attn_ext as used at attn.rs:238-249 (+ the gate at attn.rs:282-283),
 * restated after tests/attn_test.rs:285-346:
 *   out[t][h][:] = sigmoid(gate[t][h][:]) * sum_j softmax_j(scale * <q[t][h], k[j][h/G]>) v[j][h/G]
 * with block GQA (G = n_head / n_head_kv, attn_test.rs:306-312) and the causal rule of
 * graph.rs:553-559: key j is visible to query t iff j <= q_pos0 + t (and j < n_kv).
 * k/v are the DEQUANTISED cache rows [n_kv][n_head_kv][D].  Accumulation in double;
 * lse (nullable) receives ln(sum_j exp(scale*s_j)) per (t, h).
 */
void oracle_attn(const float *q, const float *k, const float *v, const float *gate,
                 int64_t n_q, int64_t n_head, int64_t n_head_kv, int64_t head_dim,
                 int64_t n_kv, int64_t q_pos0, float scale, float *out, float *lse) {
    const int64_t G = n_head / n_head_kv;
    const int64_t D = head_dim;
#pragma omp parallel
    {
        double *sc = (double *)malloc(sizeof(double) * (size_t)(n_kv > 0 ? n_kv : 1));
        double *acc = (double *)malloc(sizeof(double) * (size_t)D);
#pragma omp for schedule(dynamic, 1) collapse(2)
        for (int64_t t = 0; t < n_q; t++) {
            for (int64_t h = 0; h < n_head; h++) {
                const int64_t hk = h / G;
                const float *qr = q + (t * n_head + h) * D;
                int64_t lim = q_pos0 + t + 1;
                if (lim > n_kv) lim = n_kv;
                double mx = -INFINITY;
                for (int64_t j = 0; j < lim; j++) {
                    const float *kr = k + (j * n_head_kv + hk) * D;
                    double s = 0.0;
                    for (int64_t d = 0; d < D; d++) s += (double)qr[d] * (double)kr[d];
                    s *= (double)scale;
                    sc[j] = s;
                    if (s > mx) mx = s;
                }
                double l = 0.0;
                for (int64_t d = 0; d < D; d++) acc[d] = 0.0;
                for (int64_t j = 0; j < lim; j++) {
                    const double p = exp(sc[j] - mx);
                    l += p;
                    const float *vr = v + (j * n_head_kv + hk) * D;
                    for (int64_t d = 0; d < D; d++) acc[d] += p * (double)vr[d];
                }
                float *o = out + (t * n_head + h) * D;
                for (int64_t d = 0; d < D; d++) {
                    double y = lim > 0 ? acc[d] / l : 0.0;
                    if (gate) {
                        const double gv = (double)gate[(t * n_head + h) * D + d];
                        y *= 1.0 / (1.0 + exp(-gv));
                    }
                    o[d] = (float)y;
                }
                if (lse) lse[t * n_head + h] = lim > 0 ? (float)(mx + log(l)) : -INFINITY;
            }
        }
        free(sc);
        free(acc);
    }
}

/* ----------------------------------------------------------------- gdn ---- */

/*
 * GDN q/k L2 norm, gdn.rs:126-142: scale(rms_norm(x, eps/n), 1/sqrt(n)) == x/||x||.
 * ggml's rms_norm sums squares in double (ggml_float) and scales in float.
 */
void oracle_l2norm_rows(float *x, int64_t nrows, int64_t n, float eps) {
    for (int64_t r = 0; r < nrows; r++) {
        float *a = x + r * n;
        double sum = 0.0;
        for (int64_t i = 0; i < n; i++) sum += (double)a[i] * (double)a[i];
        const float mean = (float)(sum / (double)n);
        const float s = 1.0f / sqrtf(mean + eps / (float)n);
        const float s2 = 1.0f / sqrtf((float)n);
        for (int64_t i = 0; i < n; i++) a[i] = (a[i] * s) * s2;
    }
}

/*
 * ggml_gated_delta_net (gdn.rs:489-500), per value head hv, per token t
 * (gdn.rs:9-24):
 *     S <- S * exp(g_t)
 *     delta = (v_t - S^T k_t) * beta_t
 *     S <- S + k_t delta^T
 *     o_t = (S^T q_t) / sqrt(d)
 * with q/k head hv % H_k (tiled broadcast, gdn.rs:438-439).
 *
 * Layouts (this build's choice; the reference's tests are layout-agnostic):
 *   q, k  [T][H_k][d]; v, out [T][H_v][d]; g, beta [T][H_v]
 *   state [H_v][d (value j)][d (key i)]   -- S[i][j] stored at (hv*d + j)*d + i
 *   snaps [n_snap][H_v][d][d]: slot s = state after T - s tokens
 *         (gdn.rs:484-538, tests/gdn_prod_dim_test.rs:245-292), slot 0 = final.
 * Columns j are independent, which is what the OpenMP loop (and the CUDA kernels)
 * exploit.  The column is held in float (ggml keeps the state in f32); dot products
 * accumulate in double.
 */
void oracle_gdn(const float *q, const float *k, const float *v, const float *g,
                const float *beta, const float *state_in, int64_t T, int64_t H_k,
                int64_t H_v, int64_t d, int64_t n_snap, float *out, float *snaps) {
    const float inv_sqrt_d = 1.0f / sqrtf((float)d);
#pragma omp parallel
    {
        float *col = (float *)malloc(sizeof(float) * (size_t)d);
#pragma omp for schedule(static) collapse(2)
        for (int64_t hv = 0; hv < H_v; hv++) {
            for (int64_t j = 0; j < d; j++) {
                const int64_t hk = hv % H_k;
                memcpy(col, state_in + (hv * d + j) * d, sizeof(float) * (size_t)d);
                for (int64_t t = 0; t < T; t++) {
                    const float *kt = k + (t * H_k + hk) * d;
                    const float *qt = q + (t * H_k + hk) * d;
                    const float decay = expf(g[t * H_v + hv]);
                    double kv = 0.0;
                    for (int64_t i = 0; i < d; i++) {
                        col[i] *= decay;
                        kv += (double)col[i] * (double)kt[i];
                    }
                    const float delta =
                        (v[(t * H_v + hv) * d + j] - (float)kv) * beta[t * H_v + hv];
                    double o = 0.0;
                    for (int64_t i = 0; i < d; i++) {
                        col[i] += kt[i] * delta;
                        o += (double)col[i] * (double)qt[i];
                    }
                    out[(t * H_v + hv) * d + j] = (float)o * inv_sqrt_d;
                    const int64_t s = T - 1 - t;
                    if (snaps && s < n_snap)
                        memcpy(snaps + ((s * H_v + hv) * d + j) * d, col,
                               sizeof(float) * (size_t)d);
                }
            }
        }
        free(col);
    }
}

/* ------------------------------------------------------ gdn front end ---- */

/*
 * ggml_ssm_conv, as the reference's own kernel test states it
 * (tests/kernel_verify.rs:840-853):
 *     out[t][c] = sum_{k < K} sx[c][t + k] * w[c][k]
 * sx [C][K-1+T] (ggml [K-1+T, C]), w [C][K] (ggml [K, C]), out [T][C] (ggml [C, T]);
 * float accumulation in tap order.
 */
void oracle_ssm_conv(const float *sx, int64_t C, int64_t T, int64_t K, const float *w, float *out) {
    const int64_t ncs = K - 1 + T;
    for (int64_t t = 0; t < T; t++)
        for (int64_t c = 0; c < C; c++) {
            float s = 0.0f;
            for (int64_t k = 0; k < K; k++) s += sx[c * ncs + t + k] * w[c * K + k];
            out[t * C + c] = s;
        }
}

/* ggml_silu: x / (1 + exp(-x))  (tests/kernel_verify.rs:989). */
static float silu_f(float x) { return x / (1.0f + expf(-x)); }

/*
 * The GDN front end of build_gdn_layer for one sequence (gdn.rs:290-441):
 *   conv_input = concat(history plane `sel` [C][K-1], x^T)      (gdn.rs:353-356)
 *   y = silu(ssm_conv(conv_input, w))                           (gdn.rs:358-360)
 *   q, k = channels [0, n_qk/2), [n_qk/2, n_qk) L2-normalised per head of d
 *                                                                (gdn.rs:436-441)
 * and the conv-history writeback of gdn_step (graph.rs:913-961): with n_snap == 1
 * plane 0 <- conv_input rows [T, T+K-1); otherwise slot s < n_snap <- rows
 * [max(T-s, 0), +K-1) ("s tokens back").  Every slot is computed from the input
 * history and x before any plane is written.
 *   x [T][C]; state [n_planes][C][K-1]; out [T][C].
 */
void oracle_gdn_conv(const float *x, int64_t T, int64_t C, int64_t K, const float *w, float *state,
                     int64_t n_planes, int64_t sel, int64_t n_snap, int64_t n_qk, int64_t d, float eps,
                     float *out) {
    const int64_t ncs = K - 1 + T;
    float *sx = (float *)malloc(sizeof(float) * (size_t)(C * ncs));
    for (int64_t c = 0; c < C; c++) {
        for (int64_t r = 0; r < K - 1; r++) sx[c * ncs + r] = state[(sel * C + c) * (K - 1) + r];
        for (int64_t t = 0; t < T; t++) sx[c * ncs + K - 1 + t] = x[t * C + c];
    }
    oracle_ssm_conv(sx, C, T, K, w, out);
    for (int64_t i = 0; i < T * C; i++) out[i] = silu_f(out[i]);
    for (int64_t t = 0; t < T; t++)
        if (n_qk > 0) oracle_l2norm_rows(out + t * C, n_qk / d, d, eps);
    (void)n_planes;
    for (int64_t s = 0; s < n_snap; s++) {
        int64_t r0 = T - s;
        if (r0 < 0) r0 = 0;
        for (int64_t c = 0; c < C; c++)
            for (int64_t r = 0; r < K - 1; r++) state[(s * C + c) * (K - 1) + r] = sx[c * ncs + r0 + r];
    }
    free(sx);
}

/*
 * ggml_rms_norm over rows of n (sum of squares in double, as ggml-cpu's ggml_float;
 * y = x * (1/sqrtf(mean + eps))), then optionally * w[i] (per-head RMS norm of Q/K,
 * attn.rs:66-84) and * silu(z[i]) (norm_gated, gdn.rs:150-181: rms_norm(x) * w, then
 * * silu(z)).  w and z may be NULL.  w_stride: elements between the weight rows of
 * consecutive rows' heads (0 = one shared [n] weight); rows of w cycle with period
 * w_period rows (the head index).
 */
void oracle_rms_norm_rows(const float *x, int64_t nrows, int64_t n, float eps, const float *w,
                          int64_t w_stride, int64_t w_period, const float *z, float *out) {
    for (int64_t r = 0; r < nrows; r++) {
        const float *a = x + r * n;
        double sum = 0.0;
        for (int64_t i = 0; i < n; i++) sum += (double)a[i] * (double)a[i];
        const float mean = (float)(sum / (double)n);
        const float scale = 1.0f / sqrtf(mean + eps);
        const float *wr = w ? w + (w_period > 0 ? r % w_period : 0) * w_stride : NULL;
        for (int64_t i = 0; i < n; i++) {
            float y = a[i] * scale;
            if (wr) y = y * wr[i];
            if (z) y = y * silu_f(z[r * n + i]);
            out[r * n + i] = y;
        }
    }
}

/* Thread control for the timed CPU baseline. */
int oracle_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
    return omp_get_max_threads();
#else
    (void)n;
    return 1;
#endif
}

/* ---------------------------------------------------------- projections ---- */
/* ggml_mul_mat(w, x) as sqwen builds the mixer projections (attn.rs:127-129 QG / K / V,
 * attn.rs:285 W_o; gdn.rs:264-276 qkv / z / beta / alpha, gdn.rs:577 out): w is
 * [n_in, n_out] (n_out rows of n_in elements in a ggml block format), x [n_in, T],
 * y[t][o] = sum_i W[o][i] x[t][i].  The weight formats (ggml type ids of
 * src/backend/ffi.rs:44-101), restated from their published block layouts and pinned
 * bit-exactly against gguf-py 0.19.0's dequantizers (gguf/quants.py Q8_0, Q4_K, Q6_K):
 *   Q8_0 (8):  34 bytes per 32 values: f16 d, 32 x int8 q;          w = d q
 *   Q4_K (12): 144 bytes per 256: f16 d, f16 dmin, 12 bytes of 6-bit sub-block scales
 *              and mins (8 sub-blocks of 32), 128 bytes of nibbles (bytes 32k..32k+31:
 *              sub-block 2k in the low nibbles, 2k+1 in the high); w = d sc q - dmin m
 *   Q6_K (14): 210 bytes per 256: ql[128] (low 4 bits), qh[64] (high 2 bits), int8
 *              scales[16] (one per 16 values), f16 d;               w = d sc (q - 32)
 *   F32 (0), F16 (1), BF16 (30): plain elements. */
#define ORACLE_QK_K 256

static void q4k_scale_min(int j, const uint8_t *s, int *sc, int *m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
        *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

/* bytes of one row of n values, or 0 for an unsupported type / length */
int64_t oracle_row_bytes(int type, int64_t n) {
    switch (type) {
        case 0: return 4 * n;
        case 1: case 30: return 2 * n;
        case 8: return n % 32 ? 0 : n / 32 * 34;
        case 12: return n % ORACLE_QK_K ? 0 : n / ORACLE_QK_K * 144;
        case 14: return n % ORACLE_QK_K ? 0 : n / ORACLE_QK_K * 210;
        default: return 0;
    }
}

/* one row of n values -> f32; returns 0, or -1 for an unsupported type */
int oracle_dequant_row(const uint8_t *row, int type, int64_t n, float *out) {
    if (oracle_row_bytes(type, n) == 0) return -1;
    if (type == 0) {
        memcpy(out, row, (size_t)n * 4);
    } else if (type == 1) {
        for (int64_t i = 0; i < n; i++) out[i] = oracle_f16_to_f32((uint16_t)(row[2 * i] | (row[2 * i + 1] << 8)));
    } else if (type == 30) {
        for (int64_t i = 0; i < n; i++) {
            const uint32_t u = (uint32_t)(row[2 * i] | (row[2 * i + 1] << 8)) << 16;
            memcpy(&out[i], &u, 4);
        }
    } else if (type == 8) {
        for (int64_t b = 0; b < n / 32; b++) {
            const uint8_t *blk = row + 34 * b;
            const float d = oracle_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
            for (int i = 0; i < 32; i++) out[32 * b + i] = d * (float)(int8_t)blk[2 + i];
        }
    } else if (type == 12) {
        for (int64_t b = 0; b < n / ORACLE_QK_K; b++) {
            const uint8_t *blk = row + 144 * b;
            const float d = oracle_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
            const float dmin = oracle_f16_to_f32((uint16_t)(blk[2] | (blk[3] << 8)));
            const uint8_t *qs = blk + 16;
            for (int j = 0; j < 8; j++) {
                int sc, m;
                q4k_scale_min(j, blk + 4, &sc, &m);
                const float ds = d * (float)sc, dm = dmin * (float)m;
                for (int l = 0; l < 32; l++) {
                    const int q = (qs[32 * (j >> 1) + l] >> (4 * (j & 1))) & 0xF;
                    out[ORACLE_QK_K * b + 32 * j + l] = ds * (float)q - dm;
                }
            }
        }
    } else {  /* 14: Q6_K */
        for (int64_t b = 0; b < n / ORACLE_QK_K; b++) {
            const uint8_t *blk = row + 210 * b;
            const uint8_t *ql = blk, *qh = blk + 128;
            const int8_t *sc = (const int8_t *)(blk + 192);
            const float d = oracle_f16_to_f32((uint16_t)(blk[208] | (blk[209] << 8)));
            for (int e = 0; e < ORACLE_QK_K; e++) {
                const int half = e / 128, r = e % 128, k = r / 32, l = r % 32;
                const int lo = (ql[64 * half + 32 * (k & 1) + l] >> (4 * (k >> 1))) & 0xF;
                const int hi = (qh[32 * half + l] >> (2 * k)) & 3;
                const int q = (lo | (hi << 4)) - 32;
                out[ORACLE_QK_K * b + e] = (d * (float)sc[8 * half + 2 * k + l / 16]) * (float)q;
            }
        }
    }
    return 0;
}

/* y[t * y_stride + o] = sum_i W[o][i] x[t * x_stride + i] (double accumulation of the
 * dequantised f32 weights); returns -1 for an unsupported type / length */
int oracle_mul_mat(const uint8_t *w, int type, int64_t row_bytes, int64_t n_in, int64_t n_out, const float *x,
                   int64_t x_stride, int n_tokens, float *y, int64_t y_stride) {
    if (oracle_row_bytes(type, n_in) == 0) return -1;
    int bad = 0;
#pragma omp parallel
    {
        float *wr = (float *)malloc((size_t)n_in * sizeof(float));
#pragma omp for
        for (int64_t o = 0; o < n_out; o++) {
            if (!wr || oracle_dequant_row(w + o * row_bytes, type, n_in, wr) != 0) {
                bad = 1;
                continue;
            }
            for (int t = 0; t < n_tokens; t++) {
                double acc = 0.0;
                for (int64_t i = 0; i < n_in; i++) acc += (double)wr[i] * (double)x[t * x_stride + i];
                y[t * y_stride + o] = (float)acc;
            }
        }
        free(wr);
    }
    return bad ? -1 : 0;
}
