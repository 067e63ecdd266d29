/*
 * cpu_ggml.c -- the timed CPU baseline: the attention-mixer nodes executed the way
 * ggml's CPU backend executes them.
 *
 * TEST INFRASTRUCTURE ONLY (the same rule as sqmix_oracle.c): only tests/,
 * __graft_entry__.smoke() and bench.py's CPU legs load it; the CUDA library never
 * links or calls it.  It is not the parity checker -- sqmix_oracle.c is (double
 * accumulation, f32 inputs).  This file restates how ggml-cpu computes the same nodes
 * in single precision, so that the CPU figure next to every GPU number is the cost
 * of the reference's own CPU algorithm rather than of the checker's.
 *
 * sqwen's attention goes through ggml_flash_attn_ext (src/backend/ffi.rs:363-377,
 * called at src/model/attn.rs:238-249) on a q4_0 K/V cache; ggml (llama.cpp
 * ed7ac35e1, src/backend/ffi.rs:1) is not vendored in the reference.  ggml-cpu's
 * flash-attention kernel, for a q4_0 K and V and an f32 Q, does per query row
 * (token t, head h; K/V head h / (n_head / n_head_kv)):
 *   - Q is converted once to K's dot-product type, q8_0 (per 32 values d = amax/127,
 *     q = round(x/d), d stored as fp16);
 *   - for each visible key j: s = scale * vec_dot_q4_0_q8_0(K_j, Q) (integer dot per
 *     32-block, times the two fp16 scales, summed in f32); online softmax with a
 *     running maximum M and sum S in f32: if s > M the accumulator is rescaled by
 *     e^(M_old - M) and the key's weight is 1, else its weight is e^(s - M);
 *   - the key's V row is dequantised to f32 and accumulated: VKQ += w * V_j;
 *   - out = VKQ / S.
 * Rows (t, h) are split across threads, as ggml splits query rows.  The causal mask
 * of graph.rs:553-559 is the visible-key bound j <= q_pos0 + t (ggml skips -inf
 * mask entries).  The output gate (attn.rs:282-283) is ggml_sigmoid + ggml_mul.
 *
 * The gated delta rule (ggml_gated_delta_net, src/model/gdn.rs:489-500, recurrence
 * gdn.rs:9-24) runs token by token in f32, split across threads by (value head,
 * value column).
 *
 * Build: oracle/Makefile compiles this file with -O3 -mavx2 -mfma (vectorised inner
 * loops, as ggml-cpu's SIMD kernels are) and links it into libsqmix_oracle.so.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

float oracle_f16_to_f32(uint16_t h);
uint16_t oracle_f32_to_f16(float f);

#define QK 32
#define BLK_BYTES 18

static float g_f16[65536];
static int g_f16_ready = 0;

static void f16_table(void) {
    if (g_f16_ready) return;
#pragma omp critical(cpu_ggml_f16)
    {
        if (!g_f16_ready) {
            for (uint32_t i = 0; i < 65536; i++) g_f16[i] = oracle_f16_to_f32((uint16_t)i);
            g_f16_ready = 1;
        }
    }
}

static inline float f16v(const uint8_t *p) { return g_f16[(uint32_t)p[0] | ((uint32_t)p[1] << 8)]; }

/* quantize_row_q8_0 of one 32-value block: d = amax / 127, q = round(x / d). */
static void q8_0_block(const float *x, int8_t *q, float *d_out) {
    float amax = 0.0f;
    for (int j = 0; j < QK; j++) {
        const float a = fabsf(x[j]);
        if (a > amax) amax = a;
    }
    const float d = amax / 127.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    for (int j = 0; j < QK; j++) q[j] = (int8_t)roundf(x[j] * id);
    *d_out = g_f16[oracle_f32_to_f16(d)]; /* the scale is stored as fp16 */
}

/* vec_dot_q4_0_q8_0 over n_blk blocks: sum_b d_x d_y sum_j (x_j - 8) y_j. */
static inline float dot_q4_0_q8_0(const uint8_t *x, const int8_t *yq, const float *yd, int n_blk) {
    float sum = 0.0f;
    for (int b = 0; b < n_blk; b++) {
        const uint8_t *blk = x + b * BLK_BYTES;
        const uint8_t *qs = blk + 2;
        const int8_t *y = yq + b * QK;
        int32_t sumi = 0;
        for (int j = 0; j < 16; j++) {
            sumi += ((int32_t)(qs[j] & 15) - 8) * (int32_t)y[j];
            sumi += ((int32_t)(qs[j] >> 4) - 8) * (int32_t)y[j + 16];
        }
        sum += (float)sumi * (f16v(blk) * yd[b]);
    }
    return sum;
}

/* dequantize_row_q4_0 of n_blk blocks into out. */
static inline void dequant_q4_0(const uint8_t *x, float *out, int n_blk) {
    for (int b = 0; b < n_blk; b++) {
        const uint8_t *blk = x + b * BLK_BYTES;
        const float d = f16v(blk);
        const uint8_t *qs = blk + 2;
        for (int j = 0; j < 16; j++) {
            out[b * QK + j] = (float)((int32_t)(qs[j] & 15) - 8) * d;
            out[b * QK + j + 16] = (float)((int32_t)(qs[j] >> 4) - 8) * d;
        }
    }
}

/*
 * Flash attention over a q4_0 cache in ggml row layout: k_rows / v_rows [n_kv] rows of
 * n_head_kv * head_dim / 32 blocks (the cache of src/engine/kv.rs:124-134, one row per
 * position); q [n_q][n_head][head_dim] f32 (already rotated); gate nullable, same
 * shape; out likewise; lse nullable [n_q][n_head] (natural log, with the scale).
 */
void cpu_fa_q4_0(const float *q, const uint8_t *k_rows, const uint8_t *v_rows, const float *gate, int64_t n_q,
                 int64_t n_head, int64_t n_head_kv, int64_t head_dim, int64_t n_kv, int64_t q_pos0, float scale,
                 float *out, float *lse) {
    f16_table();
    const int64_t G = n_head / n_head_kv;
    const int n_blk = (int)(head_dim / QK);
    const int64_t row_bytes = n_head_kv * n_blk * BLK_BYTES;
#pragma omp parallel
    {
        float *acc = (float *)malloc(sizeof(float) * (size_t)head_dim);
        float *vrow = (float *)malloc(sizeof(float) * (size_t)head_dim);
        int8_t *qq = (int8_t *)malloc((size_t)head_dim);
        float *qd = (float *)malloc(sizeof(float) * (size_t)n_blk);
#pragma omp for schedule(dynamic, 1) collapse(2)
        for (int64_t t = 0; t < n_q; t++) {
            for (int64_t h = 0; h < n_head; h++) {
                const int64_t hk = h / G;
                const float *qr = q + (t * n_head + h) * head_dim;
                for (int b = 0; b < n_blk; b++) q8_0_block(qr + b * QK, qq + b * QK, qd + b);
                int64_t lim = q_pos0 + t + 1;
                if (lim > n_kv) lim = n_kv;
                float M = -INFINITY, S = 0.0f;
                for (int64_t d = 0; d < head_dim; d++) acc[d] = 0.0f;
                for (int64_t j = 0; j < lim; j++) {
                    const uint8_t *kr = k_rows + j * row_bytes + hk * n_blk * BLK_BYTES;
                    const float s = dot_q4_0_q8_0(kr, qq, qd, n_blk) * scale;
                    float ms = 1.0f, vs = 1.0f;
                    if (s > M) {
                        const float Mold = M;
                        M = s;
                        ms = expf(Mold - M);
                        for (int64_t d = 0; d < head_dim; d++) acc[d] *= ms;
                    } else {
                        vs = expf(s - M);
                    }
                    dequant_q4_0(v_rows + j * row_bytes + hk * n_blk * BLK_BYTES, vrow, n_blk);
                    for (int64_t d = 0; d < head_dim; d++) acc[d] += vrow[d] * vs;
                    S = S * ms + vs;
                }
                float *o = out + (t * n_head + h) * head_dim;
                const float inv = S > 0.0f ? 1.0f / S : 0.0f;
                for (int64_t d = 0; d < head_dim; d++) {
                    float y = acc[d] * inv;
                    if (gate) y *= 1.0f / (1.0f + expf(-gate[(t * n_head + h) * head_dim + d]));
                    o[d] = y;
                }
                if (lse) lse[t * n_head + h] = S > 0.0f ? M + logf(S) : -INFINITY;
            }
        }
        free(acc);
        free(vrow);
        free(qq);
        free(qd);
    }
}

/*
 * Gated delta rule in f32, token by token (gdn.rs:9-24): per value head hv (q/k head
 * hv % H_k) and value column j, with the state column S[:, j] (state layout
 * [H_v][d (j)][d (i)]):  S *= e^g;  delta = (v_j - S.k) beta;  S += k delta;
 * o_j = S.q / sqrt(d).  The state is updated in place.
 */
void cpu_gdn_f32(const float *q, const float *k, const float *v, const float *g, const float *beta, float *state,
                 int64_t T, int64_t H_k, int64_t H_v, int64_t d, float *out) {
    const float inv_sqrt_d = 1.0f / sqrtf((float)d);
#pragma omp parallel for schedule(static) collapse(2)
    for (int64_t hv = 0; hv < H_v; hv++) {
        for (int64_t j = 0; j < d; j++) {
            const int64_t hk = hv % H_k;
            float *col = state + (hv * d + j) * d;
            for (int64_t t = 0; t < T; t++) {
                const float *kt = k + (t * H_k + hk) * d;
                const float *qt = q + (t * H_k + hk) * d;
                const float decay = expf(g[t * H_v + hv]);
                float kv = 0.0f;
                for (int64_t i = 0; i < d; i++) {
                    col[i] *= decay;
                    kv += col[i] * kt[i];
                }
                const float delta = (v[(t * H_v + hv) * d + j] - kv) * beta[t * H_v + hv];
                float o = 0.0f;
                for (int64_t i = 0; i < d; i++) {
                    col[i] += kt[i] * delta;
                    o += col[i] * qt[i];
                }
                out[(t * H_v + hv) * d + j] = o * inv_sqrt_d;
            }
        }
    }
}

/* ---------------------------------------------------------- projections ----
 * ggml_mul_mat(w, x) of the mixer projections (attn.rs:127-129, 285; gdn.rs:264-276,
 * 577) the way ggml-cpu runs it for quantised weights: x is quantised once per token to
 * the weight's dot-product type -- q8_K (256-value blocks: f32 d, int8 q, int16 sums of
 * 16) for q4_K / q6_K, q8_0 for q8_0 -- and every weight row is an integer dot product
 * per block, scaled in f32.  f32 / f16 / bf16 weights: f32 dot products.  Rows are
 * split across threads, as ggml splits the rows of a mul_mat. */
#define QKK 256

/* quantize_row_q8_K of one 256-value block: iscale = -127 / (the value of largest
 * magnitude), q = round(iscale x) (at most 127), d = 1 / iscale, bsums of 16 values. */
static void q8_k_block(const float *x, int8_t *q, float *d_out, int16_t *bsums) {
    float amax = 0.0f, max = 0.0f;
    for (int j = 0; j < QKK; j++) {
        const float a = fabsf(x[j]);
        if (a > amax) {
            amax = a;
            max = x[j];
        }
    }
    if (amax == 0.0f) {
        *d_out = 0.0f;
        memset(q, 0, QKK);
        memset(bsums, 0, 16 * sizeof(int16_t));
        return;
    }
    const float iscale = -127.0f / max;
    for (int j = 0; j < QKK; j++) {
        int v = (int)lrintf(iscale * x[j]);
        q[j] = (int8_t)(v > 127 ? 127 : v);
    }
    for (int j = 0; j < 16; j++) {
        int s = 0;
        for (int i = 0; i < 16; i++) s += q[16 * j + i];
        bsums[j] = (int16_t)s;
    }
    *d_out = 1.0f / iscale;
}

static void q4k_scale_min_c(int j, const uint8_t *s, int *sc, int *m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
        *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

/* vec_dot_q4_K_q8_K: d_x (d sum_j sc_j sum q4 q8) - d_x dmin sum_j m_j bsum_j */
static float dot_q4_k_q8_k(const uint8_t *w, const int8_t *yq, const float *yd, const int16_t *ys, int n_blk) {
    float sum = 0.0f;
    for (int b = 0; b < n_blk; b++) {
        const uint8_t *blk = w + 144 * b;
        const uint8_t *qs = blk + 16;
        const int8_t *y = yq + QKK * b;
        const int16_t *bs = ys + 16 * b;
        int32_t isum = 0, msum = 0;
        for (int j = 0; j < 8; j++) {
            int sc, m;
            q4k_scale_min_c(j, blk + 4, &sc, &m);
            int32_t s = 0;
            const int sh = 4 * (j & 1);
            for (int l = 0; l < 32; l++) s += ((qs[32 * (j >> 1) + l] >> sh) & 0xF) * (int32_t)y[32 * j + l];
            isum += sc * s;
            msum += m * (bs[2 * j] + bs[2 * j + 1]);
        }
        sum += yd[b] * (f16v(blk) * (float)isum - f16v(blk + 2) * (float)msum);
    }
    return sum;
}

/* vec_dot_q6_K_q8_K: d_x d sum_k sc_k sum (q6 - 32) q8 */
static float dot_q6_k_q8_k(const uint8_t *w, const int8_t *yq, const float *yd, int n_blk) {
    float sum = 0.0f;
    for (int b = 0; b < n_blk; b++) {
        const uint8_t *blk = w + 210 * b;
        const int8_t *sc = (const int8_t *)(blk + 192);
        const int8_t *y = yq + QKK * b;
        int32_t isum = 0;
        for (int k = 0; k < 16; k++) {
            int32_t s = 0;
            for (int i = 0; i < 16; i++) {
                const int e = 16 * k + i, half = e / 128, r = e % 128, qq = r / 32, l = r % 32;
                const int lo = (blk[64 * half + 32 * (qq & 1) + l] >> (4 * (qq >> 1))) & 0xF;
                const int hi = (blk[128 + 32 * half + l] >> (2 * qq)) & 3;
                s += ((lo | (hi << 4)) - 32) * (int32_t)y[e];
            }
            isum += sc[k] * s;
        }
        sum += yd[b] * f16v(blk + 208) * (float)isum;
    }
    return sum;
}

/* vec_dot_q8_0_q8_0: sum_b d_w d_x sum q_w q_x */
static float dot_q8_0_q8_0(const uint8_t *w, const int8_t *yq, const float *yd, int n_blk) {
    float sum = 0.0f;
    for (int b = 0; b < n_blk; b++) {
        const uint8_t *blk = w + 34 * b;
        const int8_t *q = (const int8_t *)(blk + 2);
        const int8_t *y = yq + QK * b;
        int32_t s = 0;
        for (int j = 0; j < QK; j++) s += (int32_t)q[j] * (int32_t)y[j];
        sum += (float)s * (f16v(blk) * yd[b]);
    }
    return sum;
}

/* y[t * n_out + o] for w_type 8 / 12 / 14 (quantised) or 0 / 1 / 30; returns -1 for an
 * unsupported type or length */
int cpu_mul_mat(const uint8_t *w, int w_type, int64_t row_bytes, int64_t n_in, int64_t n_out, const float *x,
                int n_tok, float *y) {
    f16_table();
    const int kq = w_type == 12 || w_type == 14;
    if ((kq && n_in % QKK) || (w_type == 8 && n_in % QK)) return -1;
    if (!kq && w_type != 8 && w_type != 0 && w_type != 1 && w_type != 30) return -1;
    const int64_t n_blk = kq ? n_in / QKK : n_in / QK;
    int8_t *yq = (int8_t *)malloc((size_t)n_tok * n_in);
    float *yd = (float *)malloc((size_t)n_tok * n_blk * sizeof(float));
    int16_t *ys = (int16_t *)malloc((size_t)n_tok * (n_in / 16 + 1) * sizeof(int16_t));
    if (!yq || !yd || !ys) {
        free(yq);
        free(yd);
        free(ys);
        return -1;
    }
    if (kq || w_type == 8)
        for (int t = 0; t < n_tok; t++)
            for (int64_t b = 0; b < n_blk; b++) {
                if (kq)
                    q8_k_block(x + t * n_in + QKK * b, yq + t * n_in + QKK * b, yd + t * n_blk + b,
                               ys + t * (n_in / 16) + 16 * b);
                else
                    q8_0_block(x + t * n_in + QK * b, yq + t * n_in + QK * b, yd + t * n_blk + b);
            }
#pragma omp parallel for schedule(static)
    for (int64_t o = 0; o < n_out; o++) {
        const uint8_t *wr = w + o * row_bytes;
        for (int t = 0; t < n_tok; t++) {
            float r;
            if (w_type == 12)
                r = dot_q4_k_q8_k(wr, yq + t * n_in, yd + t * n_blk, ys + t * (n_in / 16), (int)n_blk);
            else if (w_type == 14)
                r = dot_q6_k_q8_k(wr, yq + t * n_in, yd + t * n_blk, (int)n_blk);
            else if (w_type == 8)
                r = dot_q8_0_q8_0(wr, yq + t * n_in, yd + t * n_blk, (int)n_blk);
            else {
                float s = 0.0f;
                for (int64_t i = 0; i < n_in; i++) {
                    float wv;
                    if (w_type == 0) {
                        memcpy(&wv, wr + 4 * i, 4);
                    } else if (w_type == 1) {
                        wv = f16v(wr + 2 * i);
                    } else {
                        const uint32_t u = (uint32_t)(wr[2 * i] | (wr[2 * i + 1] << 8)) << 16;
                        memcpy(&wv, &u, 4);
                    }
                    s += wv * x[t * n_in + i];
                }
                r = s;
            }
            y[t * n_out + o] = r;
        }
    }
    free(yq);
    free(yd);
    free(ys);
    return 0;
}
