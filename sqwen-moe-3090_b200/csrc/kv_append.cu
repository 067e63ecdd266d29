// kv_append.cu -- q4_0 KV-cache append with fused partial RoPE, and the converter
// between the tiled cache layout and ggml's q4_0 row layout.
//
// Reference path replaced: KvCache::append (src/engine/kv.rs:313-399), which emits
// ggml_set_rows into the q4_0 K cache (kv.rs:367-369) and V cache (kv.rs:394-396),
// preceded by ggml_rope_multi on K (src/model/attn.rs:183-204).
#include <math.h>

#include "common.cuh"

namespace sqmix {

struct AppendParams {
    const void *k;
    const void *v;
    int dtype;
    int64_t k_st;
    int64_t v_st;
    int n_tokens;
    const int64_t *rows;
    uint8_t *k_cache;
    uint8_t *v_cache;
    int64_t capacity;
    int rope_n_rot;
    float rope_theta_scale;
    int64_t rope_pos_offset;
};

// One warp quantises one 32-element block: lane j holds element j.
// blockIdx.x = token, threadIdx.y selects (cache, head, block) = 2 * 2 * 8 = 32 warps.
__global__ void __launch_bounds__(1024) kv_append_kernel(AppendParams p) {
    const int t = blockIdx.x;
    const int wid = threadIdx.y;  // 0..31
    const int lane = threadIdx.x;
    const int is_v = wid >> 4;
    const int h = (wid >> 3) & 1;
    const int b = wid & 7;
    const int64_t row = p.rows[t];
    if (row < 0 || row >= p.capacity) return;  // the host object validates rows

    // One cos/sin table per token (the angles depend on the pair only, not on the head).
    __shared__ float2 rope_tab[128];
    if (p.rope_n_rot > 0 && wid == 0 && lane < (p.rope_n_rot >> 1))
        rope_tab[lane] = rope_cos_sin(row + p.rope_pos_offset, p.rope_theta_scale, lane);
    if (p.rope_n_rot > 64 && wid == 1 && lane + 32 < (p.rope_n_rot >> 1))
        rope_tab[lane + 32] = rope_cos_sin(row + p.rope_pos_offset, p.rope_theta_scale, lane + 32);
    if (p.rope_n_rot > 128 && wid >= 2 && wid < 4 && lane + 32 * wid < (p.rope_n_rot >> 1))
        rope_tab[lane + 32 * wid] = rope_cos_sin(row + p.rope_pos_offset, p.rope_theta_scale, lane + 32 * wid);
    __syncthreads();

    const void *src = is_v ? p.v : p.k;
    const int64_t base = t * (is_v ? p.v_st : p.k_st) + h * 256;
    const float x = kv_row_elem(src, base, b * 32 + lane, p.dtype, is_v ? 0 : p.rope_n_rot, rope_tab);
    q4_0_store_block(x, lane, is_v ? p.v_cache : p.k_cache, row, h, b, is_v);
}

// tiled <-> ggml rows.  One thread per byte of a 288-byte row.
__global__ void kv_convert_kernel(uint8_t *tiled, uint8_t *rows, int64_t row0, int64_t n_rows,
                                  int is_v, int to_rows) {
    const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (gid >= n_rows * 288) return;
    const int64_t r = gid / 288;
    const int beta = static_cast<int>(gid % 288);
    const int h = beta / 144;
    const int blk = (beta % 144) / 18;
    const int off = beta % 18;
    const int64_t t = row0 + r;
    int64_t toff;
    if (off < 2) {
        toff = (is_v ? v_scale_offset(t, h, blk) : k_scale_offset(t, h, blk)) + off;
    } else {
        const int j = off - 2;
        toff = is_v ? v_qs_offset(t, h, blk, j) : k_qs_offset(t, h, blk, j);
    }
    if (to_rows)
        rows[gid] = tiled[toff];
    else
        tiled[toff] = rows[gid];
}

}  // namespace sqmix

using namespace sqmix;

extern "C" size_t sqmix_kv_cache_bytes(int64_t capacity) {
    if (capacity <= 0) return 0;
    return static_cast<size_t>(capacity) * 288;
}

extern "C" int sqmix_kv_append_q4_0(const sqmix_kv_append_args *a, sqmix_stream_t stream) {
    SQMIX_CHECK_ARG(a != nullptr, "kv_append: null args");
    SQMIX_CHECK_ARG(a->k && a->v && a->rows && a->k_cache && a->v_cache,
                    "kv_append: null pointer argument");
    SQMIX_CHECK_ARG(a->dtype == SQMIX_F32 || a->dtype == SQMIX_F16 || a->dtype == SQMIX_BF16,
                    "kv_append: unsupported dtype %d", a->dtype);
    SQMIX_CHECK_ARG(a->n_tokens >= 1 && a->n_tokens <= (1 << 20), "kv_append: n_tokens=%d",
                    a->n_tokens);
    SQMIX_CHECK_ARG(a->capacity > 0 && a->capacity % SQMIX_KV_PAD == 0,
                    "kv_append: capacity %lld must be a positive multiple of %d",
                    (long long)a->capacity, SQMIX_KV_PAD);
    SQMIX_CHECK_ARG(a->k_stride_tok >= 512 && a->v_stride_tok >= 512,
                    "kv_append: token strides must cover 2 heads x 256");
    SQMIX_CHECK_ARG(a->rope_n_rot >= 0 && a->rope_n_rot <= 256 && a->rope_n_rot % 2 == 0,
                    "kv_append: rope_n_rot=%d", a->rope_n_rot);
    SQMIX_CHECK_ARG(a->rope_n_rot == 0 || a->rope_freq_base > 0.0f, "kv_append: freq_base");
    AppendParams p;
    p.k = a->k;
    p.v = a->v;
    p.dtype = a->dtype;
    p.k_st = a->k_stride_tok;
    p.v_st = a->v_stride_tok;
    p.n_tokens = a->n_tokens;
    p.rows = a->rows;
    p.k_cache = static_cast<uint8_t *>(a->k_cache);
    p.v_cache = static_cast<uint8_t *>(a->v_cache);
    p.capacity = a->capacity;
    p.rope_n_rot = a->rope_n_rot;
    p.rope_pos_offset = a->rope_pos_offset;
    p.rope_theta_scale =
        a->rope_n_rot > 0 ? powf(a->rope_freq_base, -2.0f / static_cast<float>(a->rope_n_rot)) : 1.0f;
    dim3 block(32, 32);
    kv_append_kernel<<<a->n_tokens, block, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p);
    return cuda_status(cudaGetLastError(), "kv_append launch");
}

extern "C" int sqmix_kv_convert_rows(void *tiled_cache, void *rows_buf, int64_t capacity,
                                     int64_t row0, int64_t n_rows, int32_t which,
                                     int32_t to_rows, sqmix_stream_t stream) {
    SQMIX_CHECK_ARG(tiled_cache && rows_buf, "kv_convert_rows: null pointer");
    SQMIX_CHECK_ARG(capacity > 0 && capacity % SQMIX_KV_PAD == 0, "kv_convert_rows: capacity");
    SQMIX_CHECK_ARG(row0 >= 0 && n_rows >= 0 && row0 + n_rows <= capacity,
                    "kv_convert_rows: rows [%lld, %lld) outside capacity %lld", (long long)row0,
                    (long long)(row0 + n_rows), (long long)capacity);
    SQMIX_CHECK_ARG(which == 0 || which == 1, "kv_convert_rows: which must be 0 (K) or 1 (V)");
    if (n_rows == 0) return SQMIX_OK;
    const int64_t n = n_rows * 288;
    const int threads = 256;
    const int64_t blocks = (n + threads - 1) / threads;
    kv_convert_kernel<<<static_cast<unsigned>(blocks), threads, 0,
                        reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<uint8_t *>(tiled_cache), static_cast<uint8_t *>(rows_buf), row0, n_rows, which,
        to_rows);
    return cuda_status(cudaGetLastError(), "kv_convert launch");
}
