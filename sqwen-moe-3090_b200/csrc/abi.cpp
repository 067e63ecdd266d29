// abi.cpp -- layout table of the argument structs of sqmix.h.
//
// A binding written in another language (the Rust extern block a maintainer adds to
// sqwen's src/backend, a ctypes mirror) declares these structs a second time.  A
// field added, removed or reordered on one side only would make the library read
// past the caller's struct or read the wrong field.  sqwen guards its own ggml FFI
// the same way against header drift (src/backend/ffi.rs:516-588, sentinel enum
// values parsed from ggml.h); here the library itself reports, per struct, its size,
// its number of fields and the byte offset of each field in declaration order, so a
// binding's test can compare them with its own declaration.
#include <stddef.h>

#include "sqmix.h"

namespace {

#define OFF(S, f) offsetof(S, f)

const size_t kKvAppend[] = {
    OFF(sqmix_kv_append_args, k),           OFF(sqmix_kv_append_args, v),
    OFF(sqmix_kv_append_args, dtype),       OFF(sqmix_kv_append_args, k_stride_tok),
    OFF(sqmix_kv_append_args, v_stride_tok), OFF(sqmix_kv_append_args, n_tokens),
    OFF(sqmix_kv_append_args, rows),        OFF(sqmix_kv_append_args, k_cache),
    OFF(sqmix_kv_append_args, v_cache),     OFF(sqmix_kv_append_args, capacity),
    OFF(sqmix_kv_append_args, rope_n_rot),  OFF(sqmix_kv_append_args, rope_freq_base),
    OFF(sqmix_kv_append_args, rope_pos_offset),
};

const size_t kFa[] = {
    OFF(sqmix_fa_args, q),                OFF(sqmix_fa_args, q_dtype),
    OFF(sqmix_fa_args, q_stride_tok),     OFF(sqmix_fa_args, q_stride_head),
    OFF(sqmix_fa_args, gate),             OFF(sqmix_fa_args, gate_dtype),
    OFF(sqmix_fa_args, gate_stride_tok),  OFF(sqmix_fa_args, gate_stride_head),
    OFF(sqmix_fa_args, k_cache),          OFF(sqmix_fa_args, v_cache),
    OFF(sqmix_fa_args, capacity),         OFF(sqmix_fa_args, n_kv),
    OFF(sqmix_fa_args, q_pos0),           OFF(sqmix_fa_args, n_q),
    OFF(sqmix_fa_args, scale),            OFF(sqmix_fa_args, rope_n_rot),
    OFF(sqmix_fa_args, rope_freq_base),   OFF(sqmix_fa_args, rope_pos_offset),
    OFF(sqmix_fa_args, out),              OFF(sqmix_fa_args, lse),
    OFF(sqmix_fa_args, workspace),        OFF(sqmix_fa_args, workspace_bytes),
    OFF(sqmix_fa_args, n_splits),         OFF(sqmix_fa_args, config),
    OFF(sqmix_fa_args, k_new),            OFF(sqmix_fa_args, v_new),
    OFF(sqmix_fa_args, kv_new_dtype),     OFF(sqmix_fa_args, k_new_stride_tok),
    OFF(sqmix_fa_args, v_new_stride_tok), OFF(sqmix_fa_args, n_new),
    OFF(sqmix_fa_args, flags),            OFF(sqmix_fa_args, q_norm),
    OFF(sqmix_fa_args, k_norm),           OFF(sqmix_fa_args, norm_eps),
};

const size_t kFaBatch[] = {
    OFF(sqmix_fa_batch_args, n_seqs),          OFF(sqmix_fa_batch_args, q),
    OFF(sqmix_fa_batch_args, q_dtype),         OFF(sqmix_fa_batch_args, q_stride_seq),
    OFF(sqmix_fa_batch_args, q_stride_head),   OFF(sqmix_fa_batch_args, gate),
    OFF(sqmix_fa_batch_args, gate_dtype),      OFF(sqmix_fa_batch_args, gate_stride_seq),
    OFF(sqmix_fa_batch_args, gate_stride_head), OFF(sqmix_fa_batch_args, k_caches),
    OFF(sqmix_fa_batch_args, v_caches),        OFF(sqmix_fa_batch_args, capacities),
    OFF(sqmix_fa_batch_args, n_kv),            OFF(sqmix_fa_batch_args, q_pos0),
    OFF(sqmix_fa_batch_args, scale),           OFF(sqmix_fa_batch_args, rope_n_rot),
    OFF(sqmix_fa_batch_args, rope_freq_base),  OFF(sqmix_fa_batch_args, out),
    OFF(sqmix_fa_batch_args, lse),             OFF(sqmix_fa_batch_args, workspace),
    OFF(sqmix_fa_batch_args, workspace_bytes), OFF(sqmix_fa_batch_args, splits_per_seq),
    OFF(sqmix_fa_batch_args, k_new),           OFF(sqmix_fa_batch_args, v_new),
    OFF(sqmix_fa_batch_args, kv_new_dtype),    OFF(sqmix_fa_batch_args, new_stride_seq),
    OFF(sqmix_fa_batch_args, n_new),           OFF(sqmix_fa_batch_args, flags),
};

const size_t kPeerMerge[] = {
    OFF(sqmix_peer_merge_args, n_ranks),   OFF(sqmix_peer_merge_args, rank),
    OFF(sqmix_peer_merge_args, slot),      OFF(sqmix_peer_merge_args, n_slots),
    OFF(sqmix_peer_merge_args, rows),      OFF(sqmix_peer_merge_args, buffers),
    OFF(sqmix_peer_merge_args, o_local),   OFF(sqmix_peer_merge_args, lse_local),
    OFF(sqmix_peer_merge_args, gate),      OFF(sqmix_peer_merge_args, out),
    OFF(sqmix_peer_merge_args, lse_out),   OFF(sqmix_peer_merge_args, status),
};

const size_t kGdn[] = {
    OFF(sqmix_gdn_args, q),            OFF(sqmix_gdn_args, k),
    OFF(sqmix_gdn_args, v),            OFF(sqmix_gdn_args, dtype),
    OFF(sqmix_gdn_args, qk_stride_tok), OFF(sqmix_gdn_args, v_stride_tok),
    OFF(sqmix_gdn_args, qk_stride_seq), OFF(sqmix_gdn_args, v_stride_seq),
    OFF(sqmix_gdn_args, g),            OFF(sqmix_gdn_args, beta),
    OFF(sqmix_gdn_args, state),        OFF(sqmix_gdn_args, n_planes),
    OFF(sqmix_gdn_args, sel),          OFF(sqmix_gdn_args, n_seqs),
    OFF(sqmix_gdn_args, n_tokens),     OFF(sqmix_gdn_args, h_k),
    OFF(sqmix_gdn_args, h_v),          OFF(sqmix_gdn_args, n_snap),
    OFF(sqmix_gdn_args, l2_eps),       OFF(sqmix_gdn_args, out),
    OFF(sqmix_gdn_args, flags),        OFF(sqmix_gdn_args, h_v_offset),
    OFF(sqmix_gdn_args, dt_bias),      OFF(sqmix_gdn_args, ssm_a),
};

const size_t kGdnConv[] = {
    OFF(sqmix_gdn_conv_args, x),             OFF(sqmix_gdn_conv_args, x_dtype),
    OFF(sqmix_gdn_conv_args, x_stride_tok),  OFF(sqmix_gdn_conv_args, x_stride_seq),
    OFF(sqmix_gdn_conv_args, weight),        OFF(sqmix_gdn_conv_args, conv_state),
    OFF(sqmix_gdn_conv_args, n_planes),      OFF(sqmix_gdn_conv_args, sel),
    OFF(sqmix_gdn_conv_args, n_snap),        OFF(sqmix_gdn_conv_args, n_seqs),
    OFF(sqmix_gdn_conv_args, n_tokens),      OFF(sqmix_gdn_conv_args, channels),
    OFF(sqmix_gdn_conv_args, kernel),        OFF(sqmix_gdn_conv_args, head_dim),
    OFF(sqmix_gdn_conv_args, n_qk_channels), OFF(sqmix_gdn_conv_args, l2_eps),
    OFF(sqmix_gdn_conv_args, out),
};

const size_t kHeadNorm[] = {
    OFF(sqmix_head_norm_args, x),                  OFF(sqmix_head_norm_args, x_dtype),
    OFF(sqmix_head_norm_args, x_stride_tok),       OFF(sqmix_head_norm_args, x_stride_head),
    OFF(sqmix_head_norm_args, weight),             OFF(sqmix_head_norm_args, weight_stride_head),
    OFF(sqmix_head_norm_args, z),                  OFF(sqmix_head_norm_args, z_dtype),
    OFF(sqmix_head_norm_args, z_stride_tok),       OFF(sqmix_head_norm_args, z_stride_head),
    OFF(sqmix_head_norm_args, n_tokens),           OFF(sqmix_head_norm_args, n_heads),
    OFF(sqmix_head_norm_args, head_dim),           OFF(sqmix_head_norm_args, eps),
    OFF(sqmix_head_norm_args, out),                OFF(sqmix_head_norm_args, out_stride_tok),
    OFF(sqmix_head_norm_args, out_stride_head),
};

const size_t kGdnLayer[] = {
    OFF(sqmix_gdn_layer_args, x),              OFF(sqmix_gdn_layer_args, x_dtype),
    OFF(sqmix_gdn_layer_args, x_stride_tok),   OFF(sqmix_gdn_layer_args, x_stride_seq),
    OFF(sqmix_gdn_layer_args, conv_weight),    OFF(sqmix_gdn_layer_args, conv_state),
    OFF(sqmix_gdn_layer_args, kernel),         OFF(sqmix_gdn_layer_args, alpha),
    OFF(sqmix_gdn_layer_args, beta),           OFF(sqmix_gdn_layer_args, dt_bias),
    OFF(sqmix_gdn_layer_args, ssm_a),          OFF(sqmix_gdn_layer_args, state),
    OFF(sqmix_gdn_layer_args, n_planes),       OFF(sqmix_gdn_layer_args, sel),
    OFF(sqmix_gdn_layer_args, n_snap),         OFF(sqmix_gdn_layer_args, n_seqs),
    OFF(sqmix_gdn_layer_args, n_tokens),       OFF(sqmix_gdn_layer_args, h_k),
    OFF(sqmix_gdn_layer_args, h_v),            OFF(sqmix_gdn_layer_args, l2_eps),
    OFF(sqmix_gdn_layer_args, z),              OFF(sqmix_gdn_layer_args, z_dtype),
    OFF(sqmix_gdn_layer_args, z_stride_tok),   OFF(sqmix_gdn_layer_args, z_stride_seq),
    OFF(sqmix_gdn_layer_args, norm_weight),    OFF(sqmix_gdn_layer_args, norm_weight_stride_head),
    OFF(sqmix_gdn_layer_args, norm_eps),       OFF(sqmix_gdn_layer_args, out),
    OFF(sqmix_gdn_layer_args, flags),
};

const size_t kGgmlFaOp[] = {
    OFF(sqmix_ggml_fa_op, scale),           OFF(sqmix_ggml_fa_op, rope_n_rot),
    OFF(sqmix_ggml_fa_op, rope_freq_base),  OFF(sqmix_ggml_fa_op, rope_pos_offset),
    OFF(sqmix_ggml_fa_op, n_splits),        OFF(sqmix_ggml_fa_op, config),
    OFF(sqmix_ggml_fa_op, flags),           OFF(sqmix_ggml_fa_op, q_norm),
    OFF(sqmix_ggml_fa_op, k_norm),          OFF(sqmix_ggml_fa_op, norm_eps),
    OFF(sqmix_ggml_fa_op, workspace),       OFF(sqmix_ggml_fa_op, workspace_bytes),
    OFF(sqmix_ggml_fa_op, stream),          OFF(sqmix_ggml_fa_op, status),
};

const size_t kGgmlGdnOp[] = {
    OFF(sqmix_ggml_gdn_op, n_snap),     OFF(sqmix_ggml_gdn_op, l2_eps),
    OFF(sqmix_ggml_gdn_op, flags),      OFF(sqmix_ggml_gdn_op, h_v_offset),
    OFF(sqmix_ggml_gdn_op, dt_bias),    OFF(sqmix_ggml_gdn_op, ssm_a),
    OFF(sqmix_ggml_gdn_op, stream),     OFF(sqmix_ggml_gdn_op, status),
};

const size_t kMulMat[] = {
    OFF(sqmix_mul_mat_args, w),        OFF(sqmix_mul_mat_args, w_type),
    OFF(sqmix_mul_mat_args, w_row_bytes), OFF(sqmix_mul_mat_args, n_in),
    OFF(sqmix_mul_mat_args, n_out),    OFF(sqmix_mul_mat_args, x),
    OFF(sqmix_mul_mat_args, x_dtype),  OFF(sqmix_mul_mat_args, x_stride),
    OFF(sqmix_mul_mat_args, n_tokens), OFF(sqmix_mul_mat_args, y),
    OFF(sqmix_mul_mat_args, y_stride), OFF(sqmix_mul_mat_args, status),
};

#undef OFF

struct Entry {
    size_t size;
    const size_t *offsets;
    int32_t n_fields;
};

template <size_t N>
constexpr Entry entry(size_t size, const size_t (&offs)[N]) {
    return Entry{size, offs, static_cast<int32_t>(N)};
}

bool lookup(int32_t which, Entry *e) {
    switch (which) {
        case SQMIX_ABI_KV_APPEND_ARGS: *e = entry(sizeof(sqmix_kv_append_args), kKvAppend); return true;
        case SQMIX_ABI_FA_ARGS: *e = entry(sizeof(sqmix_fa_args), kFa); return true;
        case SQMIX_ABI_FA_BATCH_ARGS: *e = entry(sizeof(sqmix_fa_batch_args), kFaBatch); return true;
        case SQMIX_ABI_PEER_MERGE_ARGS: *e = entry(sizeof(sqmix_peer_merge_args), kPeerMerge); return true;
        case SQMIX_ABI_GDN_ARGS: *e = entry(sizeof(sqmix_gdn_args), kGdn); return true;
        case SQMIX_ABI_GDN_CONV_ARGS: *e = entry(sizeof(sqmix_gdn_conv_args), kGdnConv); return true;
        case SQMIX_ABI_HEAD_NORM_ARGS: *e = entry(sizeof(sqmix_head_norm_args), kHeadNorm); return true;
        case SQMIX_ABI_GDN_LAYER_ARGS: *e = entry(sizeof(sqmix_gdn_layer_args), kGdnLayer); return true;
        case SQMIX_ABI_GGML_FA_OP: *e = entry(sizeof(sqmix_ggml_fa_op), kGgmlFaOp); return true;
        case SQMIX_ABI_GGML_GDN_OP: *e = entry(sizeof(sqmix_ggml_gdn_op), kGgmlGdnOp); return true;
        case SQMIX_ABI_MUL_MAT_ARGS: *e = entry(sizeof(sqmix_mul_mat_args), kMulMat); return true;
        default: return false;
    }
}

}  // namespace

extern "C" size_t sqmix_abi_struct_size(int32_t which) {
    Entry e;
    return lookup(which, &e) ? e.size : 0;
}

extern "C" int32_t sqmix_abi_field_count(int32_t which) {
    Entry e;
    return lookup(which, &e) ? e.n_fields : -1;
}

extern "C" int64_t sqmix_abi_field_offset(int32_t which, int32_t field) {
    Entry e;
    if (!lookup(which, &e) || field < 0 || field >= e.n_fields) return -1;
    return static_cast<int64_t>(e.offsets[field]);
}
