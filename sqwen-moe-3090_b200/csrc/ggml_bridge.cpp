// ggml_bridge.cpp -- sqmix kernels as ggml custom-op nodes.
//
// A ggml graph node built with ggml_custom_4d(ctx, type, ne..., args, n_args, fun,
// n_tasks, userdata) calls fun(dst, ith, nth, userdata) when the graph runs; dst->src[]
// holds the node's arguments.  The callbacks here read the node's tensors through the
// layout of ggml's struct ggml_tensor (the public struct that sqwen's FFI declares
// field for field at src/backend/ffi.rs:22-39; mirrored below as GgmlTensor), translate
// them into sqmix_fa_args / sqmix_gdn_args and launch the kernels on the stream given
// in the userdata.  Only thread 0 of the node launches; the others return at once.
// Nothing here allocates: without a workspace the attention node uses the static
// scratch of sqmix_fa_decode_noalloc, which is what a callback inside a planned graph
// needs.
#include <stddef.h>
#include <stdint.h>

#include "common.cuh"
#include "sqmix.h"

namespace {

// ggml's tensor struct, as sqwen's FFI mirrors it (ffi.rs:22-39).
struct GgmlTensor {
    int32_t type;
    void *buffer;
    int64_t ne[4];
    size_t nb[4];
    int32_t op;
    int32_t op_params[16];
    int32_t flags;
    GgmlTensor *src[10];
    GgmlTensor *view_src;
    size_t view_offs;
    void *data;
    char name[64];
    void *extra;
    char padding[8];
};
static_assert(sizeof(void *) != 8 || sizeof(GgmlTensor) == 336, "ggml_tensor is 336 bytes on 64-bit hosts");

// ggml type ids (ffi.rs:44-101)
constexpr int32_t kTypeF32 = 0, kTypeF16 = 1, kTypeQ4_0 = 2, kTypeI32 = 26, kTypeI64 = 27, kTypeBF16 = 30;

size_t elem_bytes(int32_t t) {
    switch (t) {
        case kTypeF32: return 4;
        case kTypeF16: return 2;
        case kTypeBF16: return 2;
        case kTypeI32: return 4;
        case kTypeI64: return 8;
        default: return 0;
    }
}

bool float_type(int32_t t) { return t == kTypeF32 || t == kTypeF16 || t == kTypeBF16; }

// element stride of dimension d of t (bytes / element size; 0 if not a whole number)
int64_t estride(const GgmlTensor *t, int d) {
    const size_t e = elem_bytes(t->type);
    return e && t->nb[d] % e == 0 ? static_cast<int64_t>(t->nb[d] / e) : 0;
}

bool contiguous_f32(const GgmlTensor *t) {
    if (t->type != kTypeF32 || t->nb[0] != 4) return false;
    size_t want = 4;
    for (int d = 0; d < 4; ++d) {
        if (t->ne[d] > 1 && t->nb[d] != want) return false;
        want *= static_cast<size_t>(t->ne[d]);
    }
    return true;
}

}  // namespace

using sqmix::set_error;

extern "C" size_t sqmix_ggml_tensor_bytes(void) { return sizeof(GgmlTensor); }

extern "C" int sqmix_ggml_fa_args(const struct ggml_tensor *dst_, const sqmix_ggml_fa_op *op, sqmix_fa_args *a) {
    const GgmlTensor *dst = reinterpret_cast<const GgmlTensor *>(dst_);
    SQMIX_CHECK_ARG(dst && op && a, "ggml_fa_args: null argument");
    const GgmlTensor *q = dst->src[0], *k = dst->src[1], *v = dst->src[2], *step = dst->src[3];
    const GgmlTensor *gate = dst->src[4], *kn = dst->src[5], *vn = dst->src[6];
    SQMIX_CHECK_ARG(q && k && v && step, "ggml_fa_args: the node needs src[0..3] = Q, K, V, {n_kv, q_pos0}");
    const int64_t T = q->ne[1];
    SQMIX_CHECK_ARG(float_type(q->type) && q->ne[0] == SQMIX_HEAD_DIM && q->ne[2] == SQMIX_N_HEAD && q->ne[3] == 1 &&
                        q->nb[0] == elem_bytes(q->type) && estride(q, 1) > 0 && estride(q, 2) > 0,
                    "ggml_fa_args: Q must be [256, T, 16] F32/F16/BF16 with element-aligned strides");
    SQMIX_CHECK_ARG(T == 1 || T == 2, "ggml_fa_args: T=%lld query tokens (decode nodes take 1 or 2)", (long long)T);
    SQMIX_CHECK_ARG(dst->type == kTypeF32 && dst->ne[0] == SQMIX_HEAD_DIM && dst->ne[1] == SQMIX_N_HEAD &&
                        dst->ne[2] == T && dst->nb[0] == 4 && dst->nb[1] == 4 * SQMIX_HEAD_DIM &&
                        dst->nb[2] == 4 * SQMIX_HEAD_DIM * SQMIX_N_HEAD,
                    "ggml_fa_args: dst must be contiguous F32 [256, 16, T]");
    for (const GgmlTensor *c : {k, v})
        SQMIX_CHECK_ARG(c->type == kTypeQ4_0 && c->ne[0] == 2 * SQMIX_HEAD_DIM && c->ne[1] == k->ne[1] &&
                            c->ne[1] % SQMIX_KV_PAD == 0 && c->data,
                        "ggml_fa_args: K and V must be Q4_0 [512, capacity] tiled caches, capacity a multiple of 256");
    SQMIX_CHECK_ARG(step->type == kTypeI64 && step->ne[0] >= 2 && step->nb[0] == 8,
                    "ggml_fa_args: src[3] must be I64 [2] {n_kv, q_pos0}");
    SQMIX_CHECK_ARG(!gate || (float_type(gate->type) && gate->ne[0] == SQMIX_HEAD_DIM &&
                              gate->ne[1] == SQMIX_N_HEAD && gate->ne[2] == T && gate->nb[0] == elem_bytes(gate->type) &&
                              estride(gate, 1) > 0 && estride(gate, 2) > 0),
                    "ggml_fa_args: gate must be [256, 16, T]");
    SQMIX_CHECK_ARG((kn == nullptr) == (vn == nullptr), "ggml_fa_args: k_new and v_new come together");
    if (kn) {
        for (const GgmlTensor *c : {kn, vn})
            SQMIX_CHECK_ARG(c->type == kn->type && float_type(c->type) && c->ne[0] == SQMIX_HEAD_DIM &&
                                c->ne[1] == SQMIX_N_HEAD_KV && c->ne[2] >= 1 && c->ne[2] <= T &&
                                c->nb[0] == elem_bytes(c->type) && estride(c, 1) == SQMIX_HEAD_DIM && estride(c, 2) > 0,
                            "ggml_fa_args: k_new / v_new must be [256, 2, n_new] with contiguous heads");
        SQMIX_CHECK_ARG(vn->ne[2] == kn->ne[2], "ggml_fa_args: k_new and v_new differ in rows");
    }
    *a = sqmix_fa_args{};
    a->q = q->data;
    a->q_dtype = q->type;
    a->q_stride_tok = estride(q, 1);
    a->q_stride_head = estride(q, 2);
    if (gate) {
        a->gate = gate->data;
        a->gate_dtype = gate->type;
        a->gate_stride_head = estride(gate, 1);
        a->gate_stride_tok = estride(gate, 2);
    }
    a->k_cache = k->data;
    a->v_cache = v->data;
    a->capacity = k->ne[1];
    a->n_kv = static_cast<const int64_t *>(step->data);
    a->q_pos0 = static_cast<const int64_t *>(step->data) + 1;
    a->n_q = static_cast<int32_t>(T);
    a->scale = op->scale;
    a->rope_n_rot = op->rope_n_rot;
    a->rope_freq_base = op->rope_freq_base;
    a->rope_pos_offset = op->rope_pos_offset;
    a->out = static_cast<float *>(dst->data);
    a->workspace = op->workspace;
    a->workspace_bytes = op->workspace_bytes;
    a->n_splits = op->n_splits;
    a->config = op->config;
    if (kn) {
        a->k_new = kn->data;
        a->v_new = vn->data;
        a->kv_new_dtype = kn->type;
        a->k_new_stride_tok = estride(kn, 2);
        a->v_new_stride_tok = estride(vn, 2);
        a->n_new = static_cast<int32_t>(kn->ne[2]);
    }
    a->flags = op->flags;
    a->q_norm = op->q_norm;
    a->k_norm = op->k_norm;
    a->norm_eps = op->norm_eps;
    return SQMIX_OK;
}

extern "C" int sqmix_ggml_gdn_args(const struct ggml_tensor *dst_, const sqmix_ggml_gdn_op *op, sqmix_gdn_args *a) {
    const GgmlTensor *dst = reinterpret_cast<const GgmlTensor *>(dst_);
    SQMIX_CHECK_ARG(dst && op && a, "ggml_gdn_args: null argument");
    const GgmlTensor *q = dst->src[0], *k = dst->src[1], *v = dst->src[2], *g = dst->src[3], *b = dst->src[4];
    const GgmlTensor *st = dst->src[5], *sel = dst->src[6];
    SQMIX_CHECK_ARG(q && k && v && g && b && st,
                    "ggml_gdn_args: the node needs src[0..5] = q, k, v, g, beta, state");
    const int64_t h_k = q->ne[1], T = q->ne[2], n_seqs = q->ne[3], h_v = v->ne[1];
    const int64_t d = SQMIX_GDN_D;
    SQMIX_CHECK_ARG(float_type(q->type) && q->type == k->type && q->type == v->type && q->ne[0] == d && k->ne[0] == d &&
                        v->ne[0] == d && k->ne[1] == h_k && k->ne[2] == T && k->ne[3] == n_seqs && v->ne[2] == T &&
                        v->ne[3] == n_seqs,
                    "ggml_gdn_args: q, k [128, H_k, T, n_seqs] and v [128, H_v, T, n_seqs] of one float type");
    SQMIX_CHECK_ARG(q->nb[0] == elem_bytes(q->type) && estride(q, 1) == d && k->nb[1] == q->nb[1] &&
                        k->nb[2] == q->nb[2] && k->nb[3] == q->nb[3] && estride(v, 1) == d && v->nb[0] == q->nb[0],
                    "ggml_gdn_args: q, k and v need contiguous 128-wide heads (q and k with equal strides)");
    SQMIX_CHECK_ARG(contiguous_f32(g) && contiguous_f32(b) && g->ne[0] == 1 && g->ne[1] == h_v && g->ne[2] == T &&
                        g->ne[3] == n_seqs && b->ne[0] == 1 && b->ne[1] == h_v && b->ne[2] == T && b->ne[3] == n_seqs,
                    "ggml_gdn_args: g and beta must be contiguous F32 [1, H_v, T, n_seqs]");
    SQMIX_CHECK_ARG(contiguous_f32(st) && st->ne[0] == d * d * h_v && st->ne[2] == n_seqs && st->ne[3] == 1,
                    "ggml_gdn_args: state must be contiguous F32 [128*128*H_v, n_planes, n_seqs]");
    SQMIX_CHECK_ARG(!sel || (sel->type == kTypeI32 && sel->ne[0] == n_seqs && sel->nb[0] == 4),
                    "ggml_gdn_args: sel must be I32 [n_seqs]");
    SQMIX_CHECK_ARG(dst->type == kTypeF32 && dst->ne[0] == d && dst->ne[1] == h_v && dst->ne[2] == T &&
                        dst->ne[3] == n_seqs && contiguous_f32(dst),
                    "ggml_gdn_args: dst must be contiguous F32 [128, H_v, T, n_seqs]");
    *a = sqmix_gdn_args{};
    a->q = q->data;
    a->k = k->data;
    a->v = v->data;
    a->dtype = q->type;
    a->qk_stride_tok = estride(q, 2);
    a->v_stride_tok = estride(v, 2);
    a->qk_stride_seq = estride(q, 3);
    a->v_stride_seq = estride(v, 3);
    a->g = static_cast<const float *>(g->data);
    a->beta = static_cast<const float *>(b->data);
    a->state = static_cast<float *>(st->data);
    a->n_planes = static_cast<int32_t>(st->ne[1]);
    a->sel = sel ? static_cast<const int32_t *>(sel->data) : nullptr;
    a->n_seqs = static_cast<int32_t>(n_seqs);
    a->n_tokens = static_cast<int32_t>(T);
    a->h_k = static_cast<int32_t>(h_k);
    a->h_v = static_cast<int32_t>(h_v);
    a->n_snap = op->n_snap;
    a->l2_eps = op->l2_eps;
    a->out = static_cast<float *>(dst->data);
    a->flags = op->flags;
    a->h_v_offset = op->h_v_offset;
    a->dt_bias = op->dt_bias;
    a->ssm_a = op->ssm_a;
    return SQMIX_OK;
}

extern "C" void sqmix_ggml_fa_decode_op(struct ggml_tensor *dst, int ith, int nth, void *userdata) {
    (void)nth;
    if (ith != 0 || !userdata) return;
    auto *op = static_cast<sqmix_ggml_fa_op *>(userdata);
    sqmix_fa_args a;
    int rc = sqmix_ggml_fa_args(dst, op, &a);
    if (rc == SQMIX_OK) rc = op->workspace ? sqmix_fa_decode(&a, op->stream) : sqmix_fa_decode_noalloc(&a, op->stream);
    op->status = rc;
}

extern "C" void sqmix_ggml_gdn_decode_op(struct ggml_tensor *dst, int ith, int nth, void *userdata) {
    (void)nth;
    if (ith != 0 || !userdata) return;
    auto *op = static_cast<sqmix_ggml_gdn_op *>(userdata);
    sqmix_gdn_args a;
    int rc = sqmix_ggml_gdn_args(dst, op, &a);
    if (rc == SQMIX_OK) rc = sqmix_gdn_decode(&a, op->stream);
    op->status = rc;
}
