/*
 * sqmix.h -- C ABI of the B200 (sm_100a) attention-mixer kernels for qwen35moe.
 *
 * This library replaces, for exactly these nodes, the ggml FFI that sqwen's graph
 * builder calls (src/backend/ffi.rs:232-481):
 *
 *   ggml_set_rows (q4_0 KV append)      -> sqmix_kv_append_q4_0
 *   ggml_rope_multi (IMROPE, text pos)  -> fused into sqmix_kv_append_q4_0 (K)
 *                                          and sqmix_fa_decode (Q)
 *   ggml_flash_attn_ext + sigmoid gate  -> sqmix_fa_decode, sqmix_attn_merge_lse
 *   ggml_gated_delta_net (+ state cpy)  -> sqmix_gdn_decode
 *   ggml_get_rows (state plane select)  -> the `sel` argument of sqmix_gdn_decode
 *   ggml_cpy of GDN snapshot planes     -> written in place by sqmix_gdn_decode
 *
 * and the engine-side bookkeeping that feeds them (src/engine/kv.rs KvCache,
 * src/model/gdn.rs GdnState, src/model/graph.rs snapshot_gdn/restore_gdn).
 *
 * Conventions (all entry points):
 *   - Return int status: SQMIX_OK (0) or a negative SQMIX_E* code; a message for
 *     the last failure on the calling thread is in sqmix_last_error().  Nothing
 *     aborts the process (unlike ggml's GGML_ABORT on unsupported FA).
 *   - Kernel entry points take device pointers, launch on the given stream, never
 *     allocate, never synchronise, and read positions/lengths from device scalars
 *     so they can be replayed from a CUDA graph with fixed pointers
 *     (the same constraint sqwen meets with set_rows: src/engine/kv.rs:300-312).
 *   - Geometry is qwen35moe's: head_dim 256, 16 query heads over 2 KV heads
 *     (block GQA, kv_head = h / 8), GDN d_k = d_v = 128.
 *   - `sqmix_stream_t` is a cudaStream_t (NULL = legacy default stream).
 */
#ifndef SQMIX_H
#define SQMIX_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *sqmix_stream_t;

/* ---- status codes ------------------------------------------------------- */
#define SQMIX_OK 0
#define SQMIX_EINVAL (-1)    /* bad argument (null pointer, unsupported shape, ...) */
#define SQMIX_ECUDA (-2)     /* a CUDA runtime call failed */
#define SQMIX_ETIMEOUT (-3)  /* a bounded device-side wait gave up */
#define SQMIX_ENOSPC (-4)    /* workspace or host buffer too small */
#define SQMIX_EOVERFLOW (-5) /* KV cache overflow (kv.rs:240-245) */
#define SQMIX_ERANGE (-6)    /* position out of range (kv.rs:284-297) */

/* ---- element types (ggml type ids, src/backend/ffi.rs:44-101) ----------- */
#define SQMIX_F32 0
#define SQMIX_F16 1
#define SQMIX_Q8_0 8   /* weight block formats of sqmix_mul_mat */
#define SQMIX_Q4_K 12
#define SQMIX_Q6_K 14
#define SQMIX_BF16 30

/* ---- fixed geometry ----------------------------------------------------- */
#define SQMIX_HEAD_DIM 256     /* full-attention head_dim (arch.rs validates 256) */
#define SQMIX_N_HEAD 16        /* query heads */
#define SQMIX_N_HEAD_KV 2      /* KV heads */
#define SQMIX_QK4_0 32         /* q4_0 block (kv.rs:33) */
#define SQMIX_KV_GROUP 16      /* tokens per tile group of the tiled q4_0 cache */
#define SQMIX_KV_PAD 256       /* n_kv padding / capacity alignment (kv.rs:37) */
#define SQMIX_GDN_D 128        /* GDN head_k_dim == head_v_dim */

const char *sqmix_version(void);
/* Message for the last failing call on this thread ("" if none). */
const char *sqmix_last_error(void);
/* Number of SMs of `device` (sizes split-KV grids). */
int sqmix_device_sm_count(int device);

/* ---- ABI layout table ----------------------------------------------------
 * Size, field count and field byte offsets (declaration order) of the argument
 * structs below, as compiled into the library, so that a binding in another language
 * can check its own declaration of them (the role of the ggml header guard in
 * src/backend/ffi.rs:516-588).  Unknown `which`: size 0, count -1; a field index out
 * of range: offset -1. */
#define SQMIX_ABI_KV_APPEND_ARGS 1
#define SQMIX_ABI_FA_ARGS 2
#define SQMIX_ABI_FA_BATCH_ARGS 3
#define SQMIX_ABI_PEER_MERGE_ARGS 4
#define SQMIX_ABI_GDN_ARGS 5
#define SQMIX_ABI_GDN_CONV_ARGS 6
#define SQMIX_ABI_HEAD_NORM_ARGS 7
#define SQMIX_ABI_GDN_LAYER_ARGS 8
#define SQMIX_ABI_GGML_FA_OP 9
#define SQMIX_ABI_GGML_GDN_OP 10
#define SQMIX_ABI_MUL_MAT_ARGS 11
size_t sqmix_abi_struct_size(int32_t which);
int32_t sqmix_abi_field_count(int32_t which);
int64_t sqmix_abi_field_offset(int32_t which, int32_t field);

/* ========================================================================
 * q4_0 KV cache: tiled layout
 *
 * Each layer owns a K cache and a V cache of `capacity` token rows (capacity a
 * multiple of SQMIX_KV_PAD).  Every 32-element block is the ggml q4_0 block
 * bit-for-bit (fp16 d, 16 nibble bytes: element j low nibble of byte j, element
 * j+16 high nibble), 576 bytes per token per layer for K+V, as in
 * kv.rs:179-189.  Blocks are arranged in 16-token groups so that the decode
 * kernel's 128-bit shared-memory loads land directly in tensor-core fragments.
 * sqmix_kv_convert_rows translates to and from ggml's row layout
 * ([n_embd_k_gqa=512, cap] q4_0, kv.rs:124-134).
 * ======================================================================== */

/* Bytes of ONE K (or V) cache of `capacity` rows with SQMIX_N_HEAD_KV heads. */
size_t sqmix_kv_cache_bytes(int64_t capacity);

typedef struct sqmix_kv_append_args {
    const void *k;          /* [T][2][256] new K rows (before RoPE) */
    const void *v;          /* [T][2][256] new V rows */
    int32_t dtype;          /* SQMIX_F32 / SQMIX_F16 / SQMIX_BF16 for k and v */
    int64_t k_stride_tok;   /* elements between consecutive tokens of k (>= 512) */
    int64_t v_stride_tok;   /* same for v */
    int32_t n_tokens;       /* T >= 1 */
    const int64_t *rows;    /* device I64 [T]: destination row = absolute position
                               (ggml_set_rows idxs, kv.rs:313-320, graph.rs:476-480) */
    void *k_cache;          /* tiled q4_0 K cache of this layer */
    void *v_cache;          /* tiled q4_0 V cache of this layer */
    int64_t capacity;       /* rows in each cache */
    int32_t rope_n_rot;     /* > 0: rotate K dims [0, n_rot) at text position
                               rows[t] + rope_pos_offset */
    float rope_freq_base;   /* theta base (qwen35moe: 1e7) */
    int64_t rope_pos_offset;/* absolute position of row 0 (0 unless the cache holds a
                               slice of the sequence, e.g. split-KV across GPUs) */
} sqmix_kv_append_args;

/* KvCache::append -> ggml_set_rows(q4_0) (kv.rs:313-399), with the IMROPE of K
 * (attn.rs:183-204, text positions) fused in front of quantisation.  Quantisation
 * is bit-exact with ggml quantize_row_q4_0 for the same f32 input. */
int sqmix_kv_append_q4_0(const sqmix_kv_append_args *args, sqmix_stream_t stream);

/* Translate rows [row0, row0+n_rows) between a tiled cache and ggml row layout
 * (n_rows x 288 bytes, row r at rows_buf + (r-row0)*288).  which: 0 = K cache,
 * 1 = V cache (their tilings differ).  to_rows != 0: tiled -> rows; 0: rows ->
 * tiled (imports a ggml cache).  Device pointers. */
int sqmix_kv_convert_rows(void *tiled_cache, void *rows_buf, int64_t capacity, int64_t row0,
                          int64_t n_rows, int32_t which, int32_t to_rows, sqmix_stream_t stream);

/* ========================================================================
 * Split-KV attention decode: one cooperative launch per layer and step that does
 * the q4_0 append of the step's rows (ggml_set_rows, kv.rs:367-396), attention over
 * the cache (ggml_flash_attn_ext, attn.rs:238-249), the split merge and the sigmoid
 * output gate (attn.rs:282-283).
 * ======================================================================== */

typedef struct sqmix_fa_args {
    const void *q;            /* [n_q][16][256] queries (before RoPE) */
    int32_t q_dtype;
    int64_t q_stride_tok;     /* elements between tokens */
    int64_t q_stride_head;    /* elements between heads (512 for the QG-interleaved
                                 projection of attn.rs:131-158) */
    const void *gate;         /* nullable: [n_q][16][256], out *= sigmoid(gate) */
    int32_t gate_dtype;
    int64_t gate_stride_tok;
    int64_t gate_stride_head;
    const void *k_cache;      /* tiled q4_0 caches of this layer */
    const void *v_cache;
    int64_t capacity;
    const int64_t *n_kv;      /* device scalar: keys [0, n_kv) are stored */
    const int64_t *q_pos0;    /* device scalar: absolute position of query 0;
                                 query t sees keys j <= q_pos0 + t (graph.rs:553-559) */
    int32_t n_q;              /* 1 or 2 (decode, MTP verify) */
    float scale;              /* softmax scale (1/sqrt(256) = 1/16) */
    int32_t rope_n_rot;       /* > 0: rotate Q dims [0, n_rot) at positions
                                 q_pos0 + t + rope_pos_offset */
    float rope_freq_base;
    int64_t rope_pos_offset;  /* as in sqmix_kv_append_args */
    float *out;               /* [n_q][16][256] f32 */
    float *lse;               /* nullable [n_q][16]: ln sum_j exp(scale * s_j) */
    void *workspace;          /* device scratch, sqmix_fa_workspace_bytes(); its
                                 first 256 bytes must be zero before first use */
    size_t workspace_bytes;
    int32_t n_splits;         /* 0 = one split per SM */
    int32_t config;           /* kernel configuration, 0 = auto (see fa_decode.cu) */
    /* Fused append (n_new > 0): rows q_pos0 + t, t < n_new <= n_q, of the caches are
     * first written from k_new/v_new [n_new][2][256] (K rotated like Q), exactly as
     * sqmix_kv_append_q4_0 would write them; n_kv must already count them. */
    const void *k_new;
    const void *v_new;
    int32_t kv_new_dtype;
    int64_t k_new_stride_tok;
    int64_t v_new_stride_tok;
    int32_t n_new;
    int32_t flags;            /* SQMIX_FA_* bits below, 0 = none */
    /* Per-head RMS norm before RoPE (head_rms_norm of attn.rs:66-84, applied to Q and
     * K at attn.rs:166-175): x / sqrt(mean(x^2) + norm_eps) * w over each 256-wide
     * head, for the Q rows and for the fused-append K rows.  NULL: the inputs are
     * already normalised.  Decode only: sqmix_fa_prefill rejects them (normalise with
     * sqmix_head_norm first). */
    const float *q_norm;      /* nullable [256] attn_q_norm weight */
    const float *k_norm;      /* nullable [256] attn_k_norm weight */
    float norm_eps;           /* norm_rms_eps */
} sqmix_fa_args;

/* The decode and merge kernels are launched with programmatic stream serialisation:
 * each starts while the kernel before it on the stream drains and waits for it
 * (griddepcontrol.wait) before reading q, gate, k_new/v_new or the workspace.  The
 * merge kernel in turn lets the launch after it start as soon as it is resident, so
 * the next kernel's prologue overlaps this call's tail; a kernel launched right after
 * sqmix_fa_decode must read nothing this call writes (appended rows, workspace, out,
 * lse) before its own dependency wait -- every sqmix kernel meets that.
 * SQMIX_FA_OVERLAP_PREV also lets the decode kernel read *n_kv, *q_pos0 and request
 * cache rows below *q_pos0 BEFORE that wait, overlapping the previous kernels' tail.
 * Set it only when none of those is written by the kernel launched immediately before
 * this call on the stream, nor by a sqmix_fa_decode call that immediately precedes it
 * (a copy, or any other kernel two or more launches back, is fine): the engine's step
 * loop uploads the scalars with a copy and writes the step's rows (>= q_pos0) with the
 * fused append; consecutive layers use different caches. */
#define SQMIX_FA_OVERLAP_PREV 1

/* Workspace for n_splits splits (0 = enough for every configuration's default). */
size_t sqmix_fa_workspace_bytes(int32_t n_splits, int32_t n_q);
int sqmix_fa_decode(const sqmix_fa_args *args, sqmix_stream_t stream);
/* Reads (and clears) the device status word of a workspace: SQMIX_OK, SQMIX_ETIMEOUT
 * when a bounded device-side wait gave up, SQMIX_ERANGE when n_kv exceeded the
 * capacity.  Synchronises the stream. */
int sqmix_fa_status(void *workspace, sqmix_stream_t stream);

/* Prefill attention on the tcgen05 tensor cores: the same arguments as sqmix_fa_decode
 * for n_q = T in 1..4096 query tokens (ggml_flash_attn_ext of a prefill chunk,
 * attn.rs:238-249, causal mask graph.rs:553-559).  The step's rows must already be in
 * the cache (sqmix_kv_append_q4_0; n_new must be 0).  n_splits = number of persistent
 * CTAs, run as CTA pairs (rounded down to even, at least one pair; 0 = as many pairs as
 * are resident at once); config and flags are ignored.  q must be aligned to two
 * elements with even strides.  Launches a preparation kernel (item table and Q), the
 * main kernel and a merge kernel, the last two as programmatic dependents of the one
 * before.  The workspace (sqmix_fa_prefill_workspace_bytes, 256-byte aligned)
 * needs no initialisation; its first word holds device status bits as for decode
 * (read with sqmix_fa_status). */
size_t sqmix_fa_prefill_workspace_bytes(int32_t n_q, int32_t n_ctas);
int sqmix_fa_prefill(const sqmix_fa_args *args, sqmix_stream_t stream);

/* Sequence-batched decode (the batched decode step of many independent sequences,
 * one query token each; the engine's per-sequence ggml_flash_attn_ext calls,
 * attn.rs:238-249).  Sequence s uses tiled caches k_caches[s] / v_caches[s] with
 * capacities[s] rows, device scalars n_kv[s], q_pos0[s], query q + s*q_stride_seq
 * ([16][256]), gate likewise, output out + s*4096 ([16][256] f32) and lse + s*16.
 * k_new/v_new (n_new = 1): [n_seqs][2][256] with new_stride_seq, written at row
 * q_pos0[s] first.  The pointer and scalar arrays live in device memory.  Split
 * partials of all sequences share the workspace (sqmix_fa_batch_workspace_bytes, first
 * 256 bytes zero before first use).  splits_per_seq 0 = about 2 CTAs per SM over the
 * batch.  flags as for sqmix_fa_decode. */
typedef struct sqmix_fa_batch_args {
    int32_t n_seqs;
    const void *q;
    int32_t q_dtype;
    int64_t q_stride_seq;
    int64_t q_stride_head;
    const void *gate;         /* nullable */
    int32_t gate_dtype;
    int64_t gate_stride_seq;
    int64_t gate_stride_head;
    const void *const *k_caches;
    const void *const *v_caches;
    const int64_t *capacities;
    const int64_t *n_kv;
    const int64_t *q_pos0;
    float scale;
    int32_t rope_n_rot;
    float rope_freq_base;
    float *out;
    float *lse;               /* nullable */
    void *workspace;
    size_t workspace_bytes;
    int32_t splits_per_seq;
    const void *k_new;
    const void *v_new;
    int32_t kv_new_dtype;
    int64_t new_stride_seq;
    int32_t n_new;
    int32_t flags;
} sqmix_fa_batch_args;

size_t sqmix_fa_batch_workspace_bytes(int32_t n_seqs, int32_t splits_per_seq);
int sqmix_fa_decode_batch(const sqmix_fa_batch_args *args, sqmix_stream_t stream);

/* Cross-GPU merge of split-KV partials over peer memory (NVLink P2P), for
 * long-context decode split across ranks (one process per GPU).  Each rank creates
 * one peer buffer (n_slots = layers it merges per step), shares the IPC handle with
 * the other ranks (any host channel), opens theirs, and puts the n_ranks pointers
 * (its own at [rank]) in a device array.  The ranks push: each writes its normalised
 * partial for a slot into every other rank's buffer with 8-byte stores that pair each
 * value with a publication tag, and waits (bounded, 2 s) in its own memory until every
 * peer's words carry the tag; no flag, fence or remote polling is involved.  Then
 * out = sum_r O_r e^{lse_r - L} (* sigmoid(gate)), lse_out = L (natural log).
 * Every rank must call it once per slot per step, in the same order, and a slot is
 * used with one entry point only (sqmix_attn_merge_peers or sqmix_fa_decode_peers).
 * A wait that gives up sets bit 1 of *status (nullable) and leaves out unwritten; the
 * buffers' publication counters then no longer agree across ranks, so after any
 * nonzero status every rank resets its buffer (sqmix_peer_buffer_reset, after all
 * ranks have stopped calling) before reusing it.  Buffers start zeroed; destroy them
 * only after every rank has finished its last merge. */
#define SQMIX_IPC_HANDLE_BYTES 64
typedef struct sqmix_peer_merge_args {
    int32_t n_ranks;          /* <= 8 */
    int32_t rank;
    int32_t slot;
    int32_t n_slots;
    int32_t rows;             /* 16 x n_q, <= 32 */
    const void *const *buffers; /* device array [n_ranks] of peer buffers as mapped here */
    const float *o_local;     /* [rows][256] (sqmix_attn_merge_peers only) */
    const float *lse_local;   /* [rows] (sqmix_attn_merge_peers only) */
    const float *gate;        /* nullable [rows][256] f32 (sqmix_attn_merge_peers only) */
    float *out;               /* [rows][256] (sqmix_attn_merge_peers only) */
    float *lse_out;           /* nullable [rows] (sqmix_attn_merge_peers only) */
    void *status;             /* nullable device u32 */
} sqmix_peer_merge_args;

size_t sqmix_peer_buffer_bytes(int32_t n_slots);
int sqmix_peer_buffer_create(int32_t n_slots, void **dev_ptr, void *ipc_handle /* 64 bytes out */);
int sqmix_peer_buffer_open(const void *ipc_handle, void **peer_ptr);
int sqmix_peer_buffer_close(void *peer_ptr);
int sqmix_peer_buffer_destroy(void *dev_ptr);
/* Zeroes a buffer this rank created (async on stream): no publication, counters 0. */
int sqmix_peer_buffer_reset(void *dev_ptr, int32_t n_slots, sqmix_stream_t stream);
int sqmix_attn_merge_peers(const sqmix_peer_merge_args *args, sqmix_stream_t stream);

/* Split-KV decode of one layer across ranks in two launches: the decode kernel over
 * this rank's key slice (a: as for sqmix_fa_decode, with rope_pos_offset = the slice
 * start and n_kv / q_pos0 in slice rows; the rank owning the step's rows passes
 * k_new / v_new), then one kernel that merges the split partials of this rank, pushes
 * the result into the peers' buffers, waits for theirs and writes the merged, gated
 * output to a->out (and a->lse).  peers: n_ranks, rank, slot, n_slots, rows (= 16 n_q),
 * buffers and status as for sqmix_attn_merge_peers; its o_local, lse_local, gate, out
 * and lse_out are not used.  With n_ranks = 1 it equals sqmix_fa_decode. */
int sqmix_fa_decode_peers(const sqmix_fa_args *a, const sqmix_peer_merge_args *peers, sqmix_stream_t stream);

/* sqmix_fa_decode without a caller workspace (no reference counterpart: ggml_flash_attn_ext
 * takes its scratch from ggml's graph allocator).  For callers that cannot allocate
 * device memory at the call site, e.g. a callback inside a graph executor whose buffers
 * are all planned before compute (cudaMalloc would synchronise the device and break a
 * replayed CUDA graph's fixed addresses).  The split partials live in a file-scope
 * __device__ array of SQMIX_FA_NOALLOC_SCRATCH_BYTES (the workspace of
 * SQMIX_FA_NOALLOC_MAX_SPLITS splits at n_q 2, about 5 MiB); args->workspace and
 * workspace_bytes are ignored.  Split counts above the maximum (explicit, or one per SM
 * when n_splits is 0) are rejected with SQMIX_EINVAL / SQMIX_ENOSPC and a message.
 * The array's status header must start at zero: static device storage is
 * zero-initialised at module load, and the kernels write it only on a device-side wait
 * failure, which this entry point does not read back.  The first call on each device
 * does the setup (symbol lookup with that device current, possibly a module load, the
 * kernel's shared-memory attribute) and should precede any stream capture.  All calls
 * on a device share the one array: calls that overlap in time (other streams, other
 * threads) race on it and must be serialised by the caller. */
#define SQMIX_FA_NOALLOC_MAX_SPLITS 160
#define SQMIX_FA_NOALLOC_SCRATCH_BYTES 5284096
int sqmix_fa_decode_noalloc(const sqmix_fa_args *args, sqmix_stream_t stream);
/* Reads and clears the status word of the current device's static scratch, as
 * sqmix_fa_status does for a workspace (SQMIX_OK, SQMIX_ETIMEOUT, SQMIX_ERANGE when n_kv
 * exceeded the capacity and was clamped).  Synchronises the stream. */
int sqmix_fa_noalloc_status(sqmix_stream_t stream);

/* Merge n_parts normalised partial attentions (O_p, lse_p) over disjoint key sets
 * (split-KV across GPUs): out = sum_p O_p exp(lse_p - L) with L = log sum exp(lse_p),
 * then out *= sigmoid(gate) when gate != NULL.  o_parts [n_parts][n_rows][256],
 * lse_parts [n_parts][n_rows]; gate [n_rows][256] f32 or NULL; lse_out nullable. */
int sqmix_attn_merge_lse(int32_t n_parts, int32_t n_rows, const float *o_parts,
                         const float *lse_parts, const float *gate, float *out, float *lse_out,
                         sqmix_stream_t stream);

/* ========================================================================
 * Gated delta net (ggml_gated_delta_net, gdn.rs:489-500; recurrence gdn.rs:9-24)
 *
 * State planes: [n_seqs][n_planes][H_v][128 (value j)][128 (key i)] f32; element
 * S[i][j] of head h sits at ((h*128 + j)*128 + i).  n_planes = 1 + n_rs
 * (gdn.rs:71-106).  The kernel reads plane sel[seq] (MTP rollback, gdn.rs:445-463,
 * graph.rs:190-196) and writes the state after T-s tokens into plane s for
 * s < n_snap (slot 0 = final; gdn.rs:484-538, graph.rs:884-912).
 * ======================================================================== */

typedef struct sqmix_gdn_args {
    const void *q;            /* [n_seqs][T][H_k][128] */
    const void *k;            /* [n_seqs][T][H_k][128] */
    const void *v;            /* [n_seqs][T][H_v][128] */
    int32_t dtype;            /* of q, k, v */
    int64_t qk_stride_tok;    /* elements between tokens of q and k */
    int64_t v_stride_tok;
    int64_t qk_stride_seq;
    int64_t v_stride_seq;
    const float *g;           /* [n_seqs][T][H_v] log-decay (<= 0) */
    const float *beta;        /* [n_seqs][T][H_v] */
    float *state;             /* [n_seqs][n_planes][H_v][128][128] */
    int32_t n_planes;
    const int32_t *sel;       /* device I32 [n_seqs] plane to read; NULL = plane 0 */
    int32_t n_seqs;
    int32_t n_tokens;
    int32_t h_k;              /* q/k heads (16); value head hv reads q/k head hv % h_k */
    int32_t h_v;              /* value heads (32) */
    int32_t n_snap;           /* 1 <= n_snap <= min(T, n_planes) */
    float l2_eps;             /* > 0: L2-normalise q and k per head first (gdn.rs:126-142) */
    float *out;               /* [n_seqs][T][H_v][128] f32 */
    int32_t flags;            /* SQMIX_GDN_* bits (0 = none) */
    /* Value-head sharding (value heads split across ranks, no exchange in the
     * recurrence): value head i of this call is head h_v_offset + i of the layer and
     * reads q/k head (h_v_offset + i) % h_k; q and k hold all h_k heads, while v, g,
     * beta, the state planes and out hold this call's h_v heads.  0 for a whole layer
     * (whose h_v is a multiple of h_k: the tiling of gdn.rs:436-441). */
    int32_t h_v_offset;
    /* Gate epilogue of the projections (gdn.rs:268-287).  ssm_a == NULL: g and beta are
     * the log-decay and beta themselves.  Otherwise g holds alpha = W_alpha h and beta
     * holds b = W_beta h, and the kernels compute per token and value head (layer head
     * index hg = h_v_offset + i):
     *   beta = sigmoid(b),  g = softplus(alpha + dt_bias[hg]) * ssm_a[hg]
     * with softplus(x) = log(1 + e^x) (x itself above 20) and ssm_a = -exp(A_log) as the
     * model stores it (< 0).  dt_bias nullable (0). */
    const float *dt_bias;     /* [layer value heads] ssm_dt */
    const float *ssm_a;       /* [layer value heads] */
} sqmix_gdn_args;

/* sqmix_gdn_decode: the kernel launched immediately before this call on the stream
 * writes neither the state planes nor sel (in a decode step that kernel is the conv
 * front end, sqmix_gdn_conv).  The recurrence then reads its input state before that
 * kernel has finished (programmatic dependent launch), hiding the state load behind
 * it.  Do not set it right after sqmix_gdn_state_copy into these planes.  Ignored by
 * sqmix_gdn_prefill. */
#define SQMIX_GDN_STATE_READY 1

int sqmix_gdn_decode(const sqmix_gdn_args *args, sqmix_stream_t stream);

/* Chunked prefill form of sqmix_gdn_decode for long T (gdn.rs:489-500 over a prompt
 * chunk): the same arguments and results, computed 64 tokens at a time (the
 * chunk-parallel form of the delta rule: a unit lower-triangular solve per chunk and
 * dense chunk products), the last n_snap - 1 tokens recurrently for the snapshot
 * slots.  workspace: sqmix_gdn_prefill_workspace_bytes(n_seqs, T, h_v) bytes, 16-byte
 * aligned, its first 256 bytes zero before first use (a device status word that
 * sqmix_fa_status reads and clears, as for the decode workspace).  The input plane is
 * sel[seq] (or 0); like sqmix_gdn_decode the result planes are 0..n_snap-1. */
size_t sqmix_gdn_prefill_workspace_bytes(int32_t n_seqs, int32_t n_tokens, int32_t h_v);
int sqmix_gdn_prefill(const sqmix_gdn_args *args, void *workspace, size_t workspace_bytes,
                      sqmix_stream_t stream);

/* Copy whole planes: dst[i] <- src[i] for n_planes planes of `plane_elems` f32
 * (the state ggml_cpy of graph.rs:884-912 and get_rows of gdn.rs:445-463 when a
 * caller wants a materialised plane).  Device pointers. */
int sqmix_gdn_state_copy(float *dst, const float *src, int64_t plane_elems, int32_t n_planes,
                         sqmix_stream_t stream);

/* A GDN mixer decode step in ONE launch (T = 1 or 2 tokens per sequence): the front
 * end of sqmix_gdn_conv (short conv + SiLU over the resident history planes, q/k L2
 * norm, history slots), the gate epilogue (beta = sigmoid(b), g = softplus(alpha +
 * dt_bias) * ssm_a, gdn.rs:268-287), the recurrence of sqmix_gdn_decode (plane sel in,
 * planes 0..n_snap-1 out) and norm_gated (rms_norm(o) * norm_weight * silu(z),
 * gdn.rs:150-181), i.e. gdn.rs:290-577 between the projections and the output
 * projection.  Whole layers only (no value-head offset); conv kernel 4; H_v = H_k or
 * 2 H_k; head_dim 128.  Launched as clusters of 4 H_v / H_k CTAs per q/k head, with
 * programmatic stream serialisation; SQMIX_GDN_STATE_READY: the kernel launched just
 * before writes neither the state planes, the conv planes nor sel, and the state is
 * read before waiting for it. */
typedef struct sqmix_gdn_layer_args {
    const void *x;            /* [n_seqs][T][C] qkv_mixed, C = (2 H_k + H_v) * 128 */
    int32_t x_dtype;
    int64_t x_stride_tok;
    int64_t x_stride_seq;
    const float *conv_weight; /* [C][kernel] ssm_conv1d */
    float *conv_state;        /* [n_seqs][n_planes][C][kernel - 1] */
    int32_t kernel;           /* 4 */
    const float *alpha;       /* [n_seqs][T][H_v] W_alpha h */
    const float *beta;        /* [n_seqs][T][H_v] W_beta h (before the sigmoid) */
    const float *dt_bias;     /* nullable [H_v] ssm_dt */
    const float *ssm_a;       /* [H_v] -exp(A_log) */
    float *state;             /* [n_seqs][n_planes][H_v][128][128] */
    int32_t n_planes;
    const int32_t *sel;       /* nullable device I32 [n_seqs]: plane read (state and conv) */
    int32_t n_snap;           /* 1 <= n_snap <= min(T, n_planes) */
    int32_t n_seqs;
    int32_t n_tokens;         /* 1 or 2 */
    int32_t h_k;              /* 16 */
    int32_t h_v;              /* 32 */
    float l2_eps;             /* q/k L2 norm (norm_rms_eps); 0: none */
    const void *z;            /* nullable [n_seqs][T][H_v][128] gate projection */
    int32_t z_dtype;
    int64_t z_stride_tok;
    int64_t z_stride_seq;
    const float *norm_weight; /* nullable: [128] ssm_norm, or per head (stride below) */
    int64_t norm_weight_stride_head; /* 0: one row shared by all heads */
    float norm_eps;           /* norm_rms_eps */
    float *out;               /* [n_seqs][T][H_v][128] f32 */
    int32_t flags;            /* SQMIX_GDN_STATE_READY or 0 */
} sqmix_gdn_layer_args;

int sqmix_gdn_layer_decode(const sqmix_gdn_layer_args *args, sqmix_stream_t stream);

/* ========================================================================
 * GDN front end and the mixers' per-head norms
 * ======================================================================== */

/* Short causal convolution of the GDN qkv projection with its history planes:
 *   conv_input = concat(plane sel[seq] [C][K-1], x^T)          (gdn.rs:290-356)
 *   out[t][c]  = silu(sum_k conv_input[c][t + k] * weight[c][k])
 *                (ggml_ssm_conv + ggml_silu, gdn.rs:358-360)
 * then, when l2_eps > 0, the first n_qk_channels channels (q and k, 2*H_k*d) are
 * L2-normalised per head of head_dim (gdn.rs:436-441), and the history planes are
 * written back: plane s < n_snap <- conv_input rows [max(T - s, 0), +K-1)
 * (plane 0 = the tail; slot s = the history s tokens back, graph.rs:913-961).
 * Conv history: [n_seqs][n_planes][C][K-1] f32, i.e. ggml's [K-1, C, 1+n_rs] per
 * sequence.  The plane read may be among the planes written (updated in place).
 * x, weight, conv_state and out 16-byte aligned; x strides multiples of 4 elements.
 * Launched with programmatic stream serialisation (the taps are read before the wait
 * on the previous kernel; x and the history after it). */
typedef struct sqmix_gdn_conv_args {
    const void *x;            /* [n_seqs][T][C] qkv_mixed (ggml [C, T]) */
    int32_t x_dtype;
    int64_t x_stride_tok;     /* elements between tokens (>= C) */
    int64_t x_stride_seq;     /* elements between sequences */
    const float *weight;      /* [C][K] ssm_conv1d (ggml [K, C]) */
    float *conv_state;        /* [n_seqs][n_planes][C][K-1] */
    int32_t n_planes;
    const int32_t *sel;       /* device I32 [n_seqs]: plane read as history (clamped to
                                 [0, n_planes)); NULL = 0 */
    int32_t n_snap;           /* planes written, 1 <= n_snap <= n_planes */
    int32_t n_seqs;
    int32_t n_tokens;         /* T >= 1 */
    int32_t channels;         /* C = 2*H_k*d + H_v*d (8192), a multiple of head_dim */
    int32_t kernel;           /* K in 2..8 (4: ssm_d_conv) */
    int32_t head_dim;         /* d: 128 (ssm_d_state) */
    int32_t n_qk_channels;    /* leading channels normalised per head (2*H_k*d) */
    float l2_eps;             /* > 0: L2 norm of those channels (norm_rms_eps); 0: none */
    float *out;               /* [n_seqs][T][C] f32 */
} sqmix_gdn_conv_args;

int sqmix_gdn_conv(const sqmix_gdn_conv_args *args, sqmix_stream_t stream);

/* Per-head RMS norm y = x / sqrt(mean(x^2) + eps) over head_dim, then * weight (the
 * per-head Q/K norm of the attention layers, attn.rs:66-84 and :166-175) and
 * * silu(z) (norm_gated of the GDN output, gdn.rs:150-181 and :565-573).
 * x, z [T][H][head_dim] with element strides; out f32.  out may equal x (f32, same
 * strides): each row is read completely before it is written.  head_dim 128 or 256;
 * pointers 16-byte aligned, strides multiples of 4 elements.  Launched with
 * programmatic stream serialisation. */
typedef struct sqmix_head_norm_args {
    const void *x;
    int32_t x_dtype;
    int64_t x_stride_tok;
    int64_t x_stride_head;
    const float *weight;        /* nullable: [head_dim], or per head (weight_stride_head) */
    int64_t weight_stride_head; /* 0: one weight row shared by all heads */
    const void *z;              /* nullable gate */
    int32_t z_dtype;
    int64_t z_stride_tok;
    int64_t z_stride_head;
    int32_t n_tokens;
    int32_t n_heads;
    int32_t head_dim;
    float eps;                  /* norm_rms_eps */
    float *out;
    int64_t out_stride_tok;
    int64_t out_stride_head;
} sqmix_head_norm_args;

int sqmix_head_norm(const sqmix_head_norm_args *args, sqmix_stream_t stream);

/* ------------------------------------------------------------------------
 * Mixer projections: ggml_mul_mat(w, x) (QG / K / V attn.rs:127-129, W_o attn.rs:285;
 * qkv / z / beta / alpha gdn.rs:264-276, out gdn.rs:577):
 *   y[t * y_stride + o] = sum_i W[o][i] * x[t * x_stride + i]
 * for o < n_out, i < n_in, t < n_tokens.  W is ggml's [n_in, n_out] weight tensor: n_out
 * contiguous rows (w_row_bytes = sqmix_mul_mat_row_bytes(w_type, n_in)) in a GGUF block
 * format -- SQMIX_Q8_0, SQMIX_Q4_K, SQMIX_Q6_K -- or SQMIX_F32 / F16 / BF16 elements;
 * 16-byte aligned, n_in a multiple of 256 up to 4096 (q6_K: a multiple of 2048).  x is
 * f32 / f16 / bf16, y f32.  Two forms:
 *   - decode (n_tokens below the prefill threshold): each stream of W serves up to 4
 *     tokens; dequantised weights times x summed f32-exactly (ggml's CUDA backend
 *     quantises x to q8_1 for its quantised dot products; this is the more exact form);
 *   - prefill (n_tokens >= 128; >= 48 when the call has at least 48 tiles of 128 rows x
 *     128 tokens, >= 16 with at least 96; x rows 16-byte aligned): a tensor-core GEMM whose operands are
 *     tf32 for f32 x (weights and x truncated to a 10-bit mantissa) or x's 16-bit type,
 *     sums in f32 -- about 1e-3 of max |y|, as ggml's dequantise-to-16-bit GEMM path.
 * The weights are read before the call's dependency on the previous kernel on the
 * stream (programmatic dependent launch): W must not be written by that kernel.
 * `status` (device, may be NULL) receives bit 1 if a bounded wait of the kernel gave up.
 * ------------------------------------------------------------------------ */
typedef struct sqmix_mul_mat_args {
    const void *w;
    int32_t w_type;
    int64_t w_row_bytes;
    int64_t n_in;
    int64_t n_out;
    const void *x;
    int32_t x_dtype;
    int64_t x_stride;  /* elements between tokens of x */
    int32_t n_tokens;
    float *y;
    int64_t y_stride;  /* elements between tokens of y */
    uint32_t *status;
} sqmix_mul_mat_args;

/* Bytes of one weight row of n_in values in w_type (0: unsupported type or length). */
int64_t sqmix_mul_mat_row_bytes(int32_t w_type, int64_t n_in);
int sqmix_mul_mat(const sqmix_mul_mat_args *args, sqmix_stream_t stream);

/* A group of projections of the same x -- a layer's QG / K / V (attn.rs:127-129), or its
 * qkv / z / beta / alpha (gdn.rs:264-276) -- in one pass over x: args[0 .. n) must agree
 * on x, x_dtype, x_stride, n_tokens and n_in; each has its own w, w_type, n_out and y
 * (y must not overlap x).  The group is one launch per 4 tokens.  Bounded-wait
 * failures go to args[0].status.  Same results, to the bit, as one sqmix_mul_mat per
 * entry. */
#define SQMIX_MUL_MAT_MAX_GROUP 8
int sqmix_mul_mat_group(const sqmix_mul_mat_args *args, int32_t n, sqmix_stream_t stream);

/* ========================================================================
 * ggml custom-op bridge
 *
 * sqwen executes one ggml graph per step and replays it as a CUDA graph
 * (src/engine/runner.rs:362-389); its FFI enumerates ggml's custom ops
 * (GGML_OP_MAP_CUSTOM1..3, GGML_OP_CUSTOM: src/backend/ffi.rs:199-202).  The callbacks
 * below have ggml's custom-op signature (ggml_custom_op_t: dst, thread ith of nth,
 * userdata) so that a graph node built with ggml_custom_4d can run a sqmix kernel on
 * the node's tensors: dst and its sources are read through ggml's tensor layout (the
 * struct ggml_tensor that sqwen's FFI mirrors at src/backend/ffi.rs:22-39: type, ne[4],
 * nb[4] in bytes, src[10], data), the kernel is launched by thread 0 on the stream in
 * the userdata, and the status is stored there (the callback returns void).  Positions
 * and lengths come from a device tensor, so a replayed graph stays correct with fixed
 * pointers.  sqmix_ggml_*_args only translate a node into the argument struct (no CUDA
 * call), for checking a graph's wiring.
 *
 * FA decode node (the tensors of ggml_flash_attn_ext, attn.rs:238-249):
 *   dst    F32 [256, 16, T]  output (gated if src[4] is set)
 *   src[0] Q   [256, T, 16]  F32 / F16 / BF16, any token and head strides (nb[0] = element)
 *   src[1] K   tiled q4_0 cache as a Q4_0 tensor [512, capacity] (the bytes of ggml's
 *              [n_embd_k_gqa, cap] q4_0 cache, kv.rs:124-134, in sqmix's tiled order)
 *   src[2] V   likewise
 *   src[3] I64 [2] device {n_kv, q_pos0}
 *   src[4] gate [256, 16, T] or NULL
 *   src[5] k_new, src[6] v_new: [256, 2, n_new] rows to append (both or neither)
 * GDN decode node (ggml_gated_delta_net, gdn.rs:489-500):
 *   dst    F32 [128, H_v, T, n_seqs]
 *   src[0] q [128, H_k, T, n_seqs], src[1] k (same layout), src[2] v [128, H_v, T, n_seqs]
 *          (F32 / F16 / BF16, heads contiguous)
 *   src[3] g, src[4] beta: F32 [1, H_v, T, n_seqs] contiguous (raw alpha / b when the
 *          op's ssm_a is set)
 *   src[5] state F32 [128*128*H_v, n_planes, n_seqs]; src[6] sel I32 [n_seqs] or NULL
 * ======================================================================== */
struct ggml_tensor;

typedef struct sqmix_ggml_fa_op {
    float scale;
    int32_t rope_n_rot;
    float rope_freq_base;
    int64_t rope_pos_offset;
    int32_t n_splits;         /* 0: the default of the configuration */
    int32_t config;
    int32_t flags;            /* SQMIX_FA_* */
    const float *q_norm;      /* nullable */
    const float *k_norm;      /* nullable */
    float norm_eps;
    void *workspace;          /* NULL: sqmix_fa_decode_noalloc (no allocation in the callback) */
    size_t workspace_bytes;
    sqmix_stream_t stream;    /* the stream the graph runs on */
    int32_t status;           /* out: SQMIX_OK or the error of the last call */
} sqmix_ggml_fa_op;

typedef struct sqmix_ggml_gdn_op {
    int32_t n_snap;
    float l2_eps;
    int32_t flags;            /* SQMIX_GDN_* */
    int32_t h_v_offset;
    const float *dt_bias;     /* nullable */
    const float *ssm_a;       /* nullable: g, beta are the log-decay and beta themselves */
    sqmix_stream_t stream;
    int32_t status;           /* out */
} sqmix_ggml_gdn_op;

int sqmix_ggml_fa_args(const struct ggml_tensor *dst, const sqmix_ggml_fa_op *op, sqmix_fa_args *out);
int sqmix_ggml_gdn_args(const struct ggml_tensor *dst, const sqmix_ggml_gdn_op *op, sqmix_gdn_args *out);
/* ggml_custom_op_t callbacks; userdata is the sqmix_ggml_*_op of the node. */
void sqmix_ggml_fa_decode_op(struct ggml_tensor *dst, int ith, int nth, void *userdata);
void sqmix_ggml_gdn_decode_op(struct ggml_tensor *dst, int ith, int nth, void *userdata);
/* Byte size of the ggml tensor struct the bridge reads (336 on 64-bit hosts). */
size_t sqmix_ggml_tensor_bytes(void);

/* ========================================================================
 * Host-side state objects (the engine's bookkeeping, in C++)
 * ======================================================================== */

/* KvCache (kv.rs:67-448): per-layer tiled q4_0 K/V caches + shared cursor. */
typedef struct sqmix_kvcache sqmix_kvcache;

int sqmix_kvcache_create(int32_t n_layers, int64_t kv_cap, int32_t device, sqmix_kvcache **out);
void sqmix_kvcache_destroy(sqmix_kvcache *kv);
int sqmix_kvcache_zero(sqmix_kvcache *kv, sqmix_stream_t stream);       /* kv.rs:160-170 */
int sqmix_kvcache_begin_step(sqmix_kvcache *kv, int32_t n_tokens);    /* kv.rs:239-253 */
int sqmix_kvcache_rewind_to(sqmix_kvcache *kv, int64_t pos);          /* kv.rs:284-297 */
void sqmix_kvcache_reset(sqmix_kvcache *kv);                           /* kv.rs:274-278 */
int64_t sqmix_kvcache_n_used(const sqmix_kvcache *kv);
int64_t sqmix_kvcache_step_start(const sqmix_kvcache *kv);
int64_t sqmix_kvcache_n_kv_padded(const sqmix_kvcache *kv);           /* kv.rs:224-226 */
int64_t sqmix_kvcache_capacity(const sqmix_kvcache *kv);              /* logical kv_cap */
int64_t sqmix_kvcache_capacity_alloc(const sqmix_kvcache *kv);        /* padded to 256 */
size_t sqmix_kvcache_bytes_per_token(const sqmix_kvcache *kv);        /* kv.rs:179-189 */
void *sqmix_kvcache_k(sqmix_kvcache *kv, int32_t layer);
void *sqmix_kvcache_v(sqmix_kvcache *kv, int32_t layer);
/* Device I64 block {n_kv, q_pos0, rows[0..max_tokens)} for the current step;
 * refreshed by sqmix_kvcache_upload_step (one async H2D from pinned memory,
 * the analogue of fill_inputs, graph.rs:394-428). */
const int64_t *sqmix_kvcache_device_step(const sqmix_kvcache *kv);
int sqmix_kvcache_upload_step(sqmix_kvcache *kv, sqmix_stream_t stream);
int32_t sqmix_kvcache_max_step_tokens(const sqmix_kvcache *kv);

/* GdnState (gdn.rs:71-120) for n_layers GDN layers: 1 + n_rs planes per layer of the
 * recurrent state ([h_v][128][128] f32) and, when conv_channels > 0, of the short-conv
 * history ([conv_channels][d_conv - 1] f32, taps fastest: the conv_state tensor
 * [d_conv - 1, conv_channels, 1 + n_rs] of gdn.rs:76-104 and the state layout of
 * sqmix_gdn_conv).  sqmix_gdnstate_create has no conv history. */
typedef struct sqmix_gdnstate sqmix_gdnstate;

int sqmix_gdnstate_create(int32_t n_layers, int32_t h_v, int32_t n_rs, int32_t device,
                          sqmix_gdnstate **out);
int sqmix_gdnstate_create_conv(int32_t n_layers, int32_t h_v, int32_t n_rs, int32_t conv_channels,
                               int32_t d_conv, int32_t device, sqmix_gdnstate **out);
/* conv history planes of a layer (NULL without conv history) */
float *sqmix_gdnstate_conv_planes(sqmix_gdnstate *st, int32_t layer);
void sqmix_gdnstate_destroy(sqmix_gdnstate *st);
int sqmix_gdnstate_zero(sqmix_gdnstate *st, sqmix_stream_t stream);   /* graph.rs:206-222 */
float *sqmix_gdnstate_planes(sqmix_gdnstate *st, int32_t layer);
int32_t sqmix_gdnstate_n_planes(const sqmix_gdnstate *st);
/* set_recurrent_sel (graph.rs:190-196): clamps to n_rs; one-shot, consumed by the
 * next upload.  Returns the stored value. */
int32_t sqmix_gdnstate_set_sel(sqmix_gdnstate *st, int32_t sel);
int32_t sqmix_gdnstate_sel(const sqmix_gdnstate *st);
const int32_t *sqmix_gdnstate_device_sel(const sqmix_gdnstate *st);
int sqmix_gdnstate_upload_sel(sqmix_gdnstate *st, sqmix_stream_t stream);
/* Checkpoint of plane 0 of every layer in the byte layout of snapshot_gdn /
 * restore_gdn (graph.rs:301-350), which prompt-cache checkpoints store
 * (prompt_cache.rs:38-48): a u64 little-endian payload length, then per layer the raw
 * f32 state plane 0 followed by the conv history plane 0 (absent without conv
 * history).  snapshot: D2H + stream sync; restore rejects a length mismatch. */
size_t sqmix_gdnstate_snapshot_bytes(const sqmix_gdnstate *st);
int sqmix_gdnstate_snapshot(sqmix_gdnstate *st, void *host_buf, size_t bytes, sqmix_stream_t stream);
int sqmix_gdnstate_restore(sqmix_gdnstate *st, const void *host_buf, size_t bytes,
                           sqmix_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* SQMIX_H */
