"""ctypes binding of libsqmix.so (declared in include/sqmix.h).

The library is built in-tree by ``sqwen-moe-3090_b200/build.py``.  There is no
fallback: if the shared library is missing or fails to load, every entry point
raises, so a GPU run can never silently take another code path.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsqmix.so")

SQMIX_OK = 0
SQMIX_EINVAL = -1
SQMIX_ECUDA = -2
SQMIX_ETIMEOUT = -3
SQMIX_ENOSPC = -4
SQMIX_EOVERFLOW = -5
SQMIX_ERANGE = -6

SQMIX_F32 = 0
SQMIX_F16 = 1
SQMIX_BF16 = 30
SQMIX_MUL_MAT_MAX_GROUP = 8  # projections of one sqmix_mul_mat_group call
SQMIX_Q8_0 = 8  # weight block formats of sqmix_mul_mat
SQMIX_Q4_K = 12
SQMIX_Q6_K = 14
SQMIX_FA_OVERLAP_PREV = 1

# struct ids of the library's ABI layout table (sqmix_abi_struct_size & co.)
SQMIX_ABI_KV_APPEND_ARGS = 1
SQMIX_ABI_FA_ARGS = 2
SQMIX_ABI_FA_BATCH_ARGS = 3
SQMIX_ABI_PEER_MERGE_ARGS = 4
SQMIX_ABI_GDN_ARGS = 5
SQMIX_ABI_GDN_CONV_ARGS = 6
SQMIX_ABI_HEAD_NORM_ARGS = 7
SQMIX_ABI_GDN_LAYER_ARGS = 8
SQMIX_ABI_GGML_FA_OP = 9
SQMIX_ABI_GGML_GDN_OP = 10
SQMIX_ABI_MUL_MAT_ARGS = 11

ERROR_NAMES = {
    SQMIX_EINVAL: "SQMIX_EINVAL",
    SQMIX_ECUDA: "SQMIX_ECUDA",
    SQMIX_ETIMEOUT: "SQMIX_ETIMEOUT",
    SQMIX_ENOSPC: "SQMIX_ENOSPC",
    SQMIX_EOVERFLOW: "SQMIX_EOVERFLOW",
    SQMIX_ERANGE: "SQMIX_ERANGE",
}


class SqmixError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{ERROR_NAMES.get(code, code)}: {msg}")
        self.code = code


c_void_p = ctypes.c_void_p
c_int32 = ctypes.c_int32
c_int64 = ctypes.c_int64
c_float = ctypes.c_float
c_size_t = ctypes.c_size_t


class KvAppendArgs(ctypes.Structure):
    _fields_ = [
        ("k", c_void_p), ("v", c_void_p), ("dtype", c_int32),
        ("k_stride_tok", c_int64), ("v_stride_tok", c_int64), ("n_tokens", c_int32),
        ("rows", c_void_p), ("k_cache", c_void_p), ("v_cache", c_void_p), ("capacity", c_int64),
        ("rope_n_rot", c_int32), ("rope_freq_base", c_float), ("rope_pos_offset", c_int64),
    ]


class FaArgs(ctypes.Structure):
    _fields_ = [
        ("q", c_void_p), ("q_dtype", c_int32), ("q_stride_tok", c_int64), ("q_stride_head", c_int64),
        ("gate", c_void_p), ("gate_dtype", c_int32), ("gate_stride_tok", c_int64),
        ("gate_stride_head", c_int64),
        ("k_cache", c_void_p), ("v_cache", c_void_p), ("capacity", c_int64),
        ("n_kv", c_void_p), ("q_pos0", c_void_p), ("n_q", c_int32), ("scale", c_float),
        ("rope_n_rot", c_int32), ("rope_freq_base", c_float), ("rope_pos_offset", c_int64),
        ("out", c_void_p), ("lse", c_void_p), ("workspace", c_void_p), ("workspace_bytes", c_size_t),
        ("n_splits", c_int32), ("config", c_int32),
        ("k_new", c_void_p), ("v_new", c_void_p), ("kv_new_dtype", c_int32), ("k_new_stride_tok", c_int64),
        ("v_new_stride_tok", c_int64), ("n_new", c_int32), ("flags", c_int32),
        ("q_norm", c_void_p), ("k_norm", c_void_p), ("norm_eps", c_float),
    ]


class FaBatchArgs(ctypes.Structure):
    _fields_ = [
        ("n_seqs", c_int32), ("q", c_void_p), ("q_dtype", c_int32), ("q_stride_seq", c_int64),
        ("q_stride_head", c_int64), ("gate", c_void_p), ("gate_dtype", c_int32), ("gate_stride_seq", c_int64),
        ("gate_stride_head", c_int64), ("k_caches", c_void_p), ("v_caches", c_void_p), ("capacities", c_void_p),
        ("n_kv", c_void_p), ("q_pos0", c_void_p), ("scale", c_float), ("rope_n_rot", c_int32),
        ("rope_freq_base", c_float), ("out", c_void_p), ("lse", c_void_p), ("workspace", c_void_p),
        ("workspace_bytes", c_size_t), ("splits_per_seq", c_int32), ("k_new", c_void_p), ("v_new", c_void_p),
        ("kv_new_dtype", c_int32), ("new_stride_seq", c_int64), ("n_new", c_int32), ("flags", c_int32),
    ]


class PeerMergeArgs(ctypes.Structure):
    _fields_ = [
        ("n_ranks", c_int32), ("rank", c_int32), ("slot", c_int32), ("n_slots", c_int32), ("rows", c_int32),
        ("buffers", c_void_p), ("o_local", c_void_p), ("lse_local", c_void_p), ("gate", c_void_p),
        ("out", c_void_p), ("lse_out", c_void_p), ("status", c_void_p),
    ]


class GdnArgs(ctypes.Structure):
    _fields_ = [
        ("q", c_void_p), ("k", c_void_p), ("v", c_void_p), ("dtype", c_int32),
        ("qk_stride_tok", c_int64), ("v_stride_tok", c_int64), ("qk_stride_seq", c_int64),
        ("v_stride_seq", c_int64), ("g", c_void_p), ("beta", c_void_p), ("state", c_void_p),
        ("n_planes", c_int32), ("sel", c_void_p), ("n_seqs", c_int32), ("n_tokens", c_int32),
        ("h_k", c_int32), ("h_v", c_int32), ("n_snap", c_int32), ("l2_eps", c_float),
        ("out", c_void_p), ("flags", c_int32), ("h_v_offset", c_int32), ("dt_bias", c_void_p),
        ("ssm_a", c_void_p),
    ]


class GdnConvArgs(ctypes.Structure):
    _fields_ = [
        ("x", c_void_p), ("x_dtype", c_int32), ("x_stride_tok", c_int64), ("x_stride_seq", c_int64),
        ("weight", c_void_p), ("conv_state", c_void_p), ("n_planes", c_int32), ("sel", c_void_p),
        ("n_snap", c_int32), ("n_seqs", c_int32), ("n_tokens", c_int32), ("channels", c_int32),
        ("kernel", c_int32), ("head_dim", c_int32), ("n_qk_channels", c_int32), ("l2_eps", c_float),
        ("out", c_void_p),
    ]


class HeadNormArgs(ctypes.Structure):
    _fields_ = [
        ("x", c_void_p), ("x_dtype", c_int32), ("x_stride_tok", c_int64), ("x_stride_head", c_int64),
        ("weight", c_void_p), ("weight_stride_head", c_int64), ("z", c_void_p), ("z_dtype", c_int32),
        ("z_stride_tok", c_int64), ("z_stride_head", c_int64), ("n_tokens", c_int32), ("n_heads", c_int32),
        ("head_dim", c_int32), ("eps", c_float), ("out", c_void_p), ("out_stride_tok", c_int64),
        ("out_stride_head", c_int64),
    ]


class GdnLayerArgs(ctypes.Structure):
    _fields_ = [
        ("x", c_void_p), ("x_dtype", c_int32), ("x_stride_tok", c_int64), ("x_stride_seq", c_int64),
        ("conv_weight", c_void_p), ("conv_state", c_void_p), ("kernel", c_int32), ("alpha", c_void_p),
        ("beta", c_void_p), ("dt_bias", c_void_p), ("ssm_a", c_void_p), ("state", c_void_p),
        ("n_planes", c_int32), ("sel", c_void_p), ("n_snap", c_int32), ("n_seqs", c_int32),
        ("n_tokens", c_int32), ("h_k", c_int32), ("h_v", c_int32), ("l2_eps", c_float), ("z", c_void_p),
        ("z_dtype", c_int32), ("z_stride_tok", c_int64), ("z_stride_seq", c_int64), ("norm_weight", c_void_p),
        ("norm_weight_stride_head", c_int64), ("norm_eps", c_float), ("out", c_void_p), ("flags", c_int32),
    ]


class GgmlFaOp(ctypes.Structure):
    _fields_ = [
        ("scale", c_float), ("rope_n_rot", c_int32), ("rope_freq_base", c_float), ("rope_pos_offset", c_int64),
        ("n_splits", c_int32), ("config", c_int32), ("flags", c_int32), ("q_norm", c_void_p), ("k_norm", c_void_p),
        ("norm_eps", c_float), ("workspace", c_void_p), ("workspace_bytes", c_size_t), ("stream", c_void_p),
        ("status", c_int32),
    ]


class GgmlGdnOp(ctypes.Structure):
    _fields_ = [
        ("n_snap", c_int32), ("l2_eps", c_float), ("flags", c_int32), ("h_v_offset", c_int32), ("dt_bias", c_void_p),
        ("ssm_a", c_void_p), ("stream", c_void_p), ("status", c_int32),
    ]


class MulMatArgs(ctypes.Structure):
    _fields_ = [
        ("w", c_void_p), ("w_type", c_int32), ("w_row_bytes", c_int64), ("n_in", c_int64), ("n_out", c_int64),
        ("x", c_void_p), ("x_dtype", c_int32), ("x_stride", c_int64), ("n_tokens", c_int32), ("y", c_void_p),
        ("y_stride", c_int64), ("status", c_void_p),
    ]


class GgmlTensor(ctypes.Structure):
    """ggml's struct ggml_tensor as sqwen's FFI declares it (src/backend/ffi.rs:22-39);
    used to build graph nodes for the custom-op bridge."""


GgmlTensor._fields_ = [
    ("type", c_int32), ("buffer", c_void_p), ("ne", c_int64 * 4), ("nb", c_size_t * 4), ("op", c_int32),
    ("op_params", c_int32 * 16), ("flags", c_int32), ("src", ctypes.POINTER(GgmlTensor) * 10),
    ("view_src", ctypes.POINTER(GgmlTensor)), ("view_offs", c_size_t), ("data", c_void_p), ("name", ctypes.c_char * 64),
    ("extra", c_void_p), ("padding", ctypes.c_char * 8),
]


# name -> (restype, argtypes)
_SIGNATURES = {
    "sqmix_version": (ctypes.c_char_p, []),
    "sqmix_last_error": (ctypes.c_char_p, []),
    "sqmix_device_sm_count": (ctypes.c_int, [ctypes.c_int]),
    "sqmix_abi_struct_size": (c_size_t, [c_int32]),
    "sqmix_abi_field_count": (c_int32, [c_int32]),
    "sqmix_abi_field_offset": (c_int64, [c_int32, c_int32]),
    "sqmix_kv_cache_bytes": (c_size_t, [c_int64]),
    "sqmix_kv_append_q4_0": (ctypes.c_int, [ctypes.POINTER(KvAppendArgs), c_void_p]),
    "sqmix_kv_convert_rows": (ctypes.c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int32,
                                             c_int32, c_void_p]),
    "sqmix_fa_workspace_bytes": (c_size_t, [c_int32, c_int32]),
    "sqmix_fa_decode": (ctypes.c_int, [ctypes.POINTER(FaArgs), c_void_p]),
    "sqmix_fa_status": (ctypes.c_int, [c_void_p, c_void_p]),
    "sqmix_fa_decode_noalloc": (ctypes.c_int, [ctypes.POINTER(FaArgs), c_void_p]),
    "sqmix_fa_noalloc_status": (ctypes.c_int, [c_void_p]),
    "sqmix_fa_prefill_workspace_bytes": (c_size_t, [c_int32, c_int32]),
    "sqmix_fa_prefill": (ctypes.c_int, [ctypes.POINTER(FaArgs), c_void_p]),
    "sqmix_gdn_prefill_workspace_bytes": (c_size_t, [c_int32, c_int32, c_int32]),
    "sqmix_fa_batch_workspace_bytes": (c_size_t, [c_int32, c_int32]),
    "sqmix_peer_buffer_bytes": (c_size_t, [c_int32]),
    "sqmix_peer_buffer_create": (ctypes.c_int, [c_int32, ctypes.POINTER(c_void_p), c_void_p]),
    "sqmix_peer_buffer_open": (ctypes.c_int, [c_void_p, ctypes.POINTER(c_void_p)]),
    "sqmix_peer_buffer_close": (ctypes.c_int, [c_void_p]),
    "sqmix_peer_buffer_destroy": (ctypes.c_int, [c_void_p]),
    "sqmix_peer_buffer_reset": (ctypes.c_int, [c_void_p, c_int32, c_void_p]),
    "sqmix_attn_merge_peers": (ctypes.c_int, [ctypes.POINTER(PeerMergeArgs), c_void_p]),
    "sqmix_fa_decode_peers": (ctypes.c_int, [ctypes.POINTER(FaArgs), ctypes.POINTER(PeerMergeArgs), c_void_p]),
    "sqmix_fa_decode_batch": (ctypes.c_int, [ctypes.POINTER(FaBatchArgs), c_void_p]),
    "sqmix_gdn_prefill": (ctypes.c_int, [ctypes.POINTER(GdnArgs), c_void_p, c_size_t, c_void_p]),
    "sqmix_attn_merge_lse": (ctypes.c_int, [c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_void_p,
                                            c_void_p, c_void_p]),
    "sqmix_gdn_decode": (ctypes.c_int, [ctypes.POINTER(GdnArgs), c_void_p]),
    "sqmix_gdn_state_copy": (ctypes.c_int, [c_void_p, c_void_p, c_int64, c_int32, c_void_p]),
    "sqmix_gdn_conv": (ctypes.c_int, [ctypes.POINTER(GdnConvArgs), c_void_p]),
    "sqmix_head_norm": (ctypes.c_int, [ctypes.POINTER(HeadNormArgs), c_void_p]),
    "sqmix_gdn_layer_decode": (ctypes.c_int, [ctypes.POINTER(GdnLayerArgs), c_void_p]),
    "sqmix_mul_mat_row_bytes": (c_int64, [c_int32, c_int64]),
    "sqmix_mul_mat": (ctypes.c_int, [ctypes.POINTER(MulMatArgs), c_void_p]),
    "sqmix_mul_mat_group": (ctypes.c_int, [ctypes.POINTER(MulMatArgs), c_int32, c_void_p]),
    "sqmix_ggml_fa_args": (ctypes.c_int, [ctypes.POINTER(GgmlTensor), ctypes.POINTER(GgmlFaOp), ctypes.POINTER(FaArgs)]),
    "sqmix_ggml_gdn_args": (ctypes.c_int, [ctypes.POINTER(GgmlTensor), ctypes.POINTER(GgmlGdnOp),
                                           ctypes.POINTER(GdnArgs)]),
    "sqmix_ggml_fa_decode_op": (None, [ctypes.POINTER(GgmlTensor), ctypes.c_int, ctypes.c_int, c_void_p]),
    "sqmix_ggml_gdn_decode_op": (None, [ctypes.POINTER(GgmlTensor), ctypes.c_int, ctypes.c_int, c_void_p]),
    "sqmix_ggml_tensor_bytes": (c_size_t, []),
    "sqmix_kvcache_create": (ctypes.c_int, [c_int32, c_int64, c_int32, ctypes.POINTER(c_void_p)]),
    "sqmix_kvcache_destroy": (None, [c_void_p]),
    "sqmix_kvcache_zero": (ctypes.c_int, [c_void_p, c_void_p]),
    "sqmix_kvcache_begin_step": (ctypes.c_int, [c_void_p, c_int32]),
    "sqmix_kvcache_rewind_to": (ctypes.c_int, [c_void_p, c_int64]),
    "sqmix_kvcache_reset": (None, [c_void_p]),
    "sqmix_kvcache_n_used": (c_int64, [c_void_p]),
    "sqmix_kvcache_step_start": (c_int64, [c_void_p]),
    "sqmix_kvcache_n_kv_padded": (c_int64, [c_void_p]),
    "sqmix_kvcache_capacity": (c_int64, [c_void_p]),
    "sqmix_kvcache_capacity_alloc": (c_int64, [c_void_p]),
    "sqmix_kvcache_bytes_per_token": (c_size_t, [c_void_p]),
    "sqmix_kvcache_k": (c_void_p, [c_void_p, c_int32]),
    "sqmix_kvcache_v": (c_void_p, [c_void_p, c_int32]),
    "sqmix_kvcache_device_step": (c_void_p, [c_void_p]),
    "sqmix_kvcache_upload_step": (ctypes.c_int, [c_void_p, c_void_p]),
    "sqmix_kvcache_max_step_tokens": (c_int32, [c_void_p]),
    "sqmix_gdnstate_create": (ctypes.c_int, [c_int32, c_int32, c_int32, c_int32, ctypes.POINTER(c_void_p)]),
    "sqmix_gdnstate_create_conv": (ctypes.c_int, [c_int32, c_int32, c_int32, c_int32, c_int32, c_int32,
                                                  ctypes.POINTER(c_void_p)]),
    "sqmix_gdnstate_conv_planes": (c_void_p, [c_void_p, c_int32]),
    "sqmix_gdnstate_destroy": (None, [c_void_p]),
    "sqmix_gdnstate_zero": (ctypes.c_int, [c_void_p, c_void_p]),
    "sqmix_gdnstate_planes": (c_void_p, [c_void_p, c_int32]),
    "sqmix_gdnstate_n_planes": (c_int32, [c_void_p]),
    "sqmix_gdnstate_set_sel": (c_int32, [c_void_p, c_int32]),
    "sqmix_gdnstate_sel": (c_int32, [c_void_p]),
    "sqmix_gdnstate_device_sel": (c_void_p, [c_void_p]),
    "sqmix_gdnstate_upload_sel": (ctypes.c_int, [c_void_p, c_void_p]),
    "sqmix_gdnstate_snapshot_bytes": (c_size_t, [c_void_p]),
    "sqmix_gdnstate_snapshot": (ctypes.c_int, [c_void_p, c_void_p, c_size_t, c_void_p]),
    "sqmix_gdnstate_restore": (ctypes.c_int, [c_void_p, c_void_p, c_size_t, c_void_p]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """Load libsqmix.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python sqwen-moe-3090_b200/build.py` "
                "(there is no CPU fallback for the sqmix kernels)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def check(rc: int, what: str = "") -> None:
    if rc != SQMIX_OK:
        msg = lib().sqmix_last_error().decode(errors="replace")
        raise SqmixError(rc, f"{what}: {msg}" if what else msg)
