"""sqmix: B200 (sm_100a) attention-mixer kernels for qwen35moe behind a C ABI.

The CUDA kernels and the engine-side state objects live in libsqmix.so
(include/sqmix.h); this package is the Python mirror of that interface, used by
the tests and the benchmark.  See ops.py (kernel entry points) and state.py
(KvCache, GdnState).
"""
from ._lib import (SQMIX_BF16, SQMIX_EINVAL, SQMIX_ENOSPC, SQMIX_EOVERFLOW, SQMIX_ERANGE, SQMIX_F16,
                   SQMIX_F32, SQMIX_MUL_MAT_MAX_GROUP, SQMIX_OK, SQMIX_Q4_K, SQMIX_Q6_K, SQMIX_Q8_0, SqmixError, exported_symbols, lib)
from .ops import (GDN_D, HEAD_DIM, KV_PAD, N_HEAD, N_HEAD_KV, attn_merge_lse, fa_status, fa_workspace_bytes,
                  flash_attn_ext, flash_attn_prefill, flash_attn_decode_batch, fa_batch_workspace_bytes, fa_prefill_workspace_bytes,
                  new_fa_prefill_workspace, gated_delta_net, gdn_conv, gdn_layer_decode, gdn_prefill_workspace_bytes,
                  gdn_state_copy,
                  head_norm, kv_cache_bytes, kv_convert_rows, mul_mat, mul_mat_group, mul_mat_row_bytes, new_fa_workspace, new_kv_cache,
                  set_rows_q4_0)
from .state import GdnState, KvCache

__all__ = [
    "SqmixError", "lib", "exported_symbols", "KvCache", "GdnState", "set_rows_q4_0", "flash_attn_ext",
    "attn_merge_lse", "fa_status", "flash_attn_prefill", "flash_attn_decode_batch", "fa_batch_workspace_bytes", "fa_prefill_workspace_bytes",
    "new_fa_prefill_workspace", "gdn_prefill_workspace_bytes", "gated_delta_net", "gdn_state_copy", "gdn_conv", "gdn_layer_decode", "head_norm", "kv_convert_rows", "kv_cache_bytes",
    "new_kv_cache", "new_fa_workspace", "fa_workspace_bytes", "HEAD_DIM", "N_HEAD", "N_HEAD_KV", "GDN_D",
    "KV_PAD", "SQMIX_OK", "SQMIX_EINVAL", "SQMIX_ENOSPC", "SQMIX_EOVERFLOW", "SQMIX_ERANGE", "SQMIX_F32",
    "SQMIX_F16", "SQMIX_BF16", "SQMIX_Q8_0", "SQMIX_Q4_K", "SQMIX_Q6_K", "SQMIX_MUL_MAT_MAX_GROUP", "mul_mat", "mul_mat_group", "mul_mat_row_bytes",
]
