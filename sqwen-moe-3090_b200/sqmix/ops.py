"""Kernel entry points over torch tensors (thin wrappers of the sqmix C ABI).

Names follow the ggml nodes they replace on sqwen's attention-mixer path:

  set_rows_q4_0    <- ggml_set_rows into the q4_0 KV cache (src/engine/kv.rs:367-396),
                      with ggml_rope_multi on K fused in (src/model/attn.rs:183-204)
  flash_attn_ext   <- ggml_flash_attn_ext (src/model/attn.rs:238-249) + the sigmoid
                      gate (attn.rs:282-283), split-KV decode for 1-2 query tokens
  attn_merge_lse   <- merge of split-KV partials that live on different GPUs
  gated_delta_net  <- ggml_gated_delta_net (src/model/gdn.rs:489-500) with the
                      snapshot write-back (src/model/graph.rs:884-912) and plane
                      select (gdn.rs:445-463) done in place
  mul_mat          <- ggml_mul_mat of the mixer projections on GGUF weights
                      (src/model/attn.rs:127-129, 285; src/model/gdn.rs:264-276, 577)

Every function launches on torch's current CUDA stream and raises SqmixError on a
non-zero status, mirroring how the reference turns ggml failures into Err.
"""
from __future__ import annotations

import ctypes
import math

import torch

from ._lib import (SQMIX_BF16, SQMIX_F16, SQMIX_F32, SQMIX_FA_OVERLAP_PREV, SQMIX_MUL_MAT_MAX_GROUP, FaArgs, FaBatchArgs, GdnArgs, GdnConvArgs,
                   GdnLayerArgs, HeadNormArgs, KvAppendArgs, MulMatArgs, check, lib)

HEAD_DIM = 256
N_HEAD = 16
N_HEAD_KV = 2
GDN_D = 128
KV_PAD = 256

_DTYPES = {torch.float32: SQMIX_F32, torch.float16: SQMIX_F16, torch.bfloat16: SQMIX_BF16}


def _dt(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError as e:
        raise TypeError(f"unsupported dtype {t.dtype}") from e


def _ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(stream=None):
    if stream is None:
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream)


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("sqmix kernels take CUDA tensors (there is no CPU path)")


def kv_cache_bytes(capacity: int) -> int:
    return int(lib().sqmix_kv_cache_bytes(int(capacity)))


def new_kv_cache(capacity: int, device="cuda") -> torch.Tensor:
    """A zeroed tiled q4_0 cache (one of K or V) for `capacity` rows."""
    if capacity % KV_PAD:
        raise ValueError(f"capacity must be a multiple of {KV_PAD}")
    return torch.zeros(kv_cache_bytes(capacity), dtype=torch.uint8, device=device)


def set_rows_q4_0(k: torch.Tensor, v: torch.Tensor, rows: torch.Tensor, k_cache: torch.Tensor,
                  v_cache: torch.Tensor, capacity: int, rope_n_rot: int = 0,
                  rope_freq_base: float = 1e7, rope_pos_offset: int = 0, stream=None) -> None:
    """Quantise new K/V rows [T][2][256] to q4_0 and write them at rows[t] (I64, device)."""
    _require_cuda(k, v, rows, k_cache, v_cache)
    if k.dim() == 2:
        k = k.view(k.shape[0], N_HEAD_KV, HEAD_DIM)
    if v.dim() == 2:
        v = v.view(v.shape[0], N_HEAD_KV, HEAD_DIM)
    if k.stride(-1) != 1 or k.stride(-2) != HEAD_DIM or v.stride(-1) != 1 or v.stride(-2) != HEAD_DIM:
        raise ValueError("each token's K/V must be 2 x 256 contiguous values")
    if k.dtype != v.dtype:
        raise TypeError("k and v must share a dtype")
    if rows.dtype != torch.int64 or rows.numel() != k.shape[0]:
        raise ValueError("rows must be int64 [T]")
    a = KvAppendArgs(
        k=_ptr(k), v=_ptr(v), dtype=_dt(k), k_stride_tok=k.stride(0), v_stride_tok=v.stride(0),
        n_tokens=k.shape[0], rows=_ptr(rows), k_cache=_ptr(k_cache), v_cache=_ptr(v_cache),
        capacity=int(capacity), rope_n_rot=int(rope_n_rot), rope_freq_base=float(rope_freq_base),
        rope_pos_offset=int(rope_pos_offset))
    check(lib().sqmix_kv_append_q4_0(ctypes.byref(a), _stream(stream)), "set_rows_q4_0")


def kv_convert_rows(tiled: torch.Tensor, capacity: int, which: str, row0: int, n_rows: int,
                    rows_buf: torch.Tensor | None = None, to_rows: bool = True,
                    stream=None) -> torch.Tensor:
    """Tiled cache <-> ggml q4_0 rows ([n_rows][288] uint8).  which: 'k' or 'v'."""
    _require_cuda(tiled)
    if rows_buf is None:
        rows_buf = torch.empty((n_rows, 288), dtype=torch.uint8, device=tiled.device)
    w = {"k": 0, "v": 1}[which]
    check(lib().sqmix_kv_convert_rows(_ptr(tiled), _ptr(rows_buf), int(capacity), int(row0), int(n_rows),
                                      w, 1 if to_rows else 0, _stream(stream)), "kv_convert_rows")
    return rows_buf


def fa_workspace_bytes(n_q: int, n_splits: int = 0) -> int:
    return int(lib().sqmix_fa_workspace_bytes(int(n_splits), int(n_q)))


def new_fa_workspace(n_q: int = 2, n_splits: int = 0, device="cuda") -> torch.Tensor:
    """Scratch for flash_attn_ext; zeroed once (its header holds the error word)."""
    return torch.zeros(fa_workspace_bytes(n_q, n_splits), dtype=torch.uint8, device=device)


def _fa_args(q, k_cache, v_cache, capacity, n_kv, q_pos0, gate, scale, rope_n_rot, rope_freq_base,
             rope_pos_offset, out, lse, workspace, n_splits, config, k_new, v_new, flags, q_norm=None,
             k_norm=None, norm_eps=1e-6):
    """Validate tensors and build the sqmix_fa_args struct shared by decode and prefill."""
    _require_cuda(q, k_cache, v_cache, n_kv, q_pos0, gate)
    if q.dim() == 2:
        q = q.view(q.shape[0], N_HEAD, HEAD_DIM)
    n_q = q.shape[0]
    if q.stride(-1) != 1:
        raise ValueError("q rows must be contiguous along head_dim")
    if out is None:
        out = torch.empty((n_q, N_HEAD, HEAD_DIM), dtype=torch.float32, device=q.device)
    if gate is not None:
        if gate.dim() == 2:
            gate = gate.view(gate.shape[0], N_HEAD, HEAD_DIM)
        if gate.stride(-1) != 1:
            raise ValueError("gate rows must be contiguous along head_dim")
    n_new = 0
    if k_new is not None:
        _require_cuda(k_new, v_new)
        if k_new.dim() == 2:
            k_new = k_new.view(k_new.shape[0], N_HEAD_KV, HEAD_DIM)
        if v_new.dim() == 2:
            v_new = v_new.view(v_new.shape[0], N_HEAD_KV, HEAD_DIM)
        if (k_new.stride(-1) != 1 or k_new.stride(-2) != HEAD_DIM or v_new.stride(-1) != 1
                or v_new.stride(-2) != HEAD_DIM or k_new.dtype != v_new.dtype):
            raise ValueError("k_new/v_new must be [n_new][2][256] with contiguous heads and one dtype")
        n_new = k_new.shape[0]
    a = FaArgs(
        k_new=_ptr(k_new), v_new=_ptr(v_new), kv_new_dtype=_dt(k_new) if k_new is not None else 0,
        k_new_stride_tok=k_new.stride(0) if k_new is not None else 0,
        v_new_stride_tok=v_new.stride(0) if v_new is not None else 0, n_new=n_new,
        q=_ptr(q), q_dtype=_dt(q), q_stride_tok=q.stride(0), q_stride_head=q.stride(1),
        gate=_ptr(gate), gate_dtype=_dt(gate) if gate is not None else 0,
        gate_stride_tok=gate.stride(0) if gate is not None else 0,
        gate_stride_head=gate.stride(1) if gate is not None else 0,
        k_cache=_ptr(k_cache), v_cache=_ptr(v_cache), capacity=int(capacity), n_kv=_ptr(n_kv),
        q_pos0=_ptr(q_pos0), n_q=n_q, scale=float(scale), rope_n_rot=int(rope_n_rot),
        rope_freq_base=float(rope_freq_base), rope_pos_offset=int(rope_pos_offset), out=_ptr(out),
        lse=_ptr(lse), workspace=_ptr(workspace), workspace_bytes=workspace.numel(), n_splits=int(n_splits),
        config=int(config), flags=int(flags), q_norm=_ptr(q_norm), k_norm=_ptr(k_norm), norm_eps=float(norm_eps))
    return a, out


def flash_attn_ext(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, capacity: int,
                   n_kv: torch.Tensor, q_pos0: torch.Tensor, gate: torch.Tensor | None = None,
                   scale: float = 1.0 / 16.0, rope_n_rot: int = 0, rope_freq_base: float = 1e7,
                   rope_pos_offset: int = 0, out: torch.Tensor | None = None,
                   lse: torch.Tensor | None = None,
                   workspace: torch.Tensor | None = None, n_splits: int = 0, config: int = 0,
                   k_new: torch.Tensor | None = None, v_new: torch.Tensor | None = None,
                   overlap_prev: bool = False, q_norm: torch.Tensor | None = None,
                   k_norm: torch.Tensor | None = None, norm_eps: float = 1e-6, stream=None) -> torch.Tensor:
    """Split-KV attention of q [n_q][16][256] (n_q in {1, 2}) over the tiled q4_0 caches.

    n_kv and q_pos0 are device int64 scalars (CUDA-graph friendly).  Query t sees keys
    j <= q_pos0 + t and j < n_kv.  Returns out [n_q][16][256] f32 (gated if `gate`).
    With k_new/v_new ([n_new][2][256], n_new <= n_q) the step's rows q_pos0 + t are
    first quantised into the caches in the same launch (K rotated like Q).
    overlap_prev sets SQMIX_FA_OVERLAP_PREV: n_kv, q_pos0 and the cache rows below
    q_pos0 must then not be written by the kernel launched just before this call.
    q_norm / k_norm ([256] f32): per-head RMS norm of Q and of the appended K rows
    before RoPE (attn.rs:66-84), fused into the kernel.
    """
    for w in (q_norm, k_norm):
        if w is not None and (w.dtype != torch.float32 or w.numel() != HEAD_DIM or not w.is_contiguous()):
            raise ValueError("q_norm / k_norm must be contiguous float32 [256]")
    if workspace is None:
        workspace = new_fa_workspace(q.shape[0], n_splits, q.device)
    a, out = _fa_args(q, k_cache, v_cache, capacity, n_kv, q_pos0, gate, scale, rope_n_rot, rope_freq_base,
                      rope_pos_offset, out, lse, workspace, n_splits, config, k_new, v_new,
                      SQMIX_FA_OVERLAP_PREV if overlap_prev else 0, q_norm, k_norm, norm_eps)
    check(lib().sqmix_fa_decode(ctypes.byref(a), _stream(stream)), "flash_attn_ext")
    return out


def fa_batch_workspace_bytes(n_seqs: int, splits_per_seq: int = 0) -> int:
    return int(lib().sqmix_fa_batch_workspace_bytes(int(n_seqs), int(splits_per_seq)))


def flash_attn_decode_batch(q: torch.Tensor, k_caches: torch.Tensor, v_caches: torch.Tensor,
                            capacities: torch.Tensor, n_kv: torch.Tensor, q_pos0: torch.Tensor,
                            gate: torch.Tensor | None = None, scale: float = 1.0 / 16.0, rope_n_rot: int = 0,
                            rope_freq_base: float = 1e7, out: torch.Tensor | None = None,
                            lse: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
                            splits_per_seq: int = 0, k_new: torch.Tensor | None = None,
                            v_new: torch.Tensor | None = None, overlap_prev: bool = False,
                            stream=None) -> torch.Tensor:
    """One decode token for each of n_seqs sequences: q [n_seqs][16][256]; k_caches /
    v_caches: device int64 tensors [n_seqs] holding the data pointers of each sequence's
    tiled caches (capacities [n_seqs] rows); n_kv, q_pos0 device int64 [n_seqs].
    k_new / v_new [n_seqs][2][256] are appended at row q_pos0[s] in the same launch."""
    _require_cuda(q, k_caches, v_caches, capacities, n_kv, q_pos0, gate)
    n_seqs = q.shape[0]
    if q.dim() == 2:
        q = q.view(n_seqs, N_HEAD, HEAD_DIM)
    if q.stride(-1) != 1:
        raise ValueError("q rows must be contiguous along head_dim")
    for t in (k_caches, v_caches, capacities, n_kv, q_pos0):
        if t.dtype != torch.int64 or t.numel() != n_seqs or not t.is_contiguous():
            raise ValueError("pointer / scalar arrays must be contiguous int64 [n_seqs]")
    if out is None:
        out = torch.empty((n_seqs, N_HEAD, HEAD_DIM), dtype=torch.float32, device=q.device)
    if workspace is None:
        workspace = torch.zeros(fa_batch_workspace_bytes(n_seqs, splits_per_seq), dtype=torch.uint8,
                                device=q.device)
    n_new = 0
    if k_new is not None:
        _require_cuda(k_new, v_new)
        k_new = k_new.reshape(n_seqs, N_HEAD_KV * HEAD_DIM)
        v_new = v_new.reshape(n_seqs, N_HEAD_KV * HEAD_DIM)
        if k_new.stride(0) != v_new.stride(0) or k_new.dtype != v_new.dtype:
            raise ValueError("k_new and v_new must share dtype and layout")
        n_new = 1
    a = FaBatchArgs(
        n_seqs=n_seqs, q=_ptr(q), q_dtype=_dt(q), q_stride_seq=q.stride(0), q_stride_head=q.stride(1),
        gate=_ptr(gate), gate_dtype=_dt(gate) if gate is not None else 0,
        gate_stride_seq=gate.stride(0) if gate is not None else 0,
        gate_stride_head=gate.stride(1) if gate is not None else 0,
        k_caches=_ptr(k_caches), v_caches=_ptr(v_caches), capacities=_ptr(capacities), n_kv=_ptr(n_kv),
        q_pos0=_ptr(q_pos0), scale=float(scale), rope_n_rot=int(rope_n_rot), rope_freq_base=float(rope_freq_base),
        out=_ptr(out), lse=_ptr(lse), workspace=_ptr(workspace), workspace_bytes=workspace.numel(),
        splits_per_seq=int(splits_per_seq), k_new=_ptr(k_new), v_new=_ptr(v_new),
        kv_new_dtype=_dt(k_new) if k_new is not None else 0,
        new_stride_seq=k_new.stride(0) if k_new is not None else 0, n_new=n_new,
        flags=SQMIX_FA_OVERLAP_PREV if overlap_prev else 0)
    check(lib().sqmix_fa_decode_batch(ctypes.byref(a), _stream(stream)), "flash_attn_decode_batch")
    return out


def fa_prefill_workspace_bytes(n_q: int, n_ctas: int = 0) -> int:
    return int(lib().sqmix_fa_prefill_workspace_bytes(int(n_q), int(n_ctas)))


def new_fa_prefill_workspace(n_q: int, n_ctas: int = 0, device="cuda") -> torch.Tensor:
    """Scratch for flash_attn_prefill (item table and split partials); needs no init."""
    return torch.zeros(fa_prefill_workspace_bytes(n_q, n_ctas), dtype=torch.uint8, device=device)


def flash_attn_prefill(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, capacity: int,
                       n_kv: torch.Tensor, q_pos0: torch.Tensor, gate: torch.Tensor | None = None,
                       scale: float = 1.0 / 16.0, rope_n_rot: int = 0, rope_freq_base: float = 1e7,
                       rope_pos_offset: int = 0, out: torch.Tensor | None = None,
                       lse: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
                       n_ctas: int = 0, stream=None) -> torch.Tensor:
    """Causal attention of T query tokens q [T][16][256] over the tiled q4_0 caches on the
    tensor cores (the step's rows must already be appended).  Same semantics as
    flash_attn_ext: query t sees keys j <= q_pos0 + t and j < n_kv."""
    if workspace is None:
        workspace = new_fa_prefill_workspace(q.shape[0], n_ctas, q.device)
    a, out = _fa_args(q, k_cache, v_cache, capacity, n_kv, q_pos0, gate, scale, rope_n_rot, rope_freq_base,
                      rope_pos_offset, out, lse, workspace, n_ctas, 0, None, None, 0)
    check(lib().sqmix_fa_prefill(ctypes.byref(a), _stream(stream)), "flash_attn_prefill")
    return out


def fa_status(workspace: torch.Tensor, stream=None) -> None:
    """Raise SqmixError if a bounded device-side wait in a flash_attn_ext call gave up."""
    check(lib().sqmix_fa_status(_ptr(workspace), _stream(stream)), "flash_attn_ext device status")


def attn_merge_lse(o_parts: torch.Tensor, lse_parts: torch.Tensor, gate: torch.Tensor | None = None,
                   out: torch.Tensor | None = None, lse_out: torch.Tensor | None = None,
                   stream=None) -> torch.Tensor:
    """o_parts [P][rows][256] f32, lse_parts [P][rows] f32 -> out [rows][256]."""
    _require_cuda(o_parts, lse_parts, gate)
    P = o_parts.shape[0]
    rows = o_parts[0].numel() // HEAD_DIM
    if out is None:
        out = torch.empty((rows, HEAD_DIM), dtype=torch.float32, device=o_parts.device)
    if gate is not None and (gate.dtype != torch.float32 or not gate.is_contiguous()):
        gate = gate.float().contiguous()
    check(lib().sqmix_attn_merge_lse(P, rows, _ptr(o_parts.contiguous()), _ptr(lse_parts.contiguous()),
                                     _ptr(gate), _ptr(out), _ptr(lse_out), _stream(stream)),
          "attn_merge_lse")
    return out


GDN_CHUNK_MIN_T = 64  # from this many tokens on, gated_delta_net uses the chunked kernels


def gdn_prefill_workspace_bytes(n_seqs: int, n_tokens: int, h_v: int) -> int:
    return int(lib().sqmix_gdn_prefill_workspace_bytes(int(n_seqs), int(n_tokens), int(h_v)))


def gated_delta_net(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor,
                    beta: torch.Tensor, state: torch.Tensor, n_planes: int = 1,
                    sel: torch.Tensor | None = None, n_snap: int = 1, l2_eps: float = 0.0,
                    out: torch.Tensor | None = None, chunked: bool | None = None,
                    workspace: torch.Tensor | None = None, state_ready: bool = False,
                    h_v_offset: int = 0, dt_bias: torch.Tensor | None = None,
                    ssm_a: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """Gated delta rule over T tokens for n_seqs sequences.

    q, k [n_seqs][T][H_k][128]; v [n_seqs][T][H_v][128] (f32/bf16/f16); g, beta
    [n_seqs][T][H_v] f32; state [n_seqs][n_planes][H_v][128][128] f32 (updated in place:
    plane s <- state after T - s tokens for s < n_snap; the input plane is sel[seq]).
    3-D q/k/v/g/beta (no sequence dim) are accepted for n_seqs = 1.
    chunked: None picks the chunked prefill kernels (sqmix_gdn_prefill) for
    T >= GDN_CHUNK_MIN_T and the recurrent kernel (sqmix_gdn_decode) below.
    state_ready: the kernel launched just before on the stream writes neither the state
    nor sel (SQMIX_GDN_STATE_READY: the recurrent kernel reads the state early).
    h_v_offset: value-head sharding -- the call's value head i is head h_v_offset + i of
    the layer (q/k head (h_v_offset + i) % H_k; q and k hold all H_k heads).
    ssm_a (and dt_bias), f32 [layer value heads]: g and beta are the raw projections
    alpha and b; the kernels compute beta = sigmoid(b), g = softplus(alpha + dt_bias) *
    ssm_a (gdn.rs:268-287).
    """
    _require_cuda(q, k, v, g, beta, state, sel)
    if q.dim() == 3:
        q, k, v, g, beta = q[None], k[None], v[None], g[None], beta[None]
    n_seqs, T, H_k, d = q.shape
    H_v = v.shape[2]
    if d != GDN_D or v.shape[3] != GDN_D:
        raise ValueError("GDN head dim must be 128")
    if q.stride() != k.stride() or q.stride(-1) != 1 or q.stride(-2) != GDN_D or v.stride(-1) != 1:
        raise ValueError("q and k must share a [seq][tok][head][128] layout with contiguous heads")
    if g.dtype != torch.float32 or beta.dtype != torch.float32:
        raise TypeError("g and beta must be float32")
    g = g.contiguous()
    beta = beta.contiguous()
    if out is None:
        out = torch.empty((n_seqs, T, H_v, GDN_D), dtype=torch.float32, device=q.device)
    a = GdnArgs(
        q=_ptr(q), k=_ptr(k), v=_ptr(v), dtype=_dt(q), qk_stride_tok=q.stride(1), v_stride_tok=v.stride(1),
        qk_stride_seq=q.stride(0), v_stride_seq=v.stride(0), g=_ptr(g), beta=_ptr(beta),
        state=_ptr(state), n_planes=int(n_planes), sel=_ptr(sel), n_seqs=n_seqs, n_tokens=T, h_k=H_k,
        h_v=H_v, n_snap=int(n_snap), l2_eps=float(l2_eps), out=_ptr(out), flags=1 if state_ready else 0,
        h_v_offset=int(h_v_offset), dt_bias=_ptr(dt_bias), ssm_a=_ptr(ssm_a))
    for w in (dt_bias, ssm_a):
        if w is not None and (w.dtype != torch.float32 or not w.is_contiguous() or not w.is_cuda
                              or w.numel() < h_v_offset + H_v):
            raise ValueError("dt_bias / ssm_a must be contiguous float32 CUDA tensors over the layer's value heads")
    if dt_bias is not None and ssm_a is None:
        raise ValueError("dt_bias needs ssm_a (the gate epilogue)")
    if chunked is None:
        chunked = T >= GDN_CHUNK_MIN_T
    if chunked:
        need = gdn_prefill_workspace_bytes(n_seqs, T, H_v)
        if workspace is None or workspace.numel() < need:
            workspace = torch.zeros(need, dtype=torch.uint8, device=q.device)
        check(lib().sqmix_gdn_prefill(ctypes.byref(a), _ptr(workspace), workspace.numel(), _stream(stream)),
              "gated_delta_net (chunked)")
    else:
        check(lib().sqmix_gdn_decode(ctypes.byref(a), _stream(stream)), "gated_delta_net")
    return out


def gdn_state_copy(dst: torch.Tensor, src: torch.Tensor, plane_elems: int, n_planes: int,
                   stream=None) -> None:
    _require_cuda(dst, src)
    check(lib().sqmix_gdn_state_copy(_ptr(dst), _ptr(src), int(plane_elems), int(n_planes),
                                     _stream(stream)), "gdn_state_copy")


def gdn_conv(x: torch.Tensor, weight: torch.Tensor, conv_state: torch.Tensor, n_planes: int = 1,
             sel: torch.Tensor | None = None, n_snap: int = 1, n_qk_channels: int = 0, l2_eps: float = 0.0,
             head_dim: int = GDN_D, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """GDN short convolution (ggml_ssm_conv + silu, gdn.rs:290-360) with the history
    planes, plus the per-head L2 norm of the first n_qk_channels channels when l2_eps > 0.

    x [n_seqs][T][C] qkv_mixed (f32/bf16/f16, rows contiguous); weight [C][K] f32;
    conv_state [n_seqs][n_planes][C][K-1] f32, updated in place (plane s <- the history
    s tokens back for s < n_snap; the input plane is sel[seq]).  2-D x is one sequence.
    Returns out [n_seqs][T][C] f32."""
    _require_cuda(x, weight, conv_state, sel)
    if x.dim() == 2:
        x = x[None]
    n_seqs, T, C = x.shape
    if x.stride(-1) != 1:
        raise ValueError("x rows must be contiguous")
    if weight.dtype != torch.float32 or weight.dim() != 2 or weight.shape[0] != C or not weight.is_contiguous():
        raise ValueError("weight must be contiguous float32 [C][K]")
    K = weight.shape[1]
    if (conv_state.dtype != torch.float32 or not conv_state.is_contiguous()
            or conv_state.numel() != n_seqs * n_planes * C * (K - 1)):
        raise ValueError("conv_state must be contiguous float32 [n_seqs][n_planes][C][K-1]")
    if out is None:
        out = torch.empty((n_seqs, T, C), dtype=torch.float32, device=x.device)
    a = GdnConvArgs(x=_ptr(x), x_dtype=_dt(x), x_stride_tok=x.stride(1), x_stride_seq=x.stride(0),
                    weight=_ptr(weight), conv_state=_ptr(conv_state), n_planes=int(n_planes), sel=_ptr(sel),
                    n_snap=int(n_snap), n_seqs=n_seqs, n_tokens=T, channels=C, kernel=K, head_dim=int(head_dim),
                    n_qk_channels=int(n_qk_channels), l2_eps=float(l2_eps), out=_ptr(out))
    check(lib().sqmix_gdn_conv(ctypes.byref(a), _stream(stream)), "gdn_conv")
    return out


def head_norm(x: torch.Tensor, eps: float = 1e-6, weight: torch.Tensor | None = None,
              z: torch.Tensor | None = None, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """Per-head RMS norm over the last axis of x [T][H][d] (any strides with a unit
    last stride): x / sqrt(mean(x^2) + eps), then * weight ([d] or [H][d], f32) and
    * silu(z) (z shaped like x).  Q/K norm of the attention layers (attn.rs:66-84) and
    norm_gated of the GDN output (gdn.rs:150-181).  Returns out f32 [T][H][d]."""
    _require_cuda(x, weight, z)
    if x.dim() == 2:
        x = x[:, None]
    T, H, d = x.shape
    if x.stride(-1) != 1 or (z is not None and (z.shape != x.shape or z.stride(-1) != 1)):
        raise ValueError("x and z must be [T][H][d] with a unit last stride")
    w_sh = 0
    if weight is not None:
        if weight.dtype != torch.float32 or not weight.is_contiguous():
            raise ValueError("weight must be contiguous float32")
        if weight.numel() == H * d:
            w_sh = d
        elif weight.numel() != d:
            raise ValueError("weight must be [d] or [H][d]")
    if out is None:
        out = torch.empty((T, H, d), dtype=torch.float32, device=x.device)
    a = HeadNormArgs(x=_ptr(x), x_dtype=_dt(x), x_stride_tok=x.stride(0), x_stride_head=x.stride(1),
                     weight=_ptr(weight), weight_stride_head=w_sh, z=_ptr(z), z_dtype=_dt(z) if z is not None else 0,
                     z_stride_tok=z.stride(0) if z is not None else 0, z_stride_head=z.stride(1) if z is not None else 0,
                     n_tokens=T, n_heads=H, head_dim=d, eps=float(eps), out=_ptr(out),
                     out_stride_tok=out.stride(0), out_stride_head=out.stride(1))
    check(lib().sqmix_head_norm(ctypes.byref(a), _stream(stream)), "head_norm")
    return out


def gdn_layer_decode(x: torch.Tensor, conv_weight: torch.Tensor, conv_state: torch.Tensor, alpha: torch.Tensor,
                     beta: torch.Tensor, ssm_a: torch.Tensor, state: torch.Tensor, h_k: int = 16, h_v: int = 32,
                     dt_bias: torch.Tensor | None = None, n_planes: int = 1, sel: torch.Tensor | None = None,
                     n_snap: int = 1, l2_eps: float = 1e-6, z: torch.Tensor | None = None,
                     norm_weight: torch.Tensor | None = None, norm_eps: float = 1e-6, out: torch.Tensor | None = None,
                     state_ready: bool = False, stream=None) -> torch.Tensor:
    """A GDN mixer decode step in one launch (sqmix_gdn_layer_decode): x [n_seqs][T][C]
    qkv_mixed (T = 1 or 2, C = (2 h_k + h_v) * 128); conv_weight [C][4]; conv_state
    [n_seqs][n_planes][C][3] and state [n_seqs][n_planes][h_v][128][128] (updated in place,
    input plane sel[seq]); alpha, beta [n_seqs][T][h_v] raw projections; ssm_a, dt_bias
    [h_v]; z [n_seqs][T][h_v][128]; norm_weight [128] (or [h_v][128]).  Returns
    norm_gated(o) [n_seqs][T][h_v][128] f32."""
    _require_cuda(x, conv_weight, conv_state, alpha, beta, ssm_a, state, dt_bias, sel, z, norm_weight)
    if x.dim() == 2:
        x = x[None]
    n_seqs, T, C = x.shape
    if x.stride(-1) != 1:
        raise ValueError("x rows must be contiguous")
    for t in (alpha, beta, ssm_a, dt_bias, norm_weight, conv_weight, conv_state, state):
        if t is not None and (t.dtype != torch.float32 or not t.is_contiguous()):
            raise ValueError("float32 contiguous tensors expected for the weights, gates and states")
    if z is not None:
        z = z.reshape(n_seqs, T, h_v, GDN_D)
        if z.stride(-1) != 1 or z.stride(-2) != GDN_D:
            raise ValueError("z heads must be contiguous [.., h_v, 128]")
    if out is None:
        out = torch.empty((n_seqs, T, h_v, GDN_D), dtype=torch.float32, device=x.device)
    nw_sh = 0 if norm_weight is None or norm_weight.numel() == GDN_D else GDN_D
    a = GdnLayerArgs(
        x=_ptr(x), x_dtype=_dt(x), x_stride_tok=x.stride(1), x_stride_seq=x.stride(0),
        conv_weight=_ptr(conv_weight), conv_state=_ptr(conv_state), kernel=conv_weight.shape[-1],
        alpha=_ptr(alpha), beta=_ptr(beta), dt_bias=_ptr(dt_bias), ssm_a=_ptr(ssm_a), state=_ptr(state),
        n_planes=int(n_planes), sel=_ptr(sel), n_snap=int(n_snap), n_seqs=n_seqs, n_tokens=T, h_k=int(h_k),
        h_v=int(h_v), l2_eps=float(l2_eps), z=_ptr(z), z_dtype=_dt(z) if z is not None else 0,
        z_stride_tok=z.stride(1) if z is not None else 0, z_stride_seq=z.stride(0) if z is not None else 0,
        norm_weight=_ptr(norm_weight), norm_weight_stride_head=nw_sh, norm_eps=float(norm_eps), out=_ptr(out),
        flags=1 if state_ready else 0)
    check(lib().sqmix_gdn_layer_decode(ctypes.byref(a), _stream(stream)), "gdn_layer_decode")
    return out


def rope_theta_scale(freq_base: float, n_rot: int) -> float:
    return math.pow(freq_base, -2.0 / n_rot)


def mul_mat_row_bytes(w_type: int, n_in: int) -> int:
    """Bytes of one weight row of n_in values in ggml format w_type (0: unsupported)."""
    return int(lib().sqmix_mul_mat_row_bytes(int(w_type), int(n_in)))


def _mul_mat_entry(w: torch.Tensor, w_type: int, n_in: int, x2: torch.Tensor, out: torch.Tensor | None,
                   status: torch.Tensor | None):
    rb = mul_mat_row_bytes(w_type, n_in)
    if rb == 0:
        raise ValueError(f"unsupported weight type {w_type} for n_in={n_in}")
    if not w.is_contiguous() or w.numel() * w.element_size() % rb != 0:
        raise ValueError("w must be contiguous rows of the format")
    n_out = w.numel() * w.element_size() // rb
    T = x2.shape[0]
    if out is None:
        out = torch.empty((T, n_out), dtype=torch.float32, device=x2.device)
    a = MulMatArgs(w=w.data_ptr(), w_type=int(w_type), w_row_bytes=rb, n_in=n_in, n_out=n_out, x=x2.data_ptr(),
                   x_dtype=_dt(x2), x_stride=x2.stride(0), n_tokens=T, y=out.data_ptr(), y_stride=out.stride(0),
                   status=status.data_ptr() if status is not None else None)
    return a, out


def _tokens(x: torch.Tensor, n_in: int) -> torch.Tensor:
    x2 = x.reshape(-1, n_in)
    return x2 if x2.stride(1) == 1 else x2.contiguous()


def mul_mat(w: torch.Tensor, w_type: int, n_in: int, x: torch.Tensor, out: torch.Tensor | None = None,
            status: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """ggml_mul_mat(w, x): w [n_out][row bytes] (uint8, a GGUF block format: SQMIX_Q8_0 /
    SQMIX_Q4_K / SQMIX_Q6_K) or [n_out][n_in] f32 / f16 / bf16 elements; x [T][n_in]
    (f32 / f16 / bf16, rows contiguous).  Returns y [T][n_out] f32."""
    a, out = _mul_mat_entry(w, w_type, n_in, _tokens(x, n_in), out, status)
    check(lib().sqmix_mul_mat(ctypes.byref(a), _stream(stream)), "mul_mat")
    return out


def mul_mat_group(weights, n_in: int, x: torch.Tensor, outs=None, status: torch.Tensor | None = None,
                  stream=None) -> list:
    """Several ggml_mul_mat of the same x in one pass (sqmix_mul_mat_group): weights is a
    list of (w, w_type) as for mul_mat, outs an optional list of y tensors (None entries
    are allocated).  Returns the list of y [T][n_out] f32."""
    if not 1 <= len(weights) <= SQMIX_MUL_MAT_MAX_GROUP:
        raise ValueError(f"a group has 1..{SQMIX_MUL_MAT_MAX_GROUP} projections, not {len(weights)}")
    x2 = _tokens(x, n_in)
    outs = list(outs) if outs is not None else [None] * len(weights)
    arr = (MulMatArgs * len(weights))()
    res = []
    for i, ((w, w_type), o) in enumerate(zip(weights, outs)):
        arr[i], o = _mul_mat_entry(w, w_type, n_in, x2, o, status if i == 0 else None)
        res.append(o)
    check(lib().sqmix_mul_mat_group(arr, len(weights), _stream(stream)), "mul_mat_group")
    return res
