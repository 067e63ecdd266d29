"""CPU parity oracle for the sqmix attention-mixer kernels.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU
legs of ``bench.py`` (``cpu_baseline`` and ``--impl reference``) may import this
package.  The product library (``libsqmix.so`` and the ``sqmix`` host package) never
imports, links or calls it.

The arithmetic lives in ``sqmix_oracle.c`` (a C restatement of the ggml nodes that
sqwen calls; see that file's header for the reference citations and for which
nodes are pinned by golden vectors).  This module is a thin numpy/ctypes wrapper.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libsqmix_oracle.so")
_lib = None

QK4_0 = 32
Q4_0_BLOCK_BYTES = 18


def build() -> str:
    """Compile the oracle with its Makefile (gcc; no GPU needed)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        f32p = ctypes.POINTER(ctypes.c_float)
        u8p = ctypes.POINTER(ctypes.c_uint8)
        i32p = ctypes.POINTER(ctypes.c_int32)
        i64 = ctypes.c_int64
        L.oracle_f32_to_f16.argtypes = [ctypes.c_float]
        L.oracle_f32_to_f16.restype = ctypes.c_uint16
        L.oracle_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.oracle_f16_to_f32.restype = ctypes.c_float
        L.oracle_q4_0_quantize_rows.argtypes = [f32p, i64, i64, u8p]
        L.oracle_q4_0_dequantize_rows.argtypes = [u8p, i64, i64, f32p]
        L.oracle_rope_imrope.argtypes = [f32p, i64, i64, i64, i32p, i32p, ctypes.c_float,
                                         ctypes.c_int32]
        L.oracle_rope_text.argtypes = [f32p, i64, i64, i64, i64, ctypes.c_float, ctypes.c_int32]
        L.oracle_attn.argtypes = [f32p, f32p, f32p, f32p, i64, i64, i64, i64, i64, i64,
                                  ctypes.c_float, f32p, f32p]
        L.oracle_l2norm_rows.argtypes = [f32p, i64, i64, ctypes.c_float]
        L.oracle_gdn.argtypes = [f32p, f32p, f32p, f32p, f32p, f32p, i64, i64, i64, i64, i64,
                                 f32p, f32p]
        L.oracle_ssm_conv.argtypes = [f32p, i64, i64, i64, f32p, f32p]
        L.oracle_gdn_conv.argtypes = [f32p, i64, i64, i64, f32p, f32p, i64, i64, i64, i64, i64, ctypes.c_float,
                                      f32p]
        L.oracle_rms_norm_rows.argtypes = [f32p, i64, i64, ctypes.c_float, f32p, i64, i64, f32p, f32p]
        L.cpu_fa_q4_0.argtypes = [f32p, u8p, u8p, f32p, i64, i64, i64, i64, i64, i64, ctypes.c_float, f32p, f32p]
        L.cpu_gdn_f32.argtypes = [f32p, f32p, f32p, f32p, f32p, f32p, i64, i64, i64, i64, f32p]
        L.oracle_set_threads.argtypes = [ctypes.c_int]
        L.oracle_set_threads.restype = ctypes.c_int
        L.oracle_row_bytes.argtypes = [ctypes.c_int, i64]
        L.oracle_row_bytes.restype = i64
        L.oracle_dequant_row.argtypes = [u8p, ctypes.c_int, i64, f32p]
        L.oracle_dequant_row.restype = ctypes.c_int
        L.oracle_mul_mat.argtypes = [u8p, ctypes.c_int, i64, i64, i64, f32p, i64, ctypes.c_int, f32p, i64]
        L.oracle_mul_mat.restype = ctypes.c_int
        L.cpu_mul_mat.argtypes = [u8p, ctypes.c_int, i64, i64, i64, f32p, ctypes.c_int, f32p]
        L.cpu_mul_mat.restype = ctypes.c_int
        _lib = L
    return _lib


def _f32(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a, a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _nullf32():
    return ctypes.POINTER(ctypes.c_float)()


def set_threads(n: int) -> int:
    """Set the OpenMP thread count; returns the count now in effect."""
    return lib().oracle_set_threads(int(n))


def f32_to_f16_bits(x: float) -> int:
    return int(lib().oracle_f32_to_f16(float(x)))


def f16_bits_to_f32(h: int) -> float:
    return float(lib().oracle_f16_to_f32(int(h)))


def q4_0_quantize(x: np.ndarray) -> np.ndarray:
    """Rows of f32 (last dim a multiple of 32) -> ggml q4_0 rows (uint8, 18 B/block)."""
    x = np.asarray(x, dtype=np.float32)
    n = x.shape[-1]
    assert n % QK4_0 == 0
    rows = int(np.prod(x.shape[:-1])) if x.ndim > 1 else 1
    xs, xp = _f32(x.reshape(rows, n))
    out = np.zeros((rows, n // QK4_0 * Q4_0_BLOCK_BYTES), dtype=np.uint8)
    lib().oracle_q4_0_quantize_rows(xp, rows, n, out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)))
    return out.reshape(*x.shape[:-1], n // QK4_0 * Q4_0_BLOCK_BYTES)


def q4_0_dequantize(q: np.ndarray, n_per_row: int) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.uint8)
    rows = q.size // (n_per_row // QK4_0 * Q4_0_BLOCK_BYTES)
    out = np.zeros((rows, n_per_row), dtype=np.float32)
    lib().oracle_q4_0_dequantize_rows(q.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)), rows,
                                      n_per_row, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    return out.reshape(*q.shape[:-1], n_per_row)


def rope_imrope(x: np.ndarray, pos: np.ndarray, sections, freq_base: float, n_rot: int) -> np.ndarray:
    """x [T][H][D]; pos i32 [4*T] (t/h/w/e streams). Returns a rotated copy."""
    xs, xp = _f32(np.array(x, dtype=np.float32, copy=True))
    T, H, D = xs.shape
    pos = np.ascontiguousarray(pos, dtype=np.int32)
    sec = np.ascontiguousarray(sections, dtype=np.int32)
    i32p = ctypes.POINTER(ctypes.c_int32)
    lib().oracle_rope_imrope(xp, T, H, D, pos.ctypes.data_as(i32p), sec.ctypes.data_as(i32p),
                             float(freq_base), int(n_rot))
    return xs


def rope_text(x: np.ndarray, pos0: int, freq_base: float, n_rot: int) -> np.ndarray:
    """x [T][H][D], text positions pos0 + t in all four streams. Returns a copy."""
    xs, xp = _f32(np.array(x, dtype=np.float32, copy=True))
    T, H, D = xs.shape
    lib().oracle_rope_text(xp, T, H, D, int(pos0), float(freq_base), int(n_rot))
    return xs


def attn(q, k, v, gate=None, q_pos0: int = 0, scale: float | None = None, want_lse=False):
    """q [T][Hq][D]; k, v [n_kv][Hkv][D] (dequantised); gate [T][Hq][D] or None."""
    qs, qp = _f32(q)
    ks, kp = _f32(k)
    vs, vp = _f32(v)
    T, Hq, D = qs.shape
    n_kv, Hkv, _ = ks.shape
    if scale is None:
        scale = 1.0 / np.sqrt(D)
    if gate is not None:
        gs, gp = _f32(gate)
    else:
        gp = _nullf32()
    out = np.zeros((T, Hq, D), dtype=np.float32)
    lse = np.zeros((T, Hq), dtype=np.float32)
    f32p = ctypes.POINTER(ctypes.c_float)
    lib().oracle_attn(qp, kp, vp, gp, T, Hq, Hkv, D, n_kv, int(q_pos0), float(scale),
                      out.ctypes.data_as(f32p), lse.ctypes.data_as(f32p))
    return (out, lse) if want_lse else out


def l2norm(x: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    xs, xp = _f32(np.array(x, dtype=np.float32, copy=True))
    n = xs.shape[-1]
    lib().oracle_l2norm_rows(xp, xs.size // n, n, float(eps))
    return xs


def gdn(q, k, v, g, beta, state, n_snap: int = 1):
    """Sequential gated delta rule.

    q, k [T][Hk][d]; v [T][Hv][d]; g, beta [T][Hv]; state [Hv][d(j)][d(i)].
    Returns (out [T][Hv][d], snaps [n_snap][Hv][d][d]).
    """
    qs, qp = _f32(q)
    ks, kp = _f32(k)
    vs, vp = _f32(v)
    gs, gp = _f32(g)
    bs, bp = _f32(beta)
    ss, sp = _f32(state)
    T, Hk, d = qs.shape
    Hv = vs.shape[1]
    out = np.zeros((T, Hv, d), dtype=np.float32)
    snaps = np.zeros((n_snap, Hv, d, d), dtype=np.float32)
    f32p = ctypes.POINTER(ctypes.c_float)
    lib().oracle_gdn(qp, kp, vp, gp, bp, sp, T, Hk, Hv, d, int(n_snap),
                     out.ctypes.data_as(f32p), snaps.ctypes.data_as(f32p))
    return out, snaps


def ssm_conv(sx: np.ndarray, w: np.ndarray) -> np.ndarray:
    """ggml_ssm_conv: sx [C][K-1+T], w [C][K] -> out [T][C]."""
    sxs, sxp = _f32(sx)
    ws, wp = _f32(w)
    C, ncs = sxs.shape
    K = ws.shape[1]
    T = ncs - (K - 1)
    out = np.zeros((T, C), dtype=np.float32)
    lib().oracle_ssm_conv(sxp, C, T, K, wp, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    return out


def gdn_conv(x, w, state, sel: int = 0, n_snap: int = 1, n_qk: int = 0, d: int = 128, eps: float = 1e-6):
    """GDN front end of one sequence: x [T][C], w [C][K], state [n_planes][C][K-1]
    (not modified).  Returns (out [T][C] = silu(conv) with the first n_qk channels
    L2-normalised per head of d, new state [n_planes][C][K-1] with slots
    0..n_snap-1 rewritten)."""
    xs, xp = _f32(x)
    ws, wp = _f32(w)
    st = np.array(state, dtype=np.float32, copy=True)
    sp = st.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    T, C = xs.shape
    K = ws.shape[1]
    out = np.zeros((T, C), dtype=np.float32)
    lib().oracle_gdn_conv(xp, T, C, K, wp, sp, st.shape[0], int(sel), int(n_snap), int(n_qk), int(d),
                          float(eps), out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    return out, st


def rms_norm(x, eps: float = 1e-6, w=None, z=None):
    """Per-row RMS norm over the last axis, then * w (broadcast over rows: [n], or
    [H][n] cycling with the second-to-last axis) and * silu(z) (same shape as x)."""
    xs, xp = _f32(x)
    n = xs.shape[-1]
    nrows = xs.size // n
    f32p = ctypes.POINTER(ctypes.c_float)
    wp, w_stride, w_period = _nullf32(), 0, 0
    if w is not None:
        ws, wp = _f32(w)
        if ws.ndim == 2:
            w_stride, w_period = n, ws.shape[0]
    zp = _nullf32()
    if z is not None:
        zs, zp = _f32(z)
    out = np.zeros(xs.shape, dtype=np.float32)
    lib().oracle_rms_norm_rows(xp, nrows, n, float(eps), wp, w_stride, w_period, zp, out.ctypes.data_as(f32p))
    return out


def merge_lse(o_parts, lse_parts, gate=None):
    """Merge normalised partial attentions over disjoint key sets (split-KV):
    out = sum_p O_p exp(lse_p - L) with L = log sum_p exp(lse_p), then * sigmoid(gate).
    o_parts [P][rows][D], lse_parts [P][rows]; parts with lse = -inf carry no weight.
    Restates the merge of the split-KV decode (the LSE combination of flash-decoding)."""
    o = np.asarray(o_parts, dtype=np.float64)
    lse = np.asarray(lse_parts, dtype=np.float64)
    L = np.max(lse, axis=0)
    finite = np.isfinite(L)
    Ls = np.where(finite, L, 0.0)
    w = np.where(np.isfinite(lse), np.exp(lse - Ls[None]), 0.0)
    tot = w.sum(axis=0)
    out = (o * w[..., None]).sum(axis=0) / np.where(tot > 0, tot, 1.0)[..., None]
    out = np.where(finite[..., None], out, 0.0)
    if gate is not None:
        out = out / (1.0 + np.exp(-np.asarray(gate, dtype=np.float64)))
    lse_out = np.where(finite, Ls + np.log(np.where(tot > 0, tot, 1.0)), -np.inf)
    return out.astype(np.float32), lse_out.astype(np.float32)


# --------------------------------------------------------------------------- #
# The timed CPU baseline (cpu_ggml.c): ggml-cpu's way of running the same nodes. #
# Not the checker: these run in f32 with Q as q8_0, as ggml-cpu does.           #
# --------------------------------------------------------------------------- #

def cpu_fa_q4_0(q, k_rows, v_rows, gate=None, q_pos0: int = 0, scale: float = 1.0 / 16, want_lse=False):
    """q [T][Hq][D] f32 (rotated); k_rows, v_rows [n_kv][Hkv*D/32*18] uint8 (ggml q4_0 rows);
    gate [T][Hq][D] or None.  ggml-cpu flash attention (q8_0 Q, f32 online softmax)."""
    qs, qp = _f32(q)
    T, Hq, D = qs.shape
    kr = np.ascontiguousarray(k_rows, dtype=np.uint8)
    vr = np.ascontiguousarray(v_rows, dtype=np.uint8)
    n_kv = kr.shape[0]
    Hkv = kr.shape[1] * QK4_0 // Q4_0_BLOCK_BYTES // D
    gp = _nullf32()
    if gate is not None:
        gs, gp = _f32(gate)
    out = np.zeros((T, Hq, D), dtype=np.float32)
    lse = np.zeros((T, Hq), dtype=np.float32)
    f32p = ctypes.POINTER(ctypes.c_float)
    u8p = ctypes.POINTER(ctypes.c_uint8)
    lib().cpu_fa_q4_0(qp, kr.ctypes.data_as(u8p), vr.ctypes.data_as(u8p), gp, T, Hq, Hkv, D, n_kv, int(q_pos0),
                      float(scale), out.ctypes.data_as(f32p), lse.ctypes.data_as(f32p))
    return (out, lse) if want_lse else out


def cpu_gdn_f32(q, k, v, g, beta, state):
    """Token-by-token gated delta rule in f32; state [Hv][d][d] is updated in place
    (must be a C-contiguous float32 array).  Returns out [T][Hv][d]."""
    if not (isinstance(state, np.ndarray) and state.dtype == np.float32 and state.flags.c_contiguous):
        raise TypeError("state must be a C-contiguous float32 array (updated in place)")
    qs, qp = _f32(q)
    ks, kp = _f32(k)
    vs, vp = _f32(v)
    gs, gp = _f32(g)
    bs, bp = _f32(beta)
    T, Hk, d = qs.shape
    Hv = vs.shape[1]
    out = np.zeros((T, Hv, d), dtype=np.float32)
    f32p = ctypes.POINTER(ctypes.c_float)
    lib().cpu_gdn_f32(qp, kp, vp, gp, bp, state.ctypes.data_as(f32p), T, Hk, Hv, d, out.ctypes.data_as(f32p))
    return out


def gdn_gates(alpha, b, dt_bias, ssm_a):
    """The gate epilogue of the GDN projections, src/model/gdn.rs:268-287 (ggml_sigmoid;
    ggml_add, ggml_softplus, ggml_mul): beta = sigmoid(b), g = softplus(alpha + dt_bias)
    * ssm_a, with ssm_a = -exp(A_log) as the model stores it.  alpha, b [..., H_v];
    dt_bias, ssm_a [H_v].  softplus(x) = log1p(e^x), x itself above 20.  In double."""
    a = np.asarray(alpha, dtype=np.float64) + np.asarray(dt_bias, dtype=np.float64)
    sp = np.where(a > 20.0, a, np.log1p(np.exp(np.minimum(a, 20.0))))
    g = sp * np.asarray(ssm_a, dtype=np.float64)
    beta = 1.0 / (1.0 + np.exp(-np.asarray(b, dtype=np.float64)))
    return g.astype(np.float32), beta.astype(np.float32)


# ggml type ids of the projection weights (src/backend/ffi.rs:44-101)
GGML_F32, GGML_F16, GGML_Q8_0, GGML_Q4_K, GGML_Q6_K, GGML_BF16 = 0, 1, 8, 12, 14, 30


def row_bytes(wtype: int, n: int) -> int:
    """Bytes of one weight row of n values in ggml format wtype (0: unsupported)."""
    return int(lib().oracle_row_bytes(int(wtype), int(n)))


def dequant_rows(w: np.ndarray, wtype: int, n: int) -> np.ndarray:
    """Rows of ggml-format bytes [rows][row_bytes] -> f32 [rows][n]."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    rb = row_bytes(wtype, n)
    assert rb > 0 and w.shape[-1] == rb, (wtype, n, w.shape)
    rows = w.size // rb
    out = np.zeros((rows, n), dtype=np.float32)
    u8p, f32p = ctypes.POINTER(ctypes.c_uint8), ctypes.POINTER(ctypes.c_float)
    for r in range(rows):
        rc = lib().oracle_dequant_row(w[r].ctypes.data_as(u8p), int(wtype), n, out[r].ctypes.data_as(f32p))
        assert rc == 0
    return out


def mul_mat(w: np.ndarray, wtype: int, n_in: int, x: np.ndarray) -> np.ndarray:
    """ggml_mul_mat(w, x): w [n_out][row_bytes] in format wtype, x [T][n_in] -> y [T][n_out]."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    rb = row_bytes(wtype, n_in)
    assert rb > 0 and w.shape[-1] == rb
    n_out = w.size // rb
    xs, xp = _f32(np.asarray(x, dtype=np.float32).reshape(-1, n_in))
    T = xs.shape[0]
    y = np.zeros((T, n_out), dtype=np.float32)
    rc = lib().oracle_mul_mat(w.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)), int(wtype), rb, n_in, n_out, xp,
                              n_in, T, y.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), n_out)
    assert rc == 0
    return y


def cpu_mul_mat(w: np.ndarray, wtype: int, n_in: int, x: np.ndarray) -> np.ndarray:
    """The timed CPU baseline of ggml_mul_mat: ggml-cpu's quantised dot products (x
    quantised to q8_K / q8_0 per token), rows across threads.  Not the checker."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    rb = row_bytes(wtype, n_in)
    assert rb > 0 and w.shape[-1] == rb
    n_out = w.size // rb
    xs, xp = _f32(np.asarray(x, dtype=np.float32).reshape(-1, n_in))
    T = xs.shape[0]
    y = np.zeros((T, n_out), dtype=np.float32)
    rc = lib().cpu_mul_mat(w.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)), int(wtype), rb, n_in, n_out, xp, T,
                           y.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    assert rc == 0
    return y
