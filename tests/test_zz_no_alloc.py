"""sqmix_fa_decode_noalloc: the decode attention entry point that takes its split
scratch from a static device array instead of a caller workspace.

Collected last on purpose (file name), so the GPU case runs both alone and after
every other test in the process.  The GPU case compares two calls in a row with the
workspace entry point (sqmix_fa_decode) on the same inputs, within the attention
tolerance of the parity tests.
"""
import ctypes

import numpy as np
import pytest
import torch

ATTN_TOL = 2e-3  # max|a - b| <= ATTN_TOL * max|b|, as for attention against the oracle


def _args(sq, q, gate, kc, vc, cap, d_nkv, d_pos, out, n_splits):
    from sqmix._lib import FaArgs

    return FaArgs(
        q=q.data_ptr(), q_dtype=sq.SQMIX_F32, q_stride_tok=q.stride(0), q_stride_head=q.stride(1),
        gate=gate.data_ptr(), gate_dtype=sq.SQMIX_F32, gate_stride_tok=gate.stride(0),
        gate_stride_head=gate.stride(1), k_cache=kc.data_ptr(), v_cache=vc.data_ptr(), capacity=cap,
        n_kv=d_nkv.data_ptr(), q_pos0=d_pos.data_ptr(), n_q=q.shape[0], scale=1.0 / 16.0, rope_n_rot=64,
        rope_freq_base=1e7, rope_pos_offset=0, out=out.data_ptr(), lse=None, workspace=None,
        workspace_bytes=0, n_splits=n_splits, config=0)


def test_noalloc_rejects_split_count_above_scratch():
    import sqmix as sq
    from sqmix._lib import FaArgs

    a = FaArgs(n_q=1, n_splits=161)
    rc = sq.lib().sqmix_fa_decode_noalloc(ctypes.byref(a), None)
    assert rc == sq.SQMIX_EINVAL
    assert b"exceeds the static scratch" in sq.lib().sqmix_last_error()


@pytest.mark.gpu
@pytest.mark.parametrize("n_q,n_splits", [(1, 0), (2, 0), (1, 37)])
def test_noalloc_matches_workspace_entry_point(n_q, n_splits):
    import sqmix as sq

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(4242 + n_q)
    n_kv = 5000
    cap = (n_kv + 255) // 256 * 256
    kc, vc = sq.new_kv_cache(cap), sq.new_kv_cache(cap)
    sq.set_rows_q4_0(torch.randn((n_kv, 2, 256), generator=g, device=dev),
                     torch.randn((n_kv, 2, 256), generator=g, device=dev),
                     torch.arange(n_kv, device=dev), kc, vc, cap, rope_n_rot=64, rope_freq_base=1e7)
    q = torch.randn((n_q, 16, 256), generator=g, device=dev)
    gate = torch.randn((n_q, 16, 256), generator=g, device=dev)
    d_nkv = torch.tensor([n_kv], dtype=torch.int64, device=dev)
    d_pos = torch.tensor([n_kv - n_q], dtype=torch.int64, device=dev)

    want = sq.flash_attn_ext(q, kc, vc, cap, d_nkv, d_pos, gate=gate, rope_n_rot=64, rope_freq_base=1e7,
                             n_splits=n_splits)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for _ in range(2):  # two calls in a row on the same static scratch
        out = torch.full((n_q, 16, 256), float("nan"), device=dev)
        a = _args(sq, q, gate, kc, vc, cap, d_nkv, d_pos, out, n_splits)
        rc = sq.lib().sqmix_fa_decode_noalloc(ctypes.byref(a), stream)
        assert rc == sq.SQMIX_OK, sq.lib().sqmix_last_error()
        torch.cuda.synchronize()
        got = out.cpu().numpy().astype(np.float64)
        ref = want.cpu().numpy().astype(np.float64)
        assert np.isfinite(got).all()
        assert np.abs(got - ref).max() <= ATTN_TOL * np.abs(ref).max()
    assert sq.lib().sqmix_fa_noalloc_status(stream) == sq.SQMIX_OK
