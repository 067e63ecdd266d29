"""Parity at the benchmark's own sizes: the configuration-3 decode (172 032 keys per
layer, one split per SM, 1 query token with the fused append of its row, and the
2-token MTP verify query with both draft rows appended) and the configuration-2
prefill (pp512 and pp2048 after a 32 768-token q4_0 prefix), each against the CPU
oracle on the same cache.

The cache rows below the step are imported from oracle-quantised ggml rows; the
step's own rows are written by the kernels (fused append for decode, the append
kernel for prefill, K rotated at its position) and read back, so the oracle attends
over exactly the bytes the GPU read.  The appended rows are checked separately
against the oracle's quantisation of the rotated rows (an ulp of the rotation may
move a value across a rounding boundary, as in test_append_with_fused_rope).

Bars: attention max|gpu - ref| <= 2e-3 * max|ref| against the fp32 oracle; LSE
within 1e-3 absolute (the LSE here is about ln(n_kv) + 1, near 13).
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ATTN_TOL = 2e-3
N_ROT, THETA = 64, 1e7


@pytest.fixture(scope="module")
def sq():
    import sqmix

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return sqmix


def rel_err(got, want):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    return np.abs(got - want).max() / max(np.abs(want).max(), 1e-30)


def cap_for(n):
    return max(256, (n + 255) // 256 * 256)


def import_rows(sq, oracle, k, v, cap):
    """Fresh tiled caches holding the oracle q4_0 quantisation of k, v [n][2][256] in rows 0..n-1."""
    n = k.shape[0]
    kc, vc = sq.new_kv_cache(cap), sq.new_kv_cache(cap)
    if n:
        kq = oracle.q4_0_quantize(k.reshape(n, 512))
        vq = oracle.q4_0_quantize(v.reshape(n, 512))
        sq.kv_convert_rows(kc, cap, "k", 0, n, torch.from_numpy(kq).cuda(), to_rows=False)
        sq.kv_convert_rows(vc, cap, "v", 0, n, torch.from_numpy(vq).cuda(), to_rows=False)
    return kc, vc


def check_appended_rows(sq, oracle, kc, vc, cap, k_new, v_new, pos0):
    """Rows pos0.. written by a kernel: V bit-exact; K equal to the oracle's quantisation
    of the rotated row up to rotation ulps (a differing block dequantises within a step)."""
    T = k_new.shape[0]
    got_k = sq.kv_convert_rows(kc, cap, "k", pos0, T).cpu().numpy()
    got_v = sq.kv_convert_rows(vc, cap, "v", pos0, T).cpu().numpy()
    assert np.array_equal(got_v, oracle.q4_0_quantize(v_new.reshape(T, 512)))
    want_k = oracle.q4_0_quantize(oracle.rope_text(k_new, pos0, THETA, N_ROT).reshape(T, 512))
    gb, wb = got_k.reshape(-1, 18), want_k.reshape(-1, 18)
    assert (gb != wb).any(axis=1).mean() < 0.05
    gd = oracle.q4_0_dequantize(got_k, 512).reshape(-1, 32)
    wd = oracle.q4_0_dequantize(want_k, 512).reshape(-1, 32)
    step = np.abs(wd).max(axis=1) / 8 + 1e-12
    assert (np.abs(gd - wd).max(axis=1) <= step * 1.0001).all()


def dequantized_cache(sq, oracle, kc, vc, cap, n_kv):
    """The cache as the kernels read it, dequantised: k, v [n_kv][2][256] f32."""
    kq = sq.kv_convert_rows(kc, cap, "k", 0, n_kv).cpu().numpy()
    vq = sq.kv_convert_rows(vc, cap, "v", 0, n_kv).cpu().numpy()
    kd = oracle.q4_0_dequantize(kq, 512).reshape(n_kv, 2, 256)
    vd = oracle.q4_0_dequantize(vq, 512).reshape(n_kv, 2, 256)
    return kd, vd


@pytest.mark.parametrize("n_q,configs", [(1, (0, 3, 4, 5)), (2, (0, 2, 6))])
def test_decode_config3_172k_keys(sq, oracle, n_q, configs):
    """Configuration 3: 172 032 keys, default split count of each kernel configuration,
    the step's n_q rows appended by the decode kernel itself (n_new = n_q; rewritten
    identically by every configuration), RoPE 64 / 1e7, sigmoid gate."""
    n_kv = 172032
    q_pos0 = n_kv - n_q
    rng = np.random.default_rng(172032 + n_q)
    k = rng.standard_normal((n_kv, 2, 256), dtype=np.float32)
    v = rng.standard_normal((n_kv, 2, 256), dtype=np.float32)
    q = rng.standard_normal((n_q, 16, 256), dtype=np.float32)
    gate = rng.standard_normal((n_q, 16, 256), dtype=np.float32)
    cap = cap_for(n_kv)
    kc, vc = import_rows(sq, oracle, k[:q_pos0], v[:q_pos0], cap)
    d_nkv = torch.tensor([n_kv], dtype=torch.int64, device="cuda")
    d_pos = torch.tensor([q_pos0], dtype=torch.int64, device="cuda")
    results = {}
    for config in configs:
        lse = torch.empty((n_q, 16), dtype=torch.float32, device="cuda")
        out = sq.flash_attn_ext(torch.from_numpy(q).cuda(), kc, vc, cap, d_nkv, d_pos,
                                gate=torch.from_numpy(gate).cuda(), rope_n_rot=N_ROT, rope_freq_base=THETA, lse=lse,
                                k_new=torch.from_numpy(k[q_pos0:]).cuda(), v_new=torch.from_numpy(v[q_pos0:]).cuda(),
                                config=config)
        torch.cuda.synchronize()
        results[config] = (out.cpu().numpy(), lse.cpu().numpy())
    check_appended_rows(sq, oracle, kc, vc, cap, k[q_pos0:], v[q_pos0:], q_pos0)
    kd, vd = dequantized_cache(sq, oracle, kc, vc, cap, n_kv)
    del k, v
    want, wlse = oracle.attn(oracle.rope_text(q, q_pos0, THETA, N_ROT), kd, vd, gate, q_pos0=q_pos0, scale=1 / 16,
                             want_lse=True)
    for config, (got, got_lse) in results.items():
        assert np.isfinite(got).all(), config
        assert rel_err(got, want) <= ATTN_TOL, config
        assert np.abs(got_lse - wlse).max() < 1e-3, config


@pytest.mark.parametrize("T", [512, 2048])
def test_prefill_config2_on_32768_prefix(sq, oracle, T):
    """Configuration 2: T new tokens appended (q4_0, K rotated) after a 32 768-token q4_0
    prefix, then causal attention of the T queries (bf16) with the sigmoid gate.  pp512 is
    compared in full; pp2048 on its first, middle and last 64 query tokens (the oracle's
    double-precision attention over ~34K keys costs about 3 ms per query token)."""
    P = 32768
    n_kv = P + T
    rng = np.random.default_rng(32768 + T)
    k = rng.standard_normal((n_kv, 2, 256), dtype=np.float32)
    v = rng.standard_normal((n_kv, 2, 256), dtype=np.float32)
    cap = cap_for(n_kv)
    kc, vc = import_rows(sq, oracle, k[:P], v[:P], cap)
    sq.set_rows_q4_0(torch.from_numpy(k[P:]).cuda(), torch.from_numpy(v[P:]).cuda(),
                     torch.arange(P, n_kv, device="cuda"), kc, vc, cap, rope_n_rot=N_ROT, rope_freq_base=THETA)
    q_t = torch.from_numpy(rng.standard_normal((T, 16, 256), dtype=np.float32)).to(torch.bfloat16).cuda()
    gate = rng.standard_normal((T, 16, 256), dtype=np.float32)
    d_nkv = torch.tensor([n_kv], dtype=torch.int64, device="cuda")
    d_pos = torch.tensor([P], dtype=torch.int64, device="cuda")
    lse = torch.empty((T, 16), dtype=torch.float32, device="cuda")
    out = sq.flash_attn_prefill(q_t, kc, vc, cap, d_nkv, d_pos, gate=torch.from_numpy(gate).cuda(),
                                rope_n_rot=N_ROT, rope_freq_base=THETA, lse=lse)
    torch.cuda.synchronize()
    got, got_lse = out.cpu().numpy(), lse.cpu().numpy()
    check_appended_rows(sq, oracle, kc, vc, cap, k[P:], v[P:], P)
    kd, vd = dequantized_cache(sq, oracle, kc, vc, cap, n_kv)
    del k, v
    q_used = oracle.rope_text(q_t.float().cpu().numpy(), P, THETA, N_ROT)
    blocks = [(0, T)] if T <= 512 else [(0, 64), (T // 2 - 32, T // 2 + 32), (T - 64, T)]
    for t0, t1 in blocks:
        want, wlse = oracle.attn(q_used[t0:t1], kd, vd, gate[t0:t1], q_pos0=P + t0, scale=1 / 16, want_lse=True)
        assert np.isfinite(got[t0:t1]).all()
        assert rel_err(got[t0:t1], want) <= ATTN_TOL, (t0, t1)
        assert np.abs(got_lse[t0:t1] - wlse).max() < 1e-3, (t0, t1)
