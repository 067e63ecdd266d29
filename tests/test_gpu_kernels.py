"""GPU parity tests: the sqmix CUDA kernels, called through the C ABI, against the
CPU oracle on the same seeded inputs.

Bars: q4_0 quantisation bit-exact with quantize_row_q4_0;
attention max|gpu - ref| <= 2e-3 * max|ref| against the fp32 oracle on the same
dequantised cache; GDN outputs and states within 1e-3 relative.
"""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "q4_0_golden.npz")
ATTN_TOL = 2e-3
GDN_TOL = 1e-3


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


def make_cache_from_rows(sq, k_rows, v_rows, capacity):
    """Import ggml q4_0 rows ([n][288] uint8) into fresh tiled caches."""
    kc = sq.new_kv_cache(capacity)
    vc = sq.new_kv_cache(capacity)
    n = k_rows.shape[0]
    sq.kv_convert_rows(kc, capacity, "k", 0, n, torch.from_numpy(k_rows).cuda(), to_rows=False)
    sq.kv_convert_rows(vc, capacity, "v", 0, n, torch.from_numpy(v_rows).cuda(), to_rows=False)
    return kc, vc


def quantized_kv(oracle, rng, n_kv):
    k = rng.standard_normal((n_kv, 2, 256)).astype(np.float32)
    v = rng.standard_normal((n_kv, 2, 256)).astype(np.float32)
    kq = oracle.q4_0_quantize(k.reshape(n_kv, 512))
    vq = oracle.q4_0_quantize(v.reshape(n_kv, 512))
    kd = oracle.q4_0_dequantize(kq, 512).reshape(n_kv, 2, 256)
    vd = oracle.q4_0_dequantize(vq, 512).reshape(n_kv, 2, 256)
    return k, v, kq, vq, kd, vd


# ------------------------------------------------------------ q4_0 append ---

def test_append_bit_exact_vs_gguf_golden(sq):
    d = np.load(GOLDEN)
    x, q = d["x"], d["q"]
    # a token row is 16 blocks (2 heads x 8); the first half of the rows feed K, the rest V
    n_rows = x.shape[0] // 16
    T = n_rows // 2
    xr = x[:2 * T * 16].reshape(2 * T, 512)
    qr = q[:2 * T * 16].reshape(2 * T, 288)
    kx, vx = xr[:T].reshape(T, 2, 256), xr[T:].reshape(T, 2, 256)
    kq, vq = qr[:T], qr[T:]
    cap = cap_for(T)
    kc, vc = sq.new_kv_cache(cap), sq.new_kv_cache(cap)
    rows = torch.arange(T, dtype=torch.int64, device="cuda")
    sq.set_rows_q4_0(torch.from_numpy(kx).cuda(), torch.from_numpy(vx).cuda(), rows, kc, vc, cap)
    got_k = sq.kv_convert_rows(kc, cap, "k", 0, T).cpu().numpy()
    got_v = sq.kv_convert_rows(vc, cap, "v", 0, T).cpu().numpy()
    assert np.array_equal(got_k, kq)
    assert np.array_equal(got_v, vq)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_append_bit_exact_vs_oracle(sq, oracle, dtype):
    rng = np.random.default_rng(11)
    T, cap = 37, 512
    k = torch.from_numpy(rng.standard_normal((T, 2, 256)).astype(np.float32)).to(dtype)
    v = torch.from_numpy(rng.standard_normal((T, 2, 256)).astype(np.float32) * 3).to(dtype)
    pos = rng.permutation(cap)[:T].astype(np.int64)  # scattered rows (set_rows semantics)
    kc, vc = sq.new_kv_cache(cap), sq.new_kv_cache(cap)
    sq.set_rows_q4_0(k.cuda(), v.cuda(), torch.from_numpy(pos).cuda(), kc, vc, cap)
    got_k = sq.kv_convert_rows(kc, cap, "k", 0, cap).cpu().numpy()
    got_v = sq.kv_convert_rows(vc, cap, "v", 0, cap).cpu().numpy()
    want_k = oracle.q4_0_quantize(k.float().numpy().reshape(T, 512))
    want_v = oracle.q4_0_quantize(v.float().numpy().reshape(T, 512))
    assert np.array_equal(got_k[pos], want_k)
    assert np.array_equal(got_v[pos], want_v)
    untouched = np.setdiff1d(np.arange(cap), pos)
    assert not got_k[untouched].any() and not got_v[untouched].any()


def test_append_with_fused_rope(sq, oracle):
    rng = np.random.default_rng(12)
    T, cap, pos0 = 24, 172032 + 256, 172000
    k = rng.standard_normal((T, 2, 256)).astype(np.float32)
    v = rng.standard_normal((T, 2, 256)).astype(np.float32)
    kc, vc = sq.new_kv_cache(cap), sq.new_kv_cache(cap)
    rows = torch.arange(pos0, pos0 + T, dtype=torch.int64, device="cuda")
    sq.set_rows_q4_0(torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), rows, kc, vc, cap,
                     rope_n_rot=64, rope_freq_base=1e7)
    got = sq.kv_convert_rows(kc, cap, "k", pos0, T).cpu().numpy()
    want = oracle.q4_0_quantize(oracle.rope_text(k, pos0, 1e7, 64).reshape(T, 512))
    gb, wb = got.reshape(-1, 18), want.reshape(-1, 18)
    mism = (gb != wb).any(axis=1)
    # sincosf on the GPU and libm on the host may differ by an ulp, which can move a
    # value across a rounding boundary; those blocks must still dequantise within a step.
    assert mism.mean() < 0.02
    gd = oracle.q4_0_dequantize(got, 512).reshape(-1, 32)
    wd = oracle.q4_0_dequantize(want, 512).reshape(-1, 32)
    step = np.abs(wd).max(axis=1) / 8 + 1e-12
    assert (np.abs(gd - wd).max(axis=1) <= step * 1.0001).all()
    assert np.array_equal(sq.kv_convert_rows(vc, cap, "v", pos0, T).cpu().numpy(),
                          oracle.q4_0_quantize(v.reshape(T, 512)))


def test_convert_roundtrip_and_layout(sq):
    rng = np.random.default_rng(13)
    cap = 512
    rows = rng.integers(0, 256, (cap, 288), dtype=np.uint8)
    for which in ("k", "v"):
        t = sq.new_kv_cache(cap)
        sq.kv_convert_rows(t, cap, which, 0, cap, torch.from_numpy(rows).cuda(), to_rows=False)
        back = sq.kv_convert_rows(t, cap, which, 0, cap).cpu().numpy()
        assert np.array_equal(back, rows)
        # the tiled image is a permutation of the rows' bytes within each 16-token group
        tiled = t.cpu().numpy().reshape(cap // 16, 4608)
        grp = rows.reshape(cap // 16, 4608)
        assert np.array_equal(np.sort(tiled, axis=1), np.sort(grp, axis=1))


# ------------------------------------------------------ attention decode ---

def run_fa(sq, q, kc, vc, cap, n_kv, q_pos0, gate=None, rope=0, n_splits=0, lse=False, config=0):
    dev_nkv = torch.tensor([n_kv], dtype=torch.int64, device="cuda")
    dev_pos = torch.tensor([q_pos0], dtype=torch.int64, device="cuda")
    lse_t = torch.empty((q.shape[0], 16), dtype=torch.float32, device="cuda") if lse else None
    out = sq.flash_attn_ext(q, kc, vc, cap, dev_nkv, dev_pos, gate=gate, rope_n_rot=rope,
                            rope_freq_base=1e7, lse=lse_t, n_splits=n_splits, config=config)
    torch.cuda.synchronize()
    return out.cpu().numpy(), (lse_t.cpu().numpy() if lse else None)


def test_fa_decode_overlap_chain(sq, oracle):
    """Back-to-back launches over several layers with SQMIX_FA_OVERLAP_PREV, eagerly and
    replayed from a CUDA graph: each decode prefetches before the previous launch ends."""
    rng = np.random.default_rng(21)
    n_kv, n_layers = 3000, 3
    cap = cap_for(n_kv)
    layers = []
    for _ in range(n_layers):
        _, _, kq, vq, kd, vd = quantized_kv(oracle, rng, n_kv)
        kc, vc = make_cache_from_rows(sq, kq, vq, cap)
        q = rng.standard_normal((1, 16, 256)).astype(np.float32)
        gate = rng.standard_normal((1, 16, 256)).astype(np.float32)
        want = oracle.attn(q, kd, vd, gate, q_pos0=n_kv - 1, scale=1 / 16)
        layers.append((kc, vc, torch.from_numpy(q).cuda(), torch.from_numpy(gate).cuda(), want))
    d_nkv = torch.tensor([n_kv], dtype=torch.int64, device="cuda")
    d_pos = torch.tensor([n_kv - 1], dtype=torch.int64, device="cuda")
    ws = sq.new_fa_workspace(1, 0, "cuda")
    outs = [torch.zeros((1, 16, 256), device="cuda") for _ in range(n_layers)]

    def chain():
        for (kc, vc, q, gate, _), out in zip(layers, outs):
            sq.flash_attn_ext(q, kc, vc, cap, d_nkv, d_pos, gate=gate, out=out, workspace=ws,
                              overlap_prev=True)

    torch.cuda.synchronize()
    chain()
    torch.cuda.synchronize()
    for (_, _, _, _, want), out in zip(layers, outs):
        assert rel_err(out.cpu().numpy(), want) <= ATTN_TOL
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        chain()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        chain()
    for _ in range(2):
        for out in outs:
            out.zero_()
        graph.replay()
        torch.cuda.synchronize()
        for (_, _, _, _, want), out in zip(layers, outs):
            assert rel_err(out.cpu().numpy(), want) <= ATTN_TOL
    del graph
    sq.fa_status(ws)


def test_fa_decode_config0(sq, oracle):
    # 1 query, 16/2 heads, d 256, 4096 q4_0 keys, scale 1/16, gate
    rng = np.random.default_rng(20)
    n_kv = 4096
    _, _, kq, vq, kd, vd = quantized_kv(oracle, rng, n_kv)
    kc, vc = make_cache_from_rows(sq, kq, vq, n_kv)
    q = rng.standard_normal((1, 16, 256)).astype(np.float32)
    gate = rng.standard_normal((1, 16, 256)).astype(np.float32)
    out, lse = run_fa(sq, torch.from_numpy(q).cuda(), kc, vc, n_kv, n_kv, n_kv - 1,
                      gate=torch.from_numpy(gate).cuda(), lse=True)
    want, wlse = oracle.attn(q, kd, vd, gate, q_pos0=n_kv - 1, scale=1 / 16, want_lse=True)
    assert rel_err(out, want) <= ATTN_TOL
    assert np.abs(lse - wlse).max() < 1e-3


@pytest.mark.parametrize("n_kv", [1, 15, 16, 17, 31, 33, 64, 65, 255, 257, 1000])
@pytest.mark.parametrize("n_q,config", [(1, 0), (2, 0), (1, 4), (2, 6)])
def test_fa_decode_ragged(sq, oracle, n_kv, n_q, config):
    rng = np.random.default_rng(100 + n_kv * 3 + n_q)
    _, _, kq, vq, kd, vd = quantized_kv(oracle, rng, n_kv)
    cap = cap_for(n_kv)
    kc, vc = make_cache_from_rows(sq, kq, vq, cap)
    q = rng.standard_normal((n_q, 16, 256)).astype(np.float32)
    q_pos0 = max(n_kv - n_q, 0)
    out, lse = run_fa(sq, torch.from_numpy(q).cuda(), kc, vc, cap, n_kv, q_pos0, lse=True, config=config)
    want, wlse = oracle.attn(q, kd, vd, None, q_pos0=q_pos0, scale=1 / 16, want_lse=True)
    assert rel_err(out, want) <= ATTN_TOL
    assert np.abs(lse - wlse).max() < 1e-3


@pytest.mark.parametrize("n_splits", [1, 3, 7, 16, 17, 148, 300])  # <= 16: the per-thread merge
def test_fa_decode_split_counts(sq, oracle, n_splits):
    rng = np.random.default_rng(30 + n_splits)
    n_kv = 1500
    _, _, kq, vq, kd, vd = quantized_kv(oracle, rng, n_kv)
    cap = cap_for(n_kv)
    kc, vc = make_cache_from_rows(sq, kq, vq, cap)
    q = rng.standard_normal((2, 16, 256)).astype(np.float32)
    out, lse = run_fa(sq, torch.from_numpy(q).cuda(), kc, vc, cap, n_kv, n_kv - 2, n_splits=n_splits, lse=True)
    want, wlse = oracle.attn(q, kd, vd, None, q_pos0=n_kv - 2, scale=1 / 16, want_lse=True)
    assert rel_err(out, want) <= ATTN_TOL
    assert np.abs(lse - wlse).max() < 1e-3


@pytest.mark.parametrize("config", [3, 4, 5])
@pytest.mark.parametrize("n_kv,n_splits", [(1, 0), (17, 3), (257, 0), (1000, 7), (5000, 0), (5000, 300)])
def test_fa_decode_config3_twelve_warps(sq, oracle, n_kv, n_splits, config):
    """The n_q = 1 configurations 3 (6 warps per KV head, 3 x 55.3 KB ring slots), 4 (two
    CTAs per SM, 4 warps per KV head, the one-MMA V offset correction) and 5 (3 with that
    correction): RoPE, gate, lse and the fused append of the step's row, against the
    oracle."""
    rng = np.random.default_rng(90 + n_kv + n_splits)
    k = rng.standard_normal((n_kv, 2, 256)).astype(np.float32)
    v = rng.standard_normal((n_kv, 2, 256)).astype(np.float32)
    cap = cap_for(n_kv)
    kc, vc = sq.new_kv_cache(cap), sq.new_kv_cache(cap)
    kd_t, vd_t = torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda()
    q_pos0 = n_kv - 1
    if q_pos0 > 0:
        sq.set_rows_q4_0(kd_t[:q_pos0], vd_t[:q_pos0], torch.arange(q_pos0, device="cuda"), kc, vc, cap,
                         rope_n_rot=64, rope_freq_base=1e7)
    q = rng.standard_normal((1, 16, 256)).astype(np.float32)
    gate = rng.standard_normal((1, 16, 256)).astype(np.float32)
    lse = torch.empty((1, 16), device="cuda")
    ws = sq.new_fa_workspace(1, 300)
    out = sq.flash_attn_ext(torch.from_numpy(q).cuda(), kc, vc, cap,
                            torch.tensor([n_kv], dtype=torch.int64, device="cuda"),
                            torch.tensor([q_pos0], dtype=torch.int64, device="cuda"),
                            gate=torch.from_numpy(gate).cuda(), rope_n_rot=64, rope_freq_base=1e7, lse=lse,
                            k_new=kd_t[q_pos0:], v_new=vd_t[q_pos0:], workspace=ws, n_splits=n_splits, config=config)
    torch.cuda.synchronize()
    sq.fa_status(ws)
    kq = oracle.q4_0_quantize(oracle.rope_text(k, 0, 1e7, 64).reshape(n_kv, 512))
    vq = oracle.q4_0_quantize(v.reshape(n_kv, 512))
    assert np.array_equal(sq.kv_convert_rows(kc, cap, "k", 0, n_kv).cpu().numpy(), kq)
    assert np.array_equal(sq.kv_convert_rows(vc, cap, "v", 0, n_kv).cpu().numpy(), vq)
    kd = oracle.q4_0_dequantize(kq, 512).reshape(n_kv, 2, 256)
    vd = oracle.q4_0_dequantize(vq, 512).reshape(n_kv, 2, 256)
    want, wlse = oracle.attn(oracle.rope_text(q, q_pos0, 1e7, 64), kd, vd, gate, q_pos0=q_pos0, scale=1 / 16,
                             want_lse=True)
    assert rel_err(out.cpu().numpy(), want) <= ATTN_TOL
    assert np.abs(lse.cpu().numpy() - wlse).max() < 1e-3


@pytest.mark.parametrize("n_q,config", [(1, 0), (2, 0), (1, 4), (1, 5), (2, 6)])
@pytest.mark.parametrize("n_splits", [1, 0])
@pytest.mark.parametrize("v_amax", [1.0, 60000.0])
def test_fa_decode_rising_scores(sq, oracle, n_q, config, n_splits, v_amax):
    """Scores that climb along the cache (about 0.3 log2 units per 16-token group), so the
    running maximum keeps moving past the lazy-update threshold in every warp, with V
    blocks up to `v_amax` (60000: P * V scale stays near the top of the f16 range)."""
    rng = np.random.default_rng(7 + n_q + n_splits + int(v_amax))
    n_kv = 3000
    u = rng.standard_normal(256)
    u /= np.linalg.norm(u)
    ramp = np.linspace(0.0, 40.0, n_kv)  # score of the aligned component, in nats
    k = rng.standard_normal((n_kv, 2, 256)) + ramp[:, None, None] * u[None, None, :]
    v = rng.standard_normal((n_kv, 2, 256))
    v *= v_amax / np.abs(v).max()
    q = 16.0 * u[None, None, :] + 0.5 * rng.standard_normal((n_q, 16, 256))
    k, v, q = (x.astype(np.float32) for x in (k, v, q))
    kq = oracle.q4_0_quantize(k.reshape(n_kv, 512))
    vq = oracle.q4_0_quantize(v.reshape(n_kv, 512))
    kd = oracle.q4_0_dequantize(kq, 512).reshape(n_kv, 2, 256)
    vd = oracle.q4_0_dequantize(vq, 512).reshape(n_kv, 2, 256)
    cap = cap_for(n_kv)
    kc, vc = make_cache_from_rows(sq, kq, vq, cap)
    q_pos0 = n_kv - n_q
    out, lse = run_fa(sq, torch.from_numpy(q).cuda(), kc, vc, cap, n_kv, q_pos0, n_splits=n_splits, lse=True,
                      config=config)
    want, wlse = oracle.attn(q, kd, vd, None, q_pos0=q_pos0, scale=1 / 16, want_lse=True)
    assert np.isfinite(out).all()
    assert rel_err(out, want) <= ATTN_TOL
    # lse here is ~45: rounding Q to f16 for the tensor cores alone moves it by ~2e-3
    # (oracle with f16 Q), so its bound is relative to its size
    assert np.abs(lse - wlse).max() < 1e-4 * np.abs(wlse).max()


@pytest.mark.parametrize("n_q", [1, 2])
def test_fa_decode_fused_head_rms_norm(sq, oracle, n_q):
    """Q and the appended K rows RMS-normalised per head with the attn_q_norm /
    attn_k_norm weights inside the decode kernel (attn.rs:66-84, :166-175), then
    RoPE, append and attention, against the oracle chain rms_norm -> rope -> q4_0."""
    rng = np.random.default_rng(70 + n_q)
    n_kv = 1200
    k = (rng.standard_normal((n_kv, 2, 256)) * 3.0).astype(np.float32)
    v = rng.standard_normal((n_kv, 2, 256)).astype(np.float32)
    wq = rng.uniform(0.5, 1.5, 256).astype(np.float32)
    wk = rng.uniform(0.5, 1.5, 256).astype(np.float32)
    q = (rng.standard_normal((n_q, 16, 256)) * 2.0).astype(np.float32)
    gate = rng.standard_normal((n_q, 16, 256)).astype(np.float32)
    q_pos0 = n_kv - n_q
    kn = oracle.rms_norm(k, 1e-6, w=wk)  # the history rows were normalised when appended
    cap = cap_for(n_kv)
    kc, vc = sq.new_kv_cache(cap), sq.new_kv_cache(cap)
    sq.set_rows_q4_0(torch.from_numpy(kn[:q_pos0]).cuda(), torch.from_numpy(v[:q_pos0]).cuda(),
                     torch.arange(q_pos0, device="cuda"), kc, vc, cap, rope_n_rot=64, rope_freq_base=1e7)
    out = sq.flash_attn_ext(torch.from_numpy(q).cuda(), kc, vc, cap,
                            torch.tensor([n_kv], dtype=torch.int64, device="cuda"),
                            torch.tensor([q_pos0], dtype=torch.int64, device="cuda"),
                            gate=torch.from_numpy(gate).cuda(), rope_n_rot=64, rope_freq_base=1e7,
                            k_new=torch.from_numpy(k[q_pos0:]).cuda(), v_new=torch.from_numpy(v[q_pos0:]).cuda(),
                            q_norm=torch.from_numpy(wq).cuda(), k_norm=torch.from_numpy(wk).cuda(), norm_eps=1e-6)
    torch.cuda.synchronize()
    kq = oracle.q4_0_quantize(oracle.rope_text(kn, 0, 1e7, 64).reshape(n_kv, 512))
    vq = oracle.q4_0_quantize(v.reshape(n_kv, 512))
    got_k = sq.kv_convert_rows(kc, cap, "k", q_pos0, n_q).cpu().numpy()
    # the appended rows, quantised from the device-normalised K: a last-bit difference
    # in the norm may move a value across a rounding boundary, so almost all (not all)
    # blocks must be bit-identical to the oracle's
    same = (got_k.reshape(n_q * 16, 18) == kq[q_pos0:].reshape(n_q * 16, 18)).all(axis=1)
    assert same.mean() >= 0.9, same
    kd = oracle.q4_0_dequantize(np.concatenate([kq[:q_pos0], got_k]), 512).reshape(n_kv, 2, 256)
    vd = oracle.q4_0_dequantize(vq, 512).reshape(n_kv, 2, 256)
    qn = oracle.rope_text(oracle.rms_norm(q, 1e-6, w=wq), q_pos0, 1e7, 64)
    want = oracle.attn(qn, kd, vd, gate, q_pos0=q_pos0, scale=1 / 16)
    assert rel_err(out.cpu().numpy(), want) <= ATTN_TOL


def test_fa_decode_prefix_causal(sq, oracle):
    # queries at positions far below n_kv: only keys j <= q_pos0 + t count (graph.rs:553-559)
    rng = np.random.default_rng(40)
    n_kv = 900
    _, _, kq, vq, kd, vd = quantized_kv(oracle, rng, n_kv)
    cap = cap_for(n_kv)
    kc, vc = make_cache_from_rows(sq, kq, vq, cap)
    q = rng.standard_normal((2, 16, 256)).astype(np.float32)
    for q_pos0 in (0, 100, 511):
        out, _ = run_fa(sq, torch.from_numpy(q).cuda(), kc, vc, cap, n_kv, q_pos0)
        want = oracle.attn(q, kd, vd, None, q_pos0=q_pos0, scale=1 / 16)
        assert rel_err(out, want) <= ATTN_TOL


def test_fa_decode_qg_interleaved_bf16_rope(sq, oracle):
    # q and gate read in place from the QG projection (attn.rs:131-158): per head
    # [q(256), gate(256)], head stride 512; RoPE on q fused into the kernel prologue.
    rng = np.random.default_rng(41)
    n_kv = 700
    _, _, kq, vq, kd, vd = quantized_kv(oracle, rng, n_kv)
    cap = cap_for(n_kv)
    kc, vc = make_cache_from_rows(sq, kq, vq, cap)
    qg = torch.from_numpy(rng.standard_normal((2, 16, 512)).astype(np.float32)).to(torch.bfloat16)
    qg_d = qg.cuda()
    q_pos0 = n_kv - 2
    out, _ = run_fa(sq, qg_d[:, :, :256], kc, vc, cap, n_kv, q_pos0, gate=qg_d[:, :, 256:], rope=64)
    q = qg[:, :, :256].float().numpy()
    gate = qg[:, :, 256:].float().numpy()
    q_rot = oracle.rope_text(q, q_pos0, 1e7, 64)
    want = oracle.attn(q_rot, kd, vd, gate, q_pos0=q_pos0, scale=1 / 16)
    assert rel_err(out, want) <= ATTN_TOL


def test_fa_decode_after_gpu_append(sq, oracle):
    # append (bit-exact) then attend: the two kernels agree on the tiled layout
    rng = np.random.default_rng(42)
    n_kv = 333
    k = rng.standard_normal((n_kv, 2, 256)).astype(np.float32)
    v = rng.standard_normal((n_kv, 2, 256)).astype(np.float32)
    cap = cap_for(n_kv)
    kc, vc = sq.new_kv_cache(cap), sq.new_kv_cache(cap)
    sq.set_rows_q4_0(torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(),
                     torch.arange(n_kv, dtype=torch.int64, device="cuda"), kc, vc, cap)
    kd = oracle.q4_0_dequantize(oracle.q4_0_quantize(k.reshape(n_kv, 512)), 512).reshape(n_kv, 2, 256)
    vd = oracle.q4_0_dequantize(oracle.q4_0_quantize(v.reshape(n_kv, 512)), 512).reshape(n_kv, 2, 256)
    q = rng.standard_normal((1, 16, 256)).astype(np.float32)
    out, _ = run_fa(sq, torch.from_numpy(q).cuda(), kc, vc, cap, n_kv, n_kv - 1)
    want = oracle.attn(q, kd, vd, None, q_pos0=n_kv - 1, scale=1 / 16)
    assert rel_err(out, want) <= ATTN_TOL


def test_merge_lse_across_parts(sq, oracle):
    # split-KV across "GPUs": 3 disjoint key ranges, each attended on its own cache,
    # merged by log-sum-exp, gate applied after the merge.
    rng = np.random.default_rng(43)
    n_kv = 1200
    _, _, kq, vq, kd, vd = quantized_kv(oracle, rng, n_kv)
    q = rng.standard_normal((1, 16, 256)).astype(np.float32)
    gate = rng.standard_normal((1, 16, 256)).astype(np.float32)
    bounds = [0, 300, 301, n_kv]
    o_parts, l_parts = [], []
    for a, b in zip(bounds[:-1], bounds[1:]):
        cap = cap_for(b - a)
        kc, vc = make_cache_from_rows(sq, kq[a:b], vq[a:b], cap)
        o, l = run_fa(sq, torch.from_numpy(q).cuda(), kc, vc, cap, b - a, 10 ** 7, lse=True)
        o_parts.append(o.reshape(16, 256))
        l_parts.append(l.reshape(16))
    out = sq.attn_merge_lse(torch.from_numpy(np.stack(o_parts)).cuda(),
                            torch.from_numpy(np.stack(l_parts)).cuda(),
                            gate=torch.from_numpy(gate.reshape(16, 256)).cuda())
    want = oracle.attn(q, kd, vd, gate, q_pos0=n_kv - 1, scale=1 / 16)
    assert rel_err(out.cpu().numpy(), want.reshape(16, 256)) <= ATTN_TOL


# ------------------------------------------------------------------ GDN ---

def gdn_case(rng, n_seqs, T, Hk=16, Hv=32, d=128, state_scale=0.02, n_planes=1):
    q = rng.standard_normal((n_seqs, T, Hk, d)).astype(np.float32)
    k = rng.standard_normal((n_seqs, T, Hk, d)).astype(np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((n_seqs, T, Hv, d)).astype(np.float32)
    a_log = rng.uniform(0, 2.7, Hv).astype(np.float32)
    dt_bias = rng.standard_normal(Hv).astype(np.float32)
    sp = np.log1p(np.exp(rng.standard_normal((n_seqs, T, Hv)) + dt_bias))
    g = (-np.exp(a_log) * sp).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal((n_seqs, T, Hv))))).astype(np.float32)
    S = (rng.standard_normal((n_seqs, n_planes, Hv, d, d)) * state_scale).astype(np.float32)
    return q, k, v, g, beta, S


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_gdn_decode_config1(sq, oracle, dtype):
    # BASELINE config 1 decode: 32 value heads over 16 q/k heads, d 128, one token
    rng = np.random.default_rng(50)
    q, k, v, g, beta, S = gdn_case(rng, 1, 1)
    tq, tk, tv = (torch.from_numpy(x).to(dtype) for x in (q, k, v))
    st = torch.from_numpy(S).cuda()
    out = sq.gated_delta_net(tq.cuda(), tk.cuda(), tv.cuda(), torch.from_numpy(g).cuda(),
                             torch.from_numpy(beta).cuda(), st, n_planes=1, n_snap=1)
    torch.cuda.synchronize()
    qf, kf, vf = (x.float().numpy() for x in (tq, tk, tv))
    want, snaps = oracle.gdn(qf[0], kf[0], vf[0], g[0], beta[0], S[0, 0], n_snap=1)
    assert rel_err(out.cpu().numpy()[0], want) <= GDN_TOL
    assert rel_err(st.cpu().numpy()[0, 0], snaps[0]) <= GDN_TOL


def test_gdn_snapshots_sel_and_batch(sq, oracle):
    # 2-token verify batch (n_rs = 1): read plane sel, write slot 0 (final) and slot 1
    # (after 1 token) in place; three independent sequences with different sel.
    rng = np.random.default_rng(51)
    n_seqs, T, n_planes = 3, 2, 2
    q, k, v, g, beta, S = gdn_case(rng, n_seqs, T, n_planes=n_planes)
    sel = np.array([1, 0, 1], dtype=np.int32)
    st = torch.from_numpy(S).cuda()
    out = sq.gated_delta_net(*(torch.from_numpy(x).cuda() for x in (q, k, v, g, beta)), st,
                             n_planes=n_planes, sel=torch.from_numpy(sel).cuda(), n_snap=2)
    torch.cuda.synchronize()
    st_np, out_np = st.cpu().numpy(), out.cpu().numpy()
    for s in range(n_seqs):
        want, snaps = oracle.gdn(q[s], k[s], v[s], g[s], beta[s], S[s, sel[s]], n_snap=2)
        assert rel_err(out_np[s], want) <= GDN_TOL
        assert rel_err(st_np[s, 0], snaps[0]) <= GDN_TOL
        assert rel_err(st_np[s, 1], snaps[1]) <= GDN_TOL


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("state_ready", [False, True])
def test_gdn_decode_large_batch(sq, oracle, dtype, state_ready):
    """64 sequences x 1 token (the batch of config 4): the launch path for large batches
    (8 value columns per warp), per-sequence input planes through sel, the update
    written to plane 0; outputs and states against the oracle for every sequence."""
    rng = np.random.default_rng(53 + int(state_ready))
    n_seqs, n_planes = 64, 2
    q, k, v, g, beta, S = gdn_case(rng, n_seqs, 1, n_planes=n_planes)
    sel = rng.integers(0, n_planes, n_seqs).astype(np.int32)
    qt, kt, vt = (torch.from_numpy(x).to(dtype).cuda() for x in (q, k, v))
    st = torch.from_numpy(S).cuda()
    out = sq.gated_delta_net(qt, kt, vt, torch.from_numpy(g).cuda(), torch.from_numpy(beta).cuda(), st,
                             n_planes=n_planes, sel=torch.from_numpy(sel).cuda(), state_ready=state_ready)
    torch.cuda.synchronize()
    st_np, out_np = st.cpu().numpy(), out.cpu().numpy()
    qf, kf, vf = (x.float().cpu().numpy() for x in (qt, kt, vt))
    for s in range(n_seqs):
        want, snaps = oracle.gdn(qf[s], kf[s], vf[s], g[s], beta[s], S[s, sel[s]], n_snap=1)
        assert rel_err(out_np[s], want) <= GDN_TOL, s
        assert rel_err(st_np[s, 0], snaps[0]) <= GDN_TOL, s
        if n_planes > 1:  # plane 1 is never written
            assert np.array_equal(st_np[s, 1], S[s, 1]), s


def test_gdn_state_ready_chain_after_conv(sq, oracle):
    """SQMIX_GDN_STATE_READY: the recurrence reads its state before the preceding kernel
    (here the conv front end, then another layer's recurrence) finishes; results equal
    the oracle for each layer of the chain, twice in a row (CUDA-graph-like reuse)."""
    rng = np.random.default_rng(53)
    n_layers, T = 4, 2
    cases = [gdn_case(rng, 1, T, n_planes=2) for _ in range(n_layers)]
    sel = torch.tensor([1], dtype=torch.int32, device="cuda")
    C, K = 8192, 4
    x = torch.from_numpy(rng.standard_normal((1, T, C)).astype(np.float32)).cuda()
    w = torch.from_numpy((rng.standard_normal((C, K)) * 0.5).astype(np.float32)).cuda()
    hist = torch.zeros((1, 1, C, K - 1), device="cuda")
    for rep in range(2):
        states = [torch.from_numpy(c[5]).cuda() for c in cases]
        dev_in = [[torch.from_numpy(a).cuda() for a in c[:5]] for c in cases]
        outs = []
        for l in range(n_layers):
            if l % 2 == 0:  # the conv front end (never touches the recurrent state) runs just before
                sq.gdn_conv(x, w, hist, n_qk_channels=4096, l2_eps=1e-6)
            outs.append(sq.gated_delta_net(*dev_in[l], states[l], n_planes=2, sel=sel, n_snap=2,
                                           state_ready=True))
        torch.cuda.synchronize()
        for l, (q, k, v, g, beta, S) in enumerate(cases):
            want, snaps = oracle.gdn(q[0], k[0], v[0], g[0], beta[0], S[0, 1], n_snap=2)
            assert rel_err(outs[l].cpu().numpy()[0], want) <= GDN_TOL, (rep, l)
            st_np = states[l].cpu().numpy()
            assert rel_err(st_np[0, 0], snaps[0]) <= GDN_TOL
            assert rel_err(st_np[0, 1], snaps[1]) <= GDN_TOL


def test_gdn_fused_l2norm(sq, oracle):
    rng = np.random.default_rng(52)
    q, k, v, g, beta, S = gdn_case(rng, 1, 3)
    q = q * 5.0
    k = k * 0.3
    st = torch.from_numpy(S).cuda()
    out = sq.gated_delta_net(*(torch.from_numpy(x).cuda() for x in (q, k, v, g, beta)), st, l2_eps=1e-6)
    torch.cuda.synchronize()
    qn = oracle.l2norm(q[0], 1e-6)
    kn = oracle.l2norm(k[0], 1e-6)
    want, snaps = oracle.gdn(qn, kn, v[0], g[0], beta[0], S[0, 0])
    assert rel_err(out.cpu().numpy()[0], want) <= GDN_TOL
    assert rel_err(st.cpu().numpy()[0, 0], snaps[0]) <= GDN_TOL


def test_gdn_prefill_512_and_chunk_carry(sq, oracle):
    # config 1 prefill length: 512 tokens; and 256 + 256 == 512 through the state
    rng = np.random.default_rng(53)
    q, k, v, g, beta, S = gdn_case(rng, 1, 512)
    args = [torch.from_numpy(x).cuda() for x in (q, k, v, g, beta)]
    st = torch.from_numpy(S).cuda()
    out = sq.gated_delta_net(*args, st)
    st2 = torch.from_numpy(S).cuda()
    o_a = sq.gated_delta_net(*(a[:, :256] for a in args), st2)
    o_b = sq.gated_delta_net(*(a[:, 256:] for a in args), st2)
    torch.cuda.synchronize()
    want, snaps = oracle.gdn(q[0], k[0], v[0], g[0], beta[0], S[0, 0])
    assert rel_err(out.cpu().numpy()[0], want) <= GDN_TOL
    assert rel_err(st.cpu().numpy()[0, 0], snaps[0]) <= GDN_TOL
    full = out.cpu().numpy()[0, 256:]
    rel = np.abs(o_b.cpu().numpy()[0] - full) / np.maximum(np.abs(full), 1.0)
    assert rel.max() <= 1e-5


# --------------------------------------------------------- state objects ---

def test_kvcache_object_decode_steps(sq, oracle):
    rng = np.random.default_rng(60)
    kv = sq.KvCache(n_layers=2, kv_cap=300)
    assert kv.capacity_alloc == 512
    ks, vs = [], []
    for n in (17, 1, 2):
        kv.begin_step(n)
        kv.upload_step()
        k = rng.standard_normal((n, 2, 256)).astype(np.float32)
        v = rng.standard_normal((n, 2, 256)).astype(np.float32)
        ks.append(k)
        vs.append(v)
        kv.append(1, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda())
        q = rng.standard_normal((min(n, 2), 16, 256)).astype(np.float32)
        if n > 2:
            continue
        out = kv.attention(1, torch.from_numpy(q).cuda())
        torch.cuda.synchronize()
        K = np.concatenate(ks)
        V = np.concatenate(vs)
        nk = K.shape[0]
        kd = oracle.q4_0_dequantize(oracle.q4_0_quantize(K.reshape(nk, 512)), 512).reshape(nk, 2, 256)
        vd = oracle.q4_0_dequantize(oracle.q4_0_quantize(V.reshape(nk, 512)), 512).reshape(nk, 2, 256)
        want = oracle.attn(q, kd, vd, None, q_pos0=kv.step_start, scale=1 / 16)
        assert rel_err(out.cpu().numpy(), want) <= ATTN_TOL
    assert kv.n_used == 20 and kv.n_kv_padded() == 256
    # MTP rollback: accept 1 of the 2 verify tokens -> cursor back to 19, rows kept
    kv.rewind_to(19)
    assert kv.n_used == 19
    with pytest.raises(sq.SqmixError):
        kv.begin_step(1000)
    kv.close()


def test_gdnstate_snapshot_restore_roundtrip(sq):
    st = sq.GdnState(n_layers=2, h_v=32, n_rs=1)
    p = st.planes(1)
    p.copy_(torch.randn_like(p))
    torch.cuda.synchronize()
    blob = st.snapshot_gdn()
    saved0 = st.planes(1)[0].clone()
    st.zero_states()
    st.restore_gdn(blob)
    torch.cuda.synchronize()
    assert torch.equal(st.planes(1)[0], saved0)
    assert int.from_bytes(blob[:8], "little") == len(blob) - 8
    with pytest.raises(sq.SqmixError):
        st.restore_gdn(blob[:-4])
    st.close()


def test_gdnstate_checkpoint_layout_with_conv_history(sq, oracle):
    """Checkpoint bytes as the reference lays them out (graph.rs:316-323): u64 length,
    then per layer state plane 0 ++ conv plane 0; the conv planes are the ones
    gdn_conv updates, and restore brings both back."""
    C, K, n_layers = 8192, 4, 2
    st = sq.GdnState(n_layers=n_layers, h_v=32, n_rs=1, conv_channels=C, d_conv=K)
    rng = np.random.default_rng(54)
    x = torch.from_numpy(rng.standard_normal((1, 3, C)).astype(np.float32)).cuda()
    w = torch.from_numpy((rng.standard_normal((C, K)) * 0.5).astype(np.float32)).cuda()
    for l in range(n_layers):
        st.planes(l).copy_(torch.randn_like(st.planes(l)))
        cp = st.conv_planes(l)
        assert cp.shape == (2, C, K - 1)
        cp.copy_(torch.randn_like(cp))
        # the conv front end reads plane 0 and rewrites it (n_snap 1) in place
        want_hist = cp[0].cpu().numpy().copy()
        sq.gdn_conv(x, w, cp[None], n_planes=2, n_qk_channels=4096, l2_eps=1e-6)
        torch.cuda.synchronize()
        _, want_st = oracle.gdn_conv(x.cpu().numpy()[0], w.cpu().numpy(), np.stack([want_hist, cp[1].cpu().numpy()]),
                                     n_qk=4096, d=128, eps=1e-6)
        assert np.array_equal(cp.cpu().numpy(), want_st)
    blob = st.snapshot_gdn()
    pb, cb = 32 * 128 * 128 * 4, C * (K - 1) * 4
    assert len(blob) == 8 + n_layers * (pb + cb)
    assert int.from_bytes(blob[:8], "little") == len(blob) - 8
    saved = []
    for l in range(n_layers):
        off = 8 + l * (pb + cb)
        assert blob[off:off + pb] == st.planes(l)[0].cpu().numpy().tobytes()
        assert blob[off + pb:off + pb + cb] == st.conv_planes(l)[0].cpu().numpy().tobytes()
        saved.append((st.planes(l)[0].clone(), st.conv_planes(l)[0].clone()))
    st.zero_states()
    st.restore_gdn(blob)
    torch.cuda.synchronize()
    for l in range(n_layers):
        assert torch.equal(st.planes(l)[0], saved[l][0])
        assert torch.equal(st.conv_planes(l)[0], saved[l][1])
        assert not st.conv_planes(l)[1].any()  # only plane 0 is checkpointed
    st.close()


# ------------------------------------------------- fused append + attention ---

@pytest.mark.parametrize("n_q,n_kv", [(1, 4096), (2, 1000), (2, 17), (1, 1), (2, 2)])
def test_fa_decode_fused_append(sq, oracle, n_q, n_kv):
    # one launch appends the step's rows (q4_0, RoPE on K) and attends over the cache:
    # the rows must equal what the standalone append kernel writes, and the output the
    # oracle's attention over the quantised cache
    rng = np.random.default_rng(70 + n_kv + n_q)
    cap = cap_for(n_kv)
    q_pos0 = n_kv - n_q
    k = rng.standard_normal((n_kv, 2, 256)).astype(np.float32)
    v = rng.standard_normal((n_kv, 2, 256)).astype(np.float32)
    kc, vc = sq.new_kv_cache(cap), sq.new_kv_cache(cap)
    kc2, vc2 = sq.new_kv_cache(cap), sq.new_kv_cache(cap)
    rows = torch.arange(n_kv, dtype=torch.int64, device="cuda")
    kd_t, vd_t = torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda()
    # reference path: everything through the standalone append
    sq.set_rows_q4_0(kd_t, vd_t, rows, kc2, vc2, cap, rope_n_rot=64, rope_freq_base=1e7)
    # fused path: history through the append kernel, the step's rows inside attention
    if q_pos0 > 0:
        sq.set_rows_q4_0(kd_t[:q_pos0], vd_t[:q_pos0], rows[:q_pos0], kc, vc, cap, rope_n_rot=64,
                         rope_freq_base=1e7)
    q = rng.standard_normal((n_q, 16, 256)).astype(np.float32)
    gate = rng.standard_normal((n_q, 16, 256)).astype(np.float32)
    ws = sq.new_fa_workspace(n_q)
    out = sq.flash_attn_ext(torch.from_numpy(q).cuda(), kc, vc, cap,
                            torch.tensor([n_kv], dtype=torch.int64, device="cuda"),
                            torch.tensor([q_pos0], dtype=torch.int64, device="cuda"),
                            gate=torch.from_numpy(gate).cuda(), rope_n_rot=64, rope_freq_base=1e7,
                            k_new=kd_t[q_pos0:], v_new=vd_t[q_pos0:], workspace=ws)
    torch.cuda.synchronize()
    sq.fa_status(ws)
    assert torch.equal(kc, kc2) and torch.equal(vc, vc2)
    kq = sq.kv_convert_rows(kc, cap, "k", 0, n_kv).cpu().numpy()
    vq = sq.kv_convert_rows(vc, cap, "v", 0, n_kv).cpu().numpy()
    kd = oracle.q4_0_dequantize(kq, 512).reshape(n_kv, 2, 256)
    vd = oracle.q4_0_dequantize(vq, 512).reshape(n_kv, 2, 256)
    want = oracle.attn(oracle.rope_text(q, q_pos0, 1e7, 64), kd, vd, gate, q_pos0=q_pos0, scale=1 / 16)
    assert rel_err(out.cpu().numpy(), want) <= ATTN_TOL


def test_fa_status_clean_after_runs(sq, oracle):
    rng = np.random.default_rng(80)
    n_kv = 600
    _, _, kq, vq, kd, vd = quantized_kv(oracle, rng, n_kv)
    cap = cap_for(n_kv)
    kc, vc = make_cache_from_rows(sq, kq, vq, cap)
    ws = sq.new_fa_workspace(2)
    q = torch.from_numpy(rng.standard_normal((2, 16, 256)).astype(np.float32)).cuda()
    for _ in range(3):
        sq.flash_attn_ext(q, kc, vc, cap, torch.tensor([n_kv], device="cuda"),
                          torch.tensor([n_kv - 2], device="cuda"), workspace=ws)
    sq.fa_status(ws)  # raises on any device-side error bit
    # n_kv beyond the capacity is clamped on the device and reported, not read out of bounds
    sq.flash_attn_ext(q, kc, vc, cap, torch.tensor([cap + 5000], device="cuda"),
                      torch.tensor([n_kv - 2], device="cuda"), workspace=ws)
    with pytest.raises(sq.SqmixError) as e:
        sq.fa_status(ws)
    assert e.value.code == sq.SQMIX_ERANGE
    sq.fa_status(ws)  # cleared


@pytest.mark.gpu
@pytest.mark.parametrize("n_q", [1, 2])
@pytest.mark.parametrize("n_rot", [0, 32, 48, 64])
def test_fa_decode_rope_widths(sq, oracle, n_q, n_rot):
    """Partial RoPE of width n_rot on Q inside the decode (attn.rs:183-204): widths 0, 32
    and 64 build the one-token Q fragments from registers (each rotation pair in one
    lane), 48 and every two-token query take the staged path; fused append of the new
    rows with the same width."""
    rng = np.random.default_rng(90 + n_rot + n_q)
    n_kv = 777
    k = rng.standard_normal((n_kv, 2, 256)).astype(np.float32)
    v = rng.standard_normal((n_kv, 2, 256)).astype(np.float32)
    q = rng.standard_normal((n_q, 16, 256)).astype(np.float32)
    gate = rng.standard_normal((n_q, 16, 256)).astype(np.float32)
    q_pos0 = n_kv - n_q
    cap = cap_for(n_kv)
    kc, vc = sq.new_kv_cache(cap), sq.new_kv_cache(cap)
    sq.set_rows_q4_0(torch.from_numpy(k[:q_pos0]).cuda(), torch.from_numpy(v[:q_pos0]).cuda(),
                     torch.arange(q_pos0, device="cuda"), kc, vc, cap, rope_n_rot=n_rot, rope_freq_base=1e7)
    out = sq.flash_attn_ext(torch.from_numpy(q).cuda(), kc, vc, cap,
                            torch.tensor([n_kv], dtype=torch.int64, device="cuda"),
                            torch.tensor([q_pos0], dtype=torch.int64, device="cuda"),
                            gate=torch.from_numpy(gate).cuda(), rope_n_rot=n_rot, rope_freq_base=1e7,
                            k_new=torch.from_numpy(k[q_pos0:]).cuda(), v_new=torch.from_numpy(v[q_pos0:]).cuda())
    torch.cuda.synchronize()
    kr = oracle.rope_text(k, 0, 1e7, n_rot) if n_rot else k
    kd = oracle.q4_0_dequantize(oracle.q4_0_quantize(kr.reshape(n_kv, 512)), 512).reshape(n_kv, 2, 256)
    vd = oracle.q4_0_dequantize(oracle.q4_0_quantize(v.reshape(n_kv, 512)), 512).reshape(n_kv, 2, 256)
    qr = oracle.rope_text(q, q_pos0, 1e7, n_rot) if n_rot else q
    want = oracle.attn(qr, kd, vd, gate, q_pos0=q_pos0, scale=1 / 16)
    assert rel_err(out.cpu().numpy(), want) <= ATTN_TOL
