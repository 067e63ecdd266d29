"""Pin the CPU oracle before trusting it.

* q4_0: bit-exact against gguf-py's Q4_0 (golden fixtures, tests/golden/) and the
  reference's own round-trip bound (tests/attn_test.rs:781-833).
* RoPE / attention / gated delta rule: there are no golden vectors in the reference,
  so the oracle is checked against independent float64 numpy restatements of the
  formulas the reference's tests restate (attn_test.rs:148-359, gdn.rs:9-24) and
  against the reference's invariants (gdn_test.rs:282-378,
  gdn_prod_dim_test.rs:245-326).
"""
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "q4_0_golden.npz")


def lcg_pseudo(n, seed, scale=1.0):
    """tests/attn_test.rs:67-75 (and gdn_test.rs:94-103 with scale 0.5)."""
    s = (seed * 2654435761 + 1) & 0xFFFFFFFF
    out = np.empty(n, dtype=np.float32)
    for i in range(n):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = np.float32((s >> 8) / 8388608.0 - 1.0)
    return out * np.float32(scale)


def ramp(n, lo, hi):
    """tests/gdn_test.rs:84-88."""
    i = np.arange(n, dtype=np.float32)
    return (np.float32(lo) + np.float32(hi - lo) * (i + 1) / np.float32(n + 1)).astype(np.float32)


# ----------------------------------------------------------------- q4_0 ---

def test_q4_0_bit_exact_vs_gguf_golden(oracle):
    d = np.load(GOLDEN)
    q = oracle.q4_0_quantize(d["x"])
    mism = np.where(~(q == d["q"]).all(axis=1))[0]
    assert mism.size == 0, f"{mism.size} blocks differ, first {mism[:5]}"


def test_q4_0_dequant_vs_gguf_golden(oracle):
    d = np.load(GOLDEN)
    deq = oracle.q4_0_dequantize(d["q"], 32)
    assert np.array_equal(deq.view(np.uint32), d["deq"].view(np.uint32))


def test_q4_0_roundtrip_error_bound(oracle):
    # tests/attn_test.rs:789-833: err <= |d| and 0.1 < mean(err/d) < 0.4
    data = lcg_pseudo(32 * 8, 7)
    deq = oracle.q4_0_dequantize(oracle.q4_0_quantize(data.reshape(8, 32)), 32).reshape(-1)
    rel = []
    for r in range(8):
        blk, dq = data[r * 32:(r + 1) * 32], deq[r * 32:(r + 1) * 32]
        d = np.abs(dq).max() / 8.0
        if d == 0:
            continue
        rel.extend(np.abs(dq - blk) / d)
    rel = np.array(rel)
    assert rel.max() <= 1.0 + 1e-3
    assert 0.1 < rel.mean() < 0.4


def test_q4_0_layout(oracle):
    # element j -> low nibble of qs[j], element j+16 -> high nibble (kernel_verify.rs:270-292)
    x = np.zeros(32, dtype=np.float32)
    x[0] = -8.0  # d = 1
    x[3] = 3.0
    x[19] = -5.0
    q = oracle.q4_0_quantize(x[None])[0]
    assert int(q[0]) | (int(q[1]) << 8) == 0x3C00  # fp16(1.0)
    assert q[2 + 3] & 0x0F == 3 + 8
    assert q[2 + 3] >> 4 == -5 + 8


def test_f16_conversion_matches_numpy(oracle):
    rng = np.random.default_rng(1)
    vals = np.concatenate([
        rng.standard_normal(2000).astype(np.float32) * np.float32(10.0) ** rng.integers(-9, 6, 2000),
        np.array([0.0, -0.0, 65504, 65519.99, 65520, 1e9, -1e9, 2 ** -25, 2 ** -24, 3 * 2 ** -26,
                  6.1e-5, np.inf, -np.inf], dtype=np.float32)])
    with np.errstate(over="ignore"):
        want = vals.astype(np.float16).view(np.uint16)
    got = np.array([oracle.f32_to_f16_bits(float(v)) for v in vals], dtype=np.uint16)
    assert np.array_equal(got, want)
    allbits = np.arange(0, 65536, 97, dtype=np.uint16)
    back = np.array([oracle.f16_bits_to_f32(int(b)) for b in allbits], dtype=np.float32)
    ref = allbits.view(np.float16).astype(np.float32)
    ok = (back == ref) | (np.isnan(back) & np.isnan(ref))
    assert ok.all()


# ----------------------------------------------------------------- rope ---

def rope_numpy(x, pos0, base, n_rot):
    """NEOX pair rotation with theta_i = p * s^i by repeated float32 multiplication."""
    x = x.astype(np.float32).copy()
    T, H, D = x.shape
    s = np.float32(np.power(np.float32(base), np.float32(-2.0 / n_rot), dtype=np.float32))
    half = n_rot // 2
    for t in range(T):
        th = np.float32(pos0 + t)
        for i in range(half):
            c, sn = np.float32(np.cos(np.float64(th))), np.float32(np.sin(np.float64(th)))
            x0, x1 = x[t, :, i].copy(), x[t, :, i + half].copy()
            x[t, :, i] = x0 * c - x1 * sn
            x[t, :, i + half] = x0 * sn + x1 * c
            th = np.float32(th * s)
    return x


def test_rope_text_matches_formula(oracle):
    rng = np.random.default_rng(2)
    x = rng.standard_normal((5, 3, 256)).astype(np.float32)
    got = oracle.rope_text(x, 170000, 1e7, 64)
    want = rope_numpy(x, 170000, 1e7, 64)
    assert np.abs(got - want).max() < 2e-5
    assert np.array_equal(got[..., 64:], x[..., 64:])  # dims >= n_rot untouched


def test_imrope_sections_reduce_to_text(oracle):
    # graph.rs:457-467 writes equal positions in all four streams -> sections irrelevant
    rng = np.random.default_rng(3)
    for D, n_rot, sec in ((256, 64, (11, 11, 10, 0)), (64, 16, (3, 3, 2, 0))):
        x = rng.standard_normal((4, 2, D)).astype(np.float32)
        pos = np.tile(np.arange(9, 13, dtype=np.int32), 4)
        a = oracle.rope_imrope(x, pos, sec, 1e7, n_rot)
        b = oracle.rope_text(x, 9, 1e7, n_rot)
        assert np.array_equal(a, b)


# ------------------------------------------------------------ attention ---

def attn_numpy(q, k, v, gate, q_pos0, scale):
    T, Hq, D = q.shape
    n_kv, Hkv, _ = k.shape
    G = Hq // Hkv
    out = np.zeros((T, Hq, D))
    lse = np.zeros((T, Hq))
    for t in range(T):
        lim = min(q_pos0 + t + 1, n_kv)
        for h in range(Hq):
            s = k[:lim, h // G, :].astype(np.float64) @ q[t, h].astype(np.float64) * scale
            m = s.max()
            p = np.exp(s - m)
            o = p @ v[:lim, h // G, :].astype(np.float64) / p.sum()
            if gate is not None:
                o = o / (1 + np.exp(-gate[t, h].astype(np.float64)))
            out[t, h] = o
            lse[t, h] = m + np.log(p.sum())
    return out, lse


def test_attn_oracle_vs_numpy(oracle):
    rng = np.random.default_rng(4)
    q = rng.standard_normal((3, 16, 256)).astype(np.float32)
    k = rng.standard_normal((77, 2, 256)).astype(np.float32)
    v = rng.standard_normal((77, 2, 256)).astype(np.float32)
    gate = rng.standard_normal((3, 16, 256)).astype(np.float32)
    for q_pos0 in (0, 40, 74, 200):
        got, lse = oracle.attn(q, k, v, gate, q_pos0=q_pos0, scale=1 / 16, want_lse=True)
        want, wl = attn_numpy(q, k, v, gate, q_pos0, 1 / 16)
        assert np.abs(got - want).max() < 1e-5
        assert np.abs(lse - wl).max() < 1e-4


def test_attn_oracle_gqa_block_mapping(oracle):
    # kv_head = h / (Hq / Hkv) (tests/attn_test.rs:306-312): heads 0-7 -> 0, 8-15 -> 1
    rng = np.random.default_rng(5)
    q = rng.standard_normal((1, 16, 256)).astype(np.float32)
    k = rng.standard_normal((10, 2, 256)).astype(np.float32)
    v = np.zeros((10, 2, 256), dtype=np.float32)
    v[:, 0, :] = 1.0
    v[:, 1, :] = 2.0
    out = oracle.attn(q, k, v, None, q_pos0=9)
    assert np.allclose(out[0, :8], 1.0) and np.allclose(out[0, 8:], 2.0)


# ------------------------------------------------------------------ gdn ---

def gdn_numpy(q, k, v, g, beta, S0):
    """float64 restatement of gdn.rs:9-24 with S[i][j] stored as S0[h][j][i]."""
    T, Hk, d = q.shape
    Hv = v.shape[1]
    S = S0.astype(np.float64).transpose(0, 2, 1).copy()  # [h][i][j]
    out = np.zeros((T, Hv, d))
    for t in range(T):
        for h in range(Hv):
            kk, qq = k[t, h % Hk].astype(np.float64), q[t, h % Hk].astype(np.float64)
            S[h] *= np.exp(np.float64(g[t, h]))
            delta = (v[t, h] - S[h].T @ kk) * beta[t, h]
            S[h] += np.outer(kk, delta)
            out[t, h] = S[h].T @ qq / np.sqrt(d)
    return out, S.transpose(0, 2, 1)


def gdn_inputs(rng, T, Hk, Hv, d, state_scale=0.02):
    q = rng.standard_normal((T, Hk, d)).astype(np.float32)
    k = rng.standard_normal((T, Hk, d)).astype(np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((T, Hv, d)).astype(np.float32)
    a_log = rng.uniform(0, 2.7, Hv).astype(np.float32)
    dt_bias = rng.standard_normal(Hv).astype(np.float32)
    g = (-np.exp(a_log) * np.log1p(np.exp(rng.standard_normal((T, Hv)) + dt_bias))).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal((T, Hv))))).astype(np.float32)
    S0 = (rng.standard_normal((Hv, d, d)) * state_scale).astype(np.float32)
    return q, k, v, g, beta, S0


def test_gdn_oracle_vs_numpy(oracle):
    rng = np.random.default_rng(6)
    q, k, v, g, beta, S0 = gdn_inputs(rng, 7, 2, 4, 16)
    out, snaps = oracle.gdn(q, k, v, g, beta, S0, n_snap=1)
    want, Sw = gdn_numpy(q, k, v, g, beta, S0)
    assert np.abs(out - want).max() < 1e-5
    assert np.abs(snaps[0] - Sw).max() < 1e-5


def test_gdn_fused_chunk_equivalence(oracle):
    # tests/gdn_test.rs:282-378: s_v 8, h_v 4, h_k 2, 32 tokens vs 16 + 16, <= 1e-5
    s_v, h_v, h_k, n, cs = 8, 4, 2, 32, 16
    q = ramp(s_v * h_k * n, -0.5, 0.5).reshape(n, h_k, s_v)
    k = ramp(s_v * h_k * n, 0.5, -0.5).reshape(n, h_k, s_v)
    v = ramp(s_v * h_v * n, -1.0, 1.0).reshape(n, h_v, s_v)
    g = ramp(h_v * n, -0.5, 0.0).reshape(n, h_v)
    b = ramp(h_v * n, 0.1, 0.9).reshape(n, h_v)
    s0 = np.zeros((h_v, s_v, s_v), dtype=np.float32)
    full, _ = oracle.gdn(q, k, v, g, b, s0)
    _, sa = oracle.gdn(q[:cs], k[:cs], v[:cs], g[:cs], b[:cs], s0)
    ob, _ = oracle.gdn(q[cs:], k[cs:], v[cs:], g[cs:], b[cs:], sa[0])
    rel = np.abs(ob - full[cs:]) / np.maximum(np.abs(full[cs:]), 1.0)
    assert rel.max() <= 1e-5


def test_gdn_rollback_snapshots_match_shorter_runs(oracle):
    # tests/gdn_prod_dim_test.rs:245-292 at production dims: slot s == state after N - s
    rng = np.random.default_rng(7)
    N = 4
    q, k, v, g, beta, S0 = gdn_inputs(rng, N, 16, 32, 128)
    _, snaps = oracle.gdn(q, k, v, g, beta, S0, n_snap=N)
    for s in range(N):
        n = N - s
        _, ref = oracle.gdn(q[:n], k[:n], v[:n], g[:n], beta[:n], S0, n_snap=1)
        scale = np.abs(ref[0]).max()
        assert np.abs(snaps[s] - ref[0]).max() <= 1e-5 * scale


def test_gdn_5_plus_1_equals_6(oracle):
    # tests/gdn_prod_dim_test.rs:294-326 (op level): <= 1e-4 * scale
    rng = np.random.default_rng(8)
    q, k, v, g, beta, S0 = gdn_inputs(rng, 6, 16, 32, 128)
    full, _ = oracle.gdn(q, k, v, g, beta, S0)
    _, s5 = oracle.gdn(q[:5], k[:5], v[:5], g[:5], beta[:5], S0)
    o6, _ = oracle.gdn(q[5:], k[5:], v[5:], g[5:], beta[5:], s5[0])
    scale = np.abs(full[5]).max()
    assert np.abs(o6[0] - full[5]).max() <= 1e-4 * scale


def test_l2norm_is_unit(oracle):
    rng = np.random.default_rng(9)
    x = rng.standard_normal((10, 128)).astype(np.float32) * 3
    y = oracle.l2norm(x, 1e-6)
    assert np.allclose(np.linalg.norm(y, axis=-1), 1.0, atol=1e-5)


# ------------------------------------------------------- gdn front end ---

class KvRng:
    """The reference's test generator (tests/kernel_verify.rs:228-245), restated so
    that the front-end checks below run on the very inputs of its kernel tests."""

    def __init__(self, seed):
        self.s = (seed ^ 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF

    def next_u32(self):
        self.s = (self.s * 6364136223846793005 + 1442695040888963407) & 0xFFFFFFFFFFFFFFFF
        return self.s >> 33

    def f32(self, lo, hi, n):
        out = np.empty(n, dtype=np.float32)
        for i in range(n):
            u = np.float32((self.next_u32() >> 8) / float(1 << 24))
            out[i] = np.float32(lo) + np.float32(hi - lo) * u
        return out


def test_ssm_conv_reference_case(oracle):
    # tests/kernel_verify.rs:827-867: d_conv 4, n_t 3, d_inner 128, Rng(8) in [-1, 1)
    K, T, C = 4, 3, 128
    ncs = K - 1 + T
    rng = KvRng(8)
    sx = rng.f32(-1.0, 1.0, ncs * C).reshape(C, ncs)
    c = rng.f32(-1.0, 1.0, K * C).reshape(C, K)
    want = np.zeros((T, C), dtype=np.float32)
    for t in range(T):
        for i in range(C):
            s = np.float32(0.0)
            for k in range(K):
                s = np.float32(s + np.float32(sx[i, t + k] * c[i, k]))
            want[t, i] = s
    got = oracle.ssm_conv(sx, c)
    assert np.array_equal(got, want)


def test_silu_reference_case(oracle):
    # tests/kernel_verify.rs:981-989: Rng(11) in [-4, 4), silu = x / (1 + exp(-x))
    x = KvRng(11).f32(-4.0, 4.0, 32)
    sx = np.zeros((32, 4), dtype=np.float32)
    sx[:, 3] = x  # a conv with the single tap w = 1 is the identity: silu(conv) = silu(x)
    w = np.zeros((32, 4), dtype=np.float32)
    w[:, 3] = 1.0
    out, _ = oracle.gdn_conv(x[None, :], w, np.zeros((1, 32, 3), np.float32))
    want = x / (1.0 + np.exp(-x.astype(np.float64)))
    assert np.abs(out[0] - want).max() <= 1e-6 * np.abs(want).max()


def _conv_case(T, C=256, K=4, n_planes=3, seed=0):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, C)).astype(np.float32)
    w = (rng.standard_normal((C, K)) * 0.5).astype(np.float32)
    st = rng.standard_normal((n_planes, C, K - 1)).astype(np.float32)
    return x, w, st


def test_gdn_conv_vs_numpy(oracle):
    # conv over concat(history, x), silu, per-head L2 norm of the q/k channels
    T, C, K, d, n_qk = 5, 256, 4, 64, 128
    x, w, st = _conv_case(T, C, K)
    out, new = oracle.gdn_conv(x, w, st, sel=1, n_snap=1, n_qk=n_qk, d=d)
    sx = np.concatenate([st[1].astype(np.float64), x.T.astype(np.float64)], axis=1)  # [C][K-1+T]
    y = np.stack([(sx[:, t:t + K] * w).sum(axis=1) for t in range(T)])
    y = y / (1.0 + np.exp(-y))
    for h in range(n_qk // d):
        blk = y[:, h * d:(h + 1) * d]
        y[:, h * d:(h + 1) * d] = blk / np.sqrt((blk * blk).sum(axis=1, keepdims=True) + 1e-6)
    assert np.abs(out - y).max() <= 1e-5 * np.abs(y).max()
    # n_snap 1: plane 0 <- the last K-1 conv inputs, other planes untouched
    assert np.array_equal(new[0], sx[:, T:T + K - 1].astype(np.float32))
    assert np.array_equal(new[1:], st[1:])


def test_gdn_conv_chunk_carry_and_rollback_slots(oracle):
    # T tokens at once == T one-token steps (the conv tail carries the history), and
    # slot s of an n_snap run == the plane-0 tail of a run over the first T - s tokens
    # (graph.rs:913-961; slots with s > T keep the input history)
    T, C, K = 6, 128, 4
    x, w, st = _conv_case(T, C, K, n_planes=4, seed=3)
    out_all, new_all = oracle.gdn_conv(x, w, st, sel=0, n_snap=4)
    cur = st.copy()
    outs = []
    for t in range(T):
        o, cur = oracle.gdn_conv(x[t:t + 1], w, cur, sel=0, n_snap=1)
        outs.append(o[0])
    assert np.array_equal(np.stack(outs), out_all)
    assert np.array_equal(cur[0], new_all[0])
    for s in range(4):
        _, short = oracle.gdn_conv(x[:T - s], w, st, sel=0, n_snap=1)
        assert np.array_equal(new_all[s], short[0]), s
    _, tiny = oracle.gdn_conv(x[:2], w, st, sel=0, n_snap=4)
    assert np.array_equal(tiny[3], st[0])  # s = 3 > T = 2: the input history


def test_rms_norm_and_norm_gated_vs_numpy(oracle):
    rng = np.random.default_rng(5)
    x = rng.standard_normal((3, 4, 128)).astype(np.float32)
    z = rng.standard_normal((3, 4, 128)).astype(np.float32)
    w1 = rng.standard_normal(128).astype(np.float32)
    w2 = rng.standard_normal((4, 128)).astype(np.float32)
    xd = x.astype(np.float64)
    r = xd / np.sqrt((xd * xd).mean(axis=-1, keepdims=True) + 1e-6)
    silu = z / (1.0 + np.exp(-z.astype(np.float64)))
    for w, wb in ((w1, w1[None, None]), (w2, w2[None])):
        got = oracle.rms_norm(x, 1e-6, w=w, z=z)
        want = r * wb * silu
        assert np.abs(got - want).max() <= 1e-5 * np.abs(want).max()
    got = oracle.rms_norm(x, 1e-6)
    assert np.abs(got - r).max() <= 1e-5 * np.abs(r).max()


def test_cpu_baseline_matches_checker(oracle):
    """The timed CPU baseline (ggml-cpu's algorithm: q8_0 Q, f32 online softmax, per-key
    V dequant) computes the same attention and GDN step as the double-precision checker,
    within the error of Q's q8_0 rounding."""
    rng = np.random.default_rng(5)
    n_kv, T = 700, 3
    k = rng.standard_normal((n_kv, 512)).astype(np.float32)
    v = rng.standard_normal((n_kv, 512)).astype(np.float32)
    kq, vq = oracle.q4_0_quantize(k), oracle.q4_0_quantize(v)
    kd = oracle.q4_0_dequantize(kq, 512).reshape(n_kv, 2, 256)
    vd = oracle.q4_0_dequantize(vq, 512).reshape(n_kv, 2, 256)
    q = rng.standard_normal((T, 16, 256)).astype(np.float32)
    gate = rng.standard_normal((T, 16, 256)).astype(np.float32)
    want, wlse = oracle.attn(q, kd, vd, gate, q_pos0=n_kv - T, scale=1 / 16, want_lse=True)
    got, glse = oracle.cpu_fa_q4_0(q, kq, vq, gate, q_pos0=n_kv - T, scale=1 / 16, want_lse=True)
    assert np.abs(got - want).max() <= 2e-2 * np.abs(want).max()
    assert np.abs(glse - wlse).max() < 5e-3
    S = (rng.standard_normal((32, 128, 128)) * 0.02).astype(np.float32)
    qg = oracle.l2norm(rng.standard_normal((4, 16, 128)).astype(np.float32))
    kg = oracle.l2norm(rng.standard_normal((4, 16, 128)).astype(np.float32))
    vg = rng.standard_normal((4, 32, 128)).astype(np.float32)
    g = -rng.uniform(0.01, 1.0, (4, 32)).astype(np.float32)
    b = rng.uniform(0.1, 0.9, (4, 32)).astype(np.float32)
    want_o, snaps = oracle.gdn(qg, kg, vg, g, b, S, n_snap=1)
    st = S.copy()
    got_o = oracle.cpu_gdn_f32(qg, kg, vg, g, b, st)
    assert np.abs(got_o - want_o).max() <= 1e-4 * np.abs(want_o).max()
    assert np.abs(st - snaps[0]).max() <= 1e-4 * np.abs(snaps[0]).max()


# ---------------------------------------------------------- projections ---
PROJ_GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "proj_golden.npz")
PROJ_TYPES = (("q4_k", 12), ("q6_k", 14), ("q8_0", 8))


@pytest.mark.parametrize("name,wtype", PROJ_TYPES)
def test_proj_dequant_bit_exact_vs_gguf_golden(oracle, name, wtype):
    """q4_K / q6_K / q8_0 rows dequantised exactly as gguf-py's restatement of ggml's
    block formats (the weights of ggml_mul_mat in attn.rs:127-129 / gdn.rs:264-276)."""
    d = np.load(PROJ_GOLDEN)
    n_in = d[f"{name}_x"].shape[1]
    got = oracle.dequant_rows(d[f"{name}_w"], wtype, n_in)
    assert np.array_equal(got.view(np.uint32), d[f"{name}_deq"].view(np.uint32))


@pytest.mark.parametrize("name,wtype", PROJ_TYPES)
def test_proj_mul_mat_vs_golden(oracle, name, wtype):
    d = np.load(PROJ_GOLDEN)
    n_in = d[f"{name}_x"].shape[1]
    y = oracle.mul_mat(d[f"{name}_w"], wtype, n_in, d[f"{name}_x"])
    ref = d[f"{name}_y"]
    assert np.abs(y - ref).max() <= 1e-6 * np.abs(ref).max()


def test_proj_row_bytes_and_float_types(oracle):
    assert oracle.row_bytes(12, 2048) == 8 * 144
    assert oracle.row_bytes(14, 2048) == 8 * 210
    assert oracle.row_bytes(8, 2048) == 64 * 34
    assert oracle.row_bytes(12, 100) == 0 and oracle.row_bytes(2, 256) == 0
    rng = np.random.default_rng(5)
    w = rng.standard_normal((5, 256)).astype(np.float32)
    x = rng.standard_normal((2, 256)).astype(np.float32)
    for wtype, raw in ((0, w), (1, w.astype(np.float16)), (30, None)):
        if wtype == 30:  # bf16: the high halves of the f32 words
            raw = (w.view(np.uint32) >> 16).astype(np.uint16)
            deq = (raw.astype(np.uint32) << 16).view(np.float32)
        else:
            deq = raw.astype(np.float32)
        rows = np.ascontiguousarray(raw).view(np.uint8).reshape(5, -1)
        assert np.array_equal(oracle.dequant_rows(rows, wtype, 256), deq)
        y = oracle.mul_mat(rows, wtype, 256, x)
        assert np.allclose(y, x.astype(np.float64) @ deq.astype(np.float64).T, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("name,wtype", PROJ_TYPES)
def test_cpu_baseline_mul_mat_matches_checker(oracle, name, wtype):
    """The timed ggml-cpu restatement (x quantised to q8_K / q8_0) agrees with the exact
    checker to the accuracy of its 8-bit activations."""
    d = np.load(PROJ_GOLDEN)
    n_in = d[f"{name}_x"].shape[1]
    y = oracle.cpu_mul_mat(d[f"{name}_w"], wtype, n_in, d[f"{name}_x"])
    ref = d[f"{name}_y"]
    assert np.abs(y - ref).max() <= 2e-2 * np.abs(ref).max()
