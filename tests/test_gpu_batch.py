"""GPU parity of the sequence-batched decode (sqmix_fa_decode_batch): many sequences,
each with its own q4_0 caches and length, one launch pair; against the CPU oracle per
sequence and against the single-sequence entry point.

Bar: attention max|gpu - ref| <= 2e-3 * max|ref| (as for the single-sequence decode);
the fused append is bit-exact with quantize_row_q4_0.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ATTN_TOL = 2e-3


@pytest.fixture(scope="module")
def sq():
    import sqmix

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return sqmix


def rel_err(got, want):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    return np.abs(got - want).max() / max(np.abs(want).max(), 1e-30)


def build(sq, oracle, lens, seed, fused):
    """Per sequence: K/V rows 0..n-1 (n = len, or len - 1 with the last row appended by the
    batch launch), RoPE 64 / 1e7 on K; returns device arrays and oracle references."""
    rng = np.random.default_rng(seed)
    n_seqs = len(lens)
    caches, refs = [], []
    q = rng.standard_normal((n_seqs, 16, 256)).astype(np.float32)
    gate = rng.standard_normal((n_seqs, 16, 256)).astype(np.float32)
    k_new = rng.standard_normal((n_seqs, 2, 256)).astype(np.float32)
    v_new = rng.standard_normal((n_seqs, 2, 256)).astype(np.float32)
    for s, n in enumerate(lens):
        cap = max(256, (n + 255) // 256 * 256)
        k = rng.standard_normal((n, 2, 256)).astype(np.float32)
        v = rng.standard_normal((n, 2, 256)).astype(np.float32)
        if fused:
            k[n - 1], v[n - 1] = k_new[s], v_new[s]
        kc, vc = sq.new_kv_cache(cap), sq.new_kv_cache(cap)
        n_pre = n - 1 if fused else n
        if n_pre > 0:
            sq.set_rows_q4_0(torch.from_numpy(k[:n_pre]).cuda(), torch.from_numpy(v[:n_pre]).cuda(),
                             torch.arange(n_pre, device="cuda"), kc, vc, cap, rope_n_rot=64, rope_freq_base=1e7)
        kq = oracle.q4_0_quantize(oracle.rope_text(k, 0, 1e7, 64).reshape(n, 512))
        vq = oracle.q4_0_quantize(v.reshape(n, 512))
        kd = oracle.q4_0_dequantize(kq, 512).reshape(n, 2, 256)
        vd = oracle.q4_0_dequantize(vq, 512).reshape(n, 2, 256)
        qr = oracle.rope_text(q[s:s + 1], n - 1, 1e7, 64)
        refs.append((oracle.attn(qr, kd, vd, gate[s:s + 1], q_pos0=n - 1, scale=1 / 16)[0], kq, vq))
        caches.append((kc, vc, cap))
    dev = torch.device("cuda")
    arr = lambda xs: torch.tensor(xs, dtype=torch.int64, device=dev)
    d = dict(
        q=torch.from_numpy(q).cuda(), gate=torch.from_numpy(gate).cuda(),
        kp=arr([c[0].data_ptr() for c in caches]), vp=arr([c[1].data_ptr() for c in caches]),
        caps=arr([c[2] for c in caches]), n_kv=arr(list(lens)), q_pos0=arr([n - 1 for n in lens]),
        k_new=torch.from_numpy(k_new).cuda(), v_new=torch.from_numpy(v_new).cuda())
    return d, caches, refs


@pytest.mark.parametrize("splits", [0, 1, 3, 16, 17])  # <= 16 splits: the per-thread merge
def test_batch_decode_matches_oracle(sq, oracle, splits):
    lens = [100, 1000, 17, 3000, 256, 1]
    d, caches, refs = build(sq, oracle, lens, seed=31 + splits, fused=False)
    out = sq.flash_attn_decode_batch(d["q"], d["kp"], d["vp"], d["caps"], d["n_kv"], d["q_pos0"], gate=d["gate"],
                                     rope_n_rot=64, rope_freq_base=1e7, splits_per_seq=splits)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for s in range(len(lens)):
        assert rel_err(got[s], refs[s][0]) <= ATTN_TOL, s


def test_batch_decode_fused_append_and_single_path(sq, oracle):
    lens = [40, 700, 2049, 16]
    d, caches, refs = build(sq, oracle, lens, seed=77, fused=True)
    ws = torch.zeros(sq.fa_batch_workspace_bytes(len(lens), 0), dtype=torch.uint8, device="cuda")
    out = sq.flash_attn_decode_batch(d["q"], d["kp"], d["vp"], d["caps"], d["n_kv"], d["q_pos0"], gate=d["gate"],
                                     rope_n_rot=64, rope_freq_base=1e7, workspace=ws, k_new=d["k_new"],
                                     v_new=d["v_new"])
    torch.cuda.synchronize()
    sq.fa_status(ws)
    got = out.cpu().numpy()
    for s, (kc, vc, cap) in enumerate(caches):
        assert rel_err(got[s], refs[s][0]) <= ATTN_TOL, s
        n = lens[s]
        # the appended row is bit-exact with quantize_row_q4_0 of the rotated K / raw V
        krow = sq.kv_convert_rows(kc, cap, "k", n - 1, 1).cpu().numpy()
        vrow = sq.kv_convert_rows(vc, cap, "v", n - 1, 1).cpu().numpy()
        assert np.array_equal(krow[0], refs[s][1][n - 1])
        assert np.array_equal(vrow[0], refs[s][2][n - 1])
        # the single-sequence entry point agrees on the same cache
        single = sq.flash_attn_ext(d["q"][s:s + 1], kc, vc, cap, d["n_kv"][s:s + 1], d["q_pos0"][s:s + 1],
                                   gate=d["gate"][s:s + 1], rope_n_rot=64, rope_freq_base=1e7)
        torch.cuda.synchronize()
        assert rel_err(got[s], single.cpu().numpy()[0]) <= ATTN_TOL
