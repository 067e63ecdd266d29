"""GPU parity of the tensor-core prefill attention (sqmix_fa_prefill) against the CPU
oracle: causal attention of T query tokens over a q4_0 prefix plus the step's own rows,
GQA 16/2, head_dim 256, partial RoPE 64 / 1e7 on Q and K, sigmoid gate.

Bar: max|gpu - ref| <= 2e-3 * max|ref| against the fp32 oracle on the same dequantised
cache and the same (dtype-rounded) Q; LSE within 1e-3 absolute.
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


def build_case(sq, oracle, P, T, seed, q_dtype=torch.bfloat16):
    rng = np.random.default_rng(seed)
    n_kv = P + T
    cap = max(256, (n_kv + 255) // 256 * 256)
    k = rng.standard_normal((n_kv, 2, 256)).astype(np.float32)
    v = rng.standard_normal((n_kv, 2, 256)).astype(np.float32)
    kc, vc = sq.new_kv_cache(cap), sq.new_kv_cache(cap)
    rows = torch.arange(n_kv, device="cuda")
    sq.set_rows_q4_0(torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), rows, kc, vc, cap, rope_n_rot=64,
                     rope_freq_base=1e7)
    kd = oracle.q4_0_dequantize(oracle.q4_0_quantize(oracle.rope_text(k, 0, 1e7, 64).reshape(n_kv, 512)),
                                512).reshape(n_kv, 2, 256)
    vd = oracle.q4_0_dequantize(oracle.q4_0_quantize(v.reshape(n_kv, 512)), 512).reshape(n_kv, 2, 256)
    q_t = torch.from_numpy(rng.standard_normal((T, 16, 256)).astype(np.float32)).to(q_dtype).cuda()
    gate = rng.standard_normal((T, 16, 256)).astype(np.float32)
    q_used = q_t.float().cpu().numpy()
    want, wlse = oracle.attn(oracle.rope_text(q_used, P, 1e7, 64), kd, vd, gate, q_pos0=P, scale=1 / 16,
                             want_lse=True)
    return dict(kc=kc, vc=vc, cap=cap, n_kv=n_kv, q=q_t, gate=torch.from_numpy(gate).cuda(), want=want, wlse=wlse)


def run_prefill(sq, c, P, n_ctas=0, workspace=None):
    d_nkv = torch.tensor([c["n_kv"]], dtype=torch.int64, device="cuda")
    d_pos = torch.tensor([P], dtype=torch.int64, device="cuda")
    T = c["q"].shape[0]
    lse = torch.empty((T, 16), dtype=torch.float32, device="cuda")
    out = sq.flash_attn_prefill(c["q"], c["kc"], c["vc"], c["cap"], d_nkv, d_pos, gate=c["gate"], rope_n_rot=64,
                                rope_freq_base=1e7, lse=lse, n_ctas=n_ctas, workspace=workspace)
    torch.cuda.synchronize()
    return out.cpu().numpy(), lse.cpu().numpy()


@pytest.mark.parametrize("P,T", [(0, 1), (0, 16), (5, 17), (200, 37), (1000, 64), (64, 2), (2048, 300)])
def test_prefill_matches_oracle(sq, oracle, P, T):
    c = build_case(sq, oracle, P, T, seed=1000 + 7 * P + T)
    out, lse = run_prefill(sq, c, P)
    assert rel_err(out, c["want"]) <= ATTN_TOL
    assert np.abs(lse - c["wlse"]).max() < 1e-3


@pytest.mark.parametrize("n_ctas", [1, 3, 8, 148])
def test_prefill_item_queue(sq, oracle, n_ctas):
    """Few CTA pairs take many items each (item ring, Q reload, O hand-over between items;
    segments spanning M-tiles)."""
    P, T = 1500, 96
    c = build_case(sq, oracle, P, T, seed=77 + n_ctas)
    out, lse = run_prefill(sq, c, P, n_ctas=n_ctas)
    assert rel_err(out, c["want"]) <= ATTN_TOL
    assert np.abs(lse - c["wlse"]).max() < 1e-3


def test_prefill_pp512_on_prefix(sq, oracle):
    """Config-2 shape at a reduced prefix: 512 new tokens after 3000 cached ones."""
    P, T = 3000, 512
    c = build_case(sq, oracle, P, T, seed=512)
    ws = sq.new_fa_prefill_workspace(T)
    for _ in range(2):  # the workspace is reused without re-initialisation
        out, _ = run_prefill(sq, c, P, workspace=ws)
        assert rel_err(out, c["want"]) <= ATTN_TOL
    sq.fa_status(ws)


@pytest.mark.parametrize("layout", ["f16", "qg_view_bf16"])
def test_prefill_q_dtype_and_strided_q(sq, oracle, layout):
    """f16 Q, and Q read in place from the QG projection (per head [q(256), gate(256)],
    attn.rs:131-175: head stride 512) -- the prep kernel's other dtype path and strides."""
    P, T = 300, 40
    dt = torch.float16 if layout == "f16" else torch.bfloat16
    c = build_case(sq, oracle, P, T, seed=41 + len(layout), q_dtype=dt)
    if layout == "qg_view_bf16":
        qg = torch.empty((T, 16, 512), dtype=dt, device="cuda")
        qg[:, :, :256] = c["q"]
        qg[:, :, 256:] = 7.0  # never read
        c["q"] = qg[:, :, :256]
        assert c["q"].stride(1) == 512
    out, lse = run_prefill(sq, c, P)
    assert rel_err(out, c["want"]) <= ATTN_TOL
    assert np.abs(lse - c["wlse"]).max() < 1e-3


def test_prefill_agrees_with_decode(sq, oracle):
    P, T = 777, 2
    c = build_case(sq, oracle, P, T, seed=9, q_dtype=torch.float32)
    out, _ = run_prefill(sq, c, P)
    d_nkv = torch.tensor([c["n_kv"]], dtype=torch.int64, device="cuda")
    d_pos = torch.tensor([P], dtype=torch.int64, device="cuda")
    dec = sq.flash_attn_ext(c["q"], c["kc"], c["vc"], c["cap"], d_nkv, d_pos, gate=c["gate"], rope_n_rot=64,
                            rope_freq_base=1e7).cpu().numpy()
    assert rel_err(out, dec) <= ATTN_TOL
    assert rel_err(out, c["want"]) <= ATTN_TOL
