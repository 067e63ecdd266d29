"""GPU parity of the chunked gated-delta-net prefill (sqmix_gdn_prefill, chunk 64)
against the sequential CPU oracle, and against the recurrent kernel.

Bar: outputs and state planes within 1e-3 relative (max|gpu - ref| / max|ref|).
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

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


def gdn_case(rng, n_seqs, T, Hk=16, Hv=32, d=128, state_scale=0.02, n_planes=1, normalise=True):
    """Config-1 distributions: q, k N(0,1) (unit-normalised unless the kernel does it),
    v N(0,1), beta = sigmoid(N(0,1)), g = -exp(A_log) softplus(N(0,1) + dt_bias)."""
    q = rng.standard_normal((n_seqs, T, Hk, d)).astype(np.float32)
    k = rng.standard_normal((n_seqs, T, Hk, d)).astype(np.float32)
    if normalise:
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


def test_gdn_prefill_config1_bf16_l2norm(sq, oracle):
    """Config 1: one decode token, then a 512-token prefill (chunk 64), bf16 q/k/v with
    the per-head L2 normalisation fused (gdn.rs:440-441)."""
    rng = np.random.default_rng(71)
    q, k, v, g, beta, S = gdn_case(rng, 1, 513, normalise=False)
    tq, tk, tv = (torch.from_numpy(x).to(torch.bfloat16) for x in (q, k, v))
    qf, kf, vf = (x.float().numpy() for x in (tq, tk, tv))
    st = torch.from_numpy(S).cuda()
    gc, bc = torch.from_numpy(g).cuda(), torch.from_numpy(beta).cuda()
    o1 = sq.gated_delta_net(tq[:, :1].cuda(), tk[:, :1].cuda(), tv[:, :1].cuda(), gc[:, :1].contiguous(),
                            bc[:, :1].contiguous(), st, l2_eps=1e-6)
    o2 = sq.gated_delta_net(tq[:, 1:].cuda(), tk[:, 1:].cuda(), tv[:, 1:].cuda(), gc[:, 1:].contiguous(),
                            bc[:, 1:].contiguous(), st, l2_eps=1e-6, chunked=True)
    torch.cuda.synchronize()
    qn = oracle.l2norm(qf[0], 1e-6)
    kn = oracle.l2norm(kf[0], 1e-6)
    want, snaps = oracle.gdn(qn, kn, vf[0], g[0], beta[0], S[0, 0])
    got = np.concatenate([o1.cpu().numpy()[0], o2.cpu().numpy()[0]])
    assert rel_err(got, want) <= GDN_TOL
    assert rel_err(st.cpu().numpy()[0, 0], snaps[0]) <= GDN_TOL


@pytest.mark.parametrize("T", [1, 63, 64, 65, 100, 130, 200])
def test_gdn_prefill_ragged(sq, oracle, T):
    rng = np.random.default_rng(700 + T)
    q, k, v, g, beta, S = gdn_case(rng, 1, T, Hk=4, Hv=8)
    st = torch.from_numpy(S).cuda()
    out = sq.gated_delta_net(*(torch.from_numpy(x).cuda() for x in (q, k, v, g, beta)), st, chunked=True)
    torch.cuda.synchronize()
    want, snaps = oracle.gdn(q[0], k[0], v[0], g[0], beta[0], S[0, 0])
    assert rel_err(out.cpu().numpy()[0], want) <= GDN_TOL
    assert rel_err(st.cpu().numpy()[0, 0], snaps[0]) <= GDN_TOL


@pytest.mark.parametrize("n_snap", [2, 3])
def test_gdn_prefill_snapshots_sel_batch(sq, oracle, n_snap):
    """MTP snapshots after a prefill: slot s = state after T - s tokens, input plane sel."""
    rng = np.random.default_rng(80 + n_snap)
    n_seqs, T, n_planes = 2, 150, 3
    q, k, v, g, beta, S = gdn_case(rng, n_seqs, T, Hk=4, Hv=8, n_planes=n_planes)
    sel = np.array([2, 1], dtype=np.int32)
    st = torch.from_numpy(S).cuda()
    out = sq.gated_delta_net(*(torch.from_numpy(x).cuda() for x in (q, k, v, g, beta)), st, n_planes=n_planes,
                             sel=torch.from_numpy(sel).cuda(), n_snap=n_snap, chunked=True)
    torch.cuda.synchronize()
    st_np, out_np = st.cpu().numpy(), out.cpu().numpy()
    for s in range(n_seqs):
        want, snaps = oracle.gdn(q[s], k[s], v[s], g[s], beta[s], S[s, sel[s]], n_snap=n_snap)
        assert rel_err(out_np[s], want) <= GDN_TOL
        for slot in range(n_snap):
            assert rel_err(st_np[s, slot], snaps[slot]) <= GDN_TOL


def test_gdn_prefill_matches_recurrent(sq):
    rng = np.random.default_rng(90)
    q, k, v, g, beta, S = gdn_case(rng, 1, 300)
    args = [torch.from_numpy(x).cuda() for x in (q, k, v, g, beta)]
    st_a, st_b = torch.from_numpy(S).cuda(), torch.from_numpy(S).cuda()
    oa = sq.gated_delta_net(*args, st_a, chunked=True)
    ob = sq.gated_delta_net(*args, st_b, chunked=False)
    torch.cuda.synchronize()
    assert rel_err(oa.cpu().numpy(), ob.cpu().numpy()) <= GDN_TOL
    assert rel_err(st_a.cpu().numpy(), st_b.cpu().numpy()) <= GDN_TOL
