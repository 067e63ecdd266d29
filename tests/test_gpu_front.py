"""GPU parity of the GDN front end (sqmix_gdn_conv: short conv + SiLU + q/k L2 norm with
the conv-history planes) and the per-head norms (sqmix_head_norm: Q/K RMS norm of the
attention layers, norm_gated of the GDN output), against the CPU oracle.

Bars: conv/norm outputs within 1e-4 relative (the GDN bar is 1e-3); history planes
are copies and must match exactly.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-4
GDN_TOL = 1e-3
C, K, D, NQK = 8192, 4, 128, 4096  # config 1: 2 * 16 * 128 q/k channels + 32 * 128 v channels


@pytest.fixture(scope="module")
def sq():
    import sqmix

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return sqmix


def rel_err(got, want):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    return np.abs(got - want).max() / max(np.abs(want).max(), 1e-30)


def conv_inputs(rng, n_seqs, T, n_planes, bf16=False):
    x = rng.standard_normal((n_seqs, T, C)).astype(np.float32)
    if bf16:  # round through bf16 so that the oracle sees the values the device reads
        x = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    w = (rng.standard_normal((C, K)) * 0.5).astype(np.float32)
    st = rng.standard_normal((n_seqs, n_planes, C, K - 1)).astype(np.float32)
    return x, w, st


@pytest.mark.parametrize("T", [1, 2, 17, 512])
@pytest.mark.parametrize("x_bf16", [False, True])
def test_gdn_conv_config1(sq, oracle, T, x_bf16):
    rng = np.random.default_rng(T * 7 + x_bf16)
    n_planes = 3
    x, w, st = conv_inputs(rng, 1, T, n_planes, bf16=x_bf16)
    xd = torch.from_numpy(x).cuda()
    if x_bf16:
        xd = xd.to(torch.bfloat16)
    sd = torch.from_numpy(st).cuda()
    sel = torch.tensor([1], dtype=torch.int32, device="cuda")
    n_snap = min(3, n_planes)
    out = sq.gdn_conv(xd, torch.from_numpy(w).cuda(), sd, n_planes=n_planes, sel=sel, n_snap=n_snap,
                      n_qk_channels=NQK, l2_eps=1e-6)
    torch.cuda.synchronize()
    want, want_st = oracle.gdn_conv(x[0], w, st[0], sel=1, n_snap=n_snap, n_qk=NQK, d=D, eps=1e-6)
    assert rel_err(out.cpu().numpy()[0], want) <= TOL
    assert np.array_equal(sd.cpu().numpy()[0], want_st)


def test_gdn_conv_batch_sel_and_chunk_carry(sq, oracle):
    # three sequences with their own history planes and selectors; then T tokens in
    # one call == T one-token calls (the history tail carries the window)
    rng = np.random.default_rng(5)
    n_seqs, T, n_planes = 3, 40, 2
    x, w, st = conv_inputs(rng, n_seqs, T, n_planes)
    wd = torch.from_numpy(w).cuda()
    sd = torch.from_numpy(st).cuda()
    sel = torch.tensor([1, 0, 1], dtype=torch.int32, device="cuda")
    out = sq.gdn_conv(torch.from_numpy(x).cuda(), wd, sd, n_planes=n_planes, sel=sel, n_snap=2,
                      n_qk_channels=NQK, l2_eps=1e-6)
    torch.cuda.synchronize()
    got, got_st = out.cpu().numpy(), sd.cpu().numpy()
    for s, sl in enumerate([1, 0, 1]):
        want, want_st = oracle.gdn_conv(x[s], w, st[s], sel=sl, n_snap=2, n_qk=NQK, d=D, eps=1e-6)
        assert rel_err(got[s], want) <= TOL, s
        assert np.array_equal(got_st[s], want_st), s
    # one token at a time from the same starting planes (plane 0 read and rewritten)
    sd1 = torch.from_numpy(st[:1].copy()).cuda()
    steps = []
    for t in range(T):
        o = sq.gdn_conv(torch.from_numpy(x[:1, t:t + 1].copy()).cuda(), wd, sd1, n_planes=n_planes,
                        n_qk_channels=NQK, l2_eps=1e-6)
        steps.append(o.cpu().numpy()[0, 0])
    full = sq.gdn_conv(torch.from_numpy(x[:1]).cuda(), wd, torch.from_numpy(st[:1].copy()).cuda(),
                       n_planes=n_planes, n_qk_channels=NQK, l2_eps=1e-6)
    torch.cuda.synchronize()
    assert np.array_equal(np.stack(steps), full.cpu().numpy()[0])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_head_norm_q_k_of_attention(sq, oracle, dtype):
    # Q read in place from the QG projection (per head [q(256), gate(256)], attn.rs:131-175)
    rng = np.random.default_rng(11)
    T = 5
    qg = rng.standard_normal((T, 16, 512)).astype(np.float32)
    kk = rng.standard_normal((T, 2, 256)).astype(np.float32)
    wq = rng.standard_normal(256).astype(np.float32)
    wk = rng.standard_normal(256).astype(np.float32)
    qgd = torch.from_numpy(qg).cuda().to(dtype)
    kd = torch.from_numpy(kk).cuda().to(dtype)
    qn = sq.head_norm(qgd[:, :, :256], 1e-6, weight=torch.from_numpy(wq).cuda())
    kn = sq.head_norm(kd, 1e-6, weight=torch.from_numpy(wk).cuda())
    torch.cuda.synchronize()
    q_in = qgd[:, :, :256].float().cpu().numpy()
    k_in = kd.float().cpu().numpy()
    assert rel_err(qn.cpu().numpy(), oracle.rms_norm(q_in, 1e-6, w=wq)) <= TOL
    assert rel_err(kn.cpu().numpy(), oracle.rms_norm(k_in, 1e-6, w=wk)) <= TOL


@pytest.mark.parametrize("per_head_weight", [False, True])
def test_norm_gated_and_in_place(sq, oracle, per_head_weight):
    rng = np.random.default_rng(12 + per_head_weight)
    T = 9
    o = rng.standard_normal((T, 32, 128)).astype(np.float32)
    z = rng.standard_normal((T, 32 * 128)).astype(np.float32)
    w = rng.standard_normal((32, 128) if per_head_weight else 128).astype(np.float32)
    zd = torch.from_numpy(z).cuda().to(torch.bfloat16)
    z_used = zd.float().cpu().numpy().reshape(T, 32, 128)
    od = torch.from_numpy(o).cuda()
    got = sq.head_norm(od, 1e-6, weight=torch.from_numpy(w).cuda(), z=zd.view(T, 32, 128), out=od)  # in place
    torch.cuda.synchronize()
    assert got.data_ptr() == od.data_ptr()
    want = oracle.rms_norm(o, 1e-6, w=w, z=z_used)
    assert rel_err(od.cpu().numpy(), want) <= TOL


def test_gdn_mixer_chain_conv_recurrence_norm_gated(sq, oracle):
    # the GDN mixer between its projections (gdn.rs:290-573): conv front end -> gated
    # delta rule (q/k already L2-normalised by the front end) -> norm_gated
    rng = np.random.default_rng(21)
    T, H_k, H_v = 8, 16, 32
    x, w, st = conv_inputs(rng, 1, T, 1)
    z = rng.standard_normal((T, H_v, D)).astype(np.float32)
    wn = rng.standard_normal(D).astype(np.float32)
    g = (-np.exp(rng.uniform(0, 2.7, (T, H_v))) * np.log1p(np.exp(rng.standard_normal((T, H_v))))).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal((T, H_v))))).astype(np.float32)
    S0 = (rng.standard_normal((H_v, D, D)) * 0.02).astype(np.float32)

    conv = sq.gdn_conv(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(), torch.from_numpy(st).cuda(),
                       n_qk_channels=NQK, l2_eps=1e-6)[0]
    q = conv[:, :H_k * D].view(T, H_k, D)
    k = conv[:, H_k * D:2 * H_k * D].view(T, H_k, D)
    v = conv[:, 2 * H_k * D:].view(T, H_v, D)
    state = torch.from_numpy(S0.copy()).cuda()[None, None]
    o = sq.gated_delta_net(q.contiguous(), k.contiguous(), v.contiguous(), torch.from_numpy(g).cuda(),
                           torch.from_numpy(beta).cuda(), state)
    y = sq.head_norm(o[0], 1e-6, weight=torch.from_numpy(wn).cuda(), z=torch.from_numpy(z).cuda())
    torch.cuda.synchronize()

    cw, _ = oracle.gdn_conv(x[0], w, st[0], n_qk=NQK, d=D, eps=1e-6)
    qo = cw[:, :H_k * D].reshape(T, H_k, D)
    ko = cw[:, H_k * D:2 * H_k * D].reshape(T, H_k, D)
    vo = cw[:, 2 * H_k * D:].reshape(T, H_v, D)
    oo, _ = oracle.gdn(qo, ko, vo, g, beta, S0)
    want = oracle.rms_norm(oo, 1e-6, w=wn, z=z)
    assert rel_err(y.cpu().numpy(), want) <= GDN_TOL
