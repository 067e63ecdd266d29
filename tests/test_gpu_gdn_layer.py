"""GPU parity of the one-launch GDN decode layer (sqmix_gdn_layer_decode): conv + SiLU +
q/k L2 norm + gate epilogue + recurrence with snapshot slots + norm_gated, against

- the three-launch path (sqmix_gdn_conv -> sqmix_gdn_decode with the gate epilogue ->
  sqmix_head_norm) on the same inputs: outputs, state planes and conv-history planes;
- the oracle chain (gdn_conv -> gdn_gates -> gdn -> rms_norm), within the GDN bar of
  1e-3 relative;

for one and two tokens (the MTP verify with two snapshot slots), a rollback plane
selector, one and three sequences, f32 and bf16 projections.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

C, K, D, H_K, H_V = 8192, 4, 128, 16, 32
NQK = 2 * H_K * D
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


def _case(seed, n_seqs, T, n_planes, bf16):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((n_seqs, T, C)).astype(np.float32)
    z = rng.standard_normal((n_seqs, T, H_V, D)).astype(np.float32)
    if bf16:  # round through bf16 so that every path sees the values the device reads
        x = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
        z = torch.from_numpy(z).to(torch.bfloat16).float().numpy()
    return dict(
        x=x, z=z,
        w=(rng.standard_normal((C, K)) * 0.5).astype(np.float32),
        cst=rng.standard_normal((n_seqs, n_planes, C, K - 1)).astype(np.float32),
        S=(rng.standard_normal((n_seqs, n_planes, H_V, D, D)) * 0.02).astype(np.float32),
        alpha=(rng.standard_normal((n_seqs, T, H_V)) * 2.0).astype(np.float32),
        b=rng.standard_normal((n_seqs, T, H_V)).astype(np.float32),
        dt=rng.standard_normal(H_V).astype(np.float32),
        ssm_a=(-np.exp(rng.uniform(0.0, 2.7, H_V))).astype(np.float32),
        wn=rng.uniform(0.5, 1.5, D).astype(np.float32),
    )


def _dev(a, bf16=False):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t.to(torch.bfloat16) if bf16 else t


@pytest.mark.parametrize("n_seqs,T,n_planes,sel,bf16", [(1, 1, 1, 0, False), (1, 1, 3, 2, True),
                                                        (1, 2, 3, 1, False), (3, 2, 2, 1, True),
                                                        (3, 1, 2, 0, False)])
def test_gdn_layer_decode(sq, oracle, n_seqs, T, n_planes, sel, bf16):
    c = _case(1000 + 10 * n_seqs + T + n_planes + bf16, n_seqs, T, n_planes, bf16)
    n_snap = min(T, n_planes)
    sel_t = torch.full((n_seqs,), sel, dtype=torch.int32, device="cuda")
    x, z = _dev(c["x"], bf16), _dev(c["z"], bf16)
    w, dt, ssm_a, wn = _dev(c["w"]), _dev(c["dt"]), _dev(c["ssm_a"]), _dev(c["wn"])
    alpha, b = _dev(c["alpha"]), _dev(c["b"])

    # one launch
    cst1, S1 = _dev(c["cst"]), _dev(c["S"])
    y1 = sq.gdn_layer_decode(x, w, cst1, alpha, b, ssm_a, S1, dt_bias=dt, n_planes=n_planes, sel=sel_t,
                             n_snap=n_snap, l2_eps=1e-6, z=z, norm_weight=wn, norm_eps=1e-6)
    # three launches
    cst3, S3 = _dev(c["cst"]), _dev(c["S"])
    conv = sq.gdn_conv(x, w, cst3, n_planes=n_planes, sel=sel_t, n_snap=n_snap, n_qk_channels=NQK, l2_eps=1e-6)
    q = conv[:, :, :H_K * D].reshape(n_seqs, T, H_K, D)
    k = conv[:, :, H_K * D:NQK].reshape(n_seqs, T, H_K, D)
    v = conv[:, :, NQK:].reshape(n_seqs, T, H_V, D)
    o = sq.gated_delta_net(q.contiguous(), k.contiguous(), v.contiguous(), alpha, b, S3, n_planes=n_planes, sel=sel_t,
                           n_snap=n_snap, dt_bias=dt, ssm_a=ssm_a)
    y3 = sq.head_norm(o.reshape(n_seqs * T, H_V, D), 1e-6, weight=wn, z=z.reshape(n_seqs * T, H_V, D))
    torch.cuda.synchronize()
    assert rel_err(y1.cpu().numpy(), y3.reshape(n_seqs, T, H_V, D).cpu().numpy()) <= 1e-4
    assert torch.equal(cst1, cst3)  # the history slots are the same bytes
    assert rel_err(S1.cpu().numpy(), S3.cpu().numpy()) <= 1e-4

    # the oracle chain, per sequence
    g_ref, b_ref = oracle.gdn_gates(c["alpha"], c["b"], c["dt"], c["ssm_a"])
    for s in range(n_seqs):
        cw, st_want = oracle.gdn_conv(c["x"][s], c["w"], c["cst"][s], sel=sel, n_snap=n_snap, n_qk=NQK, d=D, eps=1e-6)
        qo = cw[:, :H_K * D].reshape(T, H_K, D)
        ko = cw[:, H_K * D:NQK].reshape(T, H_K, D)
        vo = cw[:, NQK:].reshape(T, H_V, D)
        oo, snaps = oracle.gdn(qo, ko, vo, g_ref[s], b_ref[s], c["S"][s, sel], n_snap=n_snap)
        want = oracle.rms_norm(oo, 1e-6, w=c["wn"], z=c["z"][s])
        assert rel_err(y1[s].cpu().numpy(), want) <= GDN_TOL, s
        assert np.array_equal(cst1[s].cpu().numpy(), st_want), s
        for slot in range(n_snap):
            assert rel_err(S1[s, slot].cpu().numpy(), snaps[slot]) <= GDN_TOL, (s, slot)


def test_gdn_layer_decode_rejects_long_chunks(sq):
    c = _case(7, 1, 3, 1, False)
    with pytest.raises(sq.SqmixError, match="n_tokens=3"):
        sq.gdn_layer_decode(_dev(c["x"]), _dev(c["w"]), _dev(c["cst"]), _dev(c["alpha"]), _dev(c["b"]),
                            _dev(c["ssm_a"]), _dev(c["S"]))
