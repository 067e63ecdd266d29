"""GPU tests of the GDN value-head offset (row e3: value heads split across ranks) and the
on-device gate epilogue (row a11: beta = sigmoid(b), g = softplus(alpha + dt_bias) * ssm_a,
gdn.rs:268-287), for the recurrent decode kernel and the chunked prefill.

- shards: the 32 value heads run as 2 halves and 4 quarters (h_v_offset 0, 8, 16, 24 ...)
  with all 16 q/k heads; outputs and state planes equal the whole-layer call;
- gates: raw alpha / b with dt_bias and ssm_a equal the call with g and beta computed by
  the oracle's restatement of the epilogue, and the oracle recurrence within 1e-3.
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


def _inputs(seed, T, n_planes=1):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    q = torch.randn((1, T, 16, 128), generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn((1, T, 16, 128), generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn((1, T, 32, 128), generator=g, device="cuda").to(torch.bfloat16)
    gl = -torch.rand((1, T, 32), generator=g, device="cuda") * 0.9 - 0.01
    b = torch.rand((1, T, 32), generator=g, device="cuda") * 0.8 + 0.1
    S = torch.randn((1, n_planes, 32, 128, 128), generator=g, device="cuda") * 0.02
    return q, k, v, gl, b, S


@pytest.mark.parametrize("T,n_snap,chunked", [(1, 1, False), (2, 2, False), (200, 1, True), (130, 2, True)])
@pytest.mark.parametrize("world", [2, 4])
def test_gdn_head_offset_matches_whole_layer(sq, T, n_snap, chunked, world):
    q, k, v, gl, b, S = _inputs(300 + T + world, T, n_planes=n_snap)
    S_full = S.clone()
    out_full = sq.gated_delta_net(q, k, v, gl, b, S_full, n_planes=n_snap, n_snap=n_snap, l2_eps=1e-6,
                                  chunked=chunked)
    n = 32 // world
    for r in range(world):
        h0 = r * n
        S_loc = S[:, :, h0:h0 + n].clone().contiguous()
        out = sq.gated_delta_net(q, k, v[:, :, h0:h0 + n], gl[:, :, h0:h0 + n].contiguous(),
                                 b[:, :, h0:h0 + n].contiguous(), S_loc, n_planes=n_snap, n_snap=n_snap,
                                 l2_eps=1e-6, chunked=chunked, h_v_offset=h0)
        torch.cuda.synchronize()
        assert torch.allclose(out, out_full[:, :, h0:h0 + n], rtol=1e-5, atol=1e-6), r
        assert torch.allclose(S_loc, S_full[:, :, h0:h0 + n], rtol=1e-5, atol=1e-6), r


@pytest.mark.parametrize("T,chunked", [(1, False), (2, False), (130, True)])
def test_gdn_gate_epilogue(sq, oracle, T, chunked):
    q, k, v, _, _, S = _inputs(400 + T, T)
    rng = np.random.default_rng(400 + T)
    alpha = rng.standard_normal((1, T, 32)).astype(np.float32) * 3.0
    alpha[0, 0, :4] = [25.0, -30.0, 19.5, 20.5]  # both sides of the softplus threshold
    braw = rng.standard_normal((1, T, 32)).astype(np.float32) * 2.0
    dt = rng.standard_normal(32).astype(np.float32)
    a_log = rng.uniform(0.0, 2.7, 32)
    ssm_a = (-np.exp(a_log)).astype(np.float32)
    g_ref, b_ref = oracle.gdn_gates(alpha, braw, dt, ssm_a)
    S_a, S_b = S.clone(), S.clone()
    out_raw = sq.gated_delta_net(q, k, v, torch.from_numpy(alpha).cuda(), torch.from_numpy(braw).cuda(), S_a,
                                 l2_eps=1e-6, chunked=chunked, dt_bias=torch.from_numpy(dt).cuda(),
                                 ssm_a=torch.from_numpy(ssm_a).cuda())
    out_pre = sq.gated_delta_net(q, k, v, torch.from_numpy(g_ref).cuda(), torch.from_numpy(b_ref).cuda(), S_b,
                                 l2_eps=1e-6, chunked=chunked)
    torch.cuda.synchronize()
    # the device's f32 softplus and the oracle's double one differ by an ulp of g, which
    # the decay compounds over the tokens (130 tokens: ~4e-5 of the largest element)
    for a_, b_ in ((out_raw, out_pre), (S_a, S_b)):
        assert float((a_ - b_).abs().max() / b_.abs().max()) <= 1e-4
    qn = oracle.l2norm(q.float().cpu().numpy()[0])
    kn = oracle.l2norm(k.float().cpu().numpy()[0])
    want, snaps = oracle.gdn(qn, kn, v.float().cpu().numpy()[0], g_ref[0], b_ref[0], S.cpu().numpy()[0, 0], n_snap=1)
    got = out_raw.cpu().numpy()[0]
    assert np.abs(got - want).max() <= GDN_TOL * np.abs(want).max()
    st = S_a.cpu().numpy()[0, 0]
    assert np.abs(st - snaps[0]).max() <= GDN_TOL * np.abs(snaps[0]).max()
