"""One process driving two GPUs: the kernels that need more than 48 KB of dynamic shared
memory (decode, prefill, chunked GDN prefill) must launch on the second device too (the
attribute that allows it is per device).  Skipped with fewer than two GPUs."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _run_on(sq, dev):
    with torch.cuda.device(dev):
        g = torch.Generator(device=dev)
        g.manual_seed(3)
        n_kv, cap = 600, 768
        kc, vc = sq.new_kv_cache(cap, device=dev), sq.new_kv_cache(cap, device=dev)
        sq.set_rows_q4_0(torch.randn((n_kv, 2, 256), generator=g, device=dev),
                         torch.randn((n_kv, 2, 256), generator=g, device=dev),
                         torch.arange(n_kv, device=dev), kc, vc, cap, rope_n_rot=64, rope_freq_base=1e7)
        d = torch.tensor([n_kv, n_kv - 40], dtype=torch.int64, device=dev)
        q = torch.randn((40, 16, 256), generator=g, device=dev).to(torch.bfloat16)
        pf = sq.flash_attn_prefill(q, kc, vc, cap, d[0:1], d[1:2], rope_n_rot=64, rope_freq_base=1e7)
        d1 = torch.tensor([n_kv, n_kv - 1], dtype=torch.int64, device=dev)
        dec = sq.flash_attn_ext(q[-1:].float(), kc, vc, cap, d1[0:1], d1[1:2], rope_n_rot=64, rope_freq_base=1e7)
        S = torch.randn((1, 1, 32, 128, 128), generator=g, device=dev) * 0.02
        qk = torch.nn.functional.normalize(torch.randn((1, 128, 16, 128), generator=g, device=dev), dim=-1)
        v = torch.randn((1, 128, 32, 128), generator=g, device=dev)
        gg = -torch.rand((1, 128, 32), generator=g, device=dev)
        bt = torch.rand((1, 128, 32), generator=g, device=dev)
        o = sq.gated_delta_net(qk, qk.clone(), v, gg, bt, S, chunked=True)
        torch.cuda.synchronize(dev)
        return pf.cpu().numpy(), dec.cpu().numpy(), o.cpu().numpy()


def test_kernels_launch_on_two_devices_of_one_process():
    import sqmix

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    a = _run_on(sqmix, torch.device("cuda", 0))
    b = _run_on(sqmix, torch.device("cuda", 1))
    for x, y in zip(a, b):  # same seeded inputs: the same results on both devices
        assert np.array_equal(x, y)
    # decode of the last prompt token equals the prefill's last row
    assert np.abs(a[0][-1] - a[1][0]).max() <= 2e-3 * np.abs(a[0][-1]).max()
