"""GPU tests of the cross-GPU split-KV merge over peer memory (sqmix_attn_merge_peers).

- loopback (one rank, runs on any GPU box): publish + merge of a single partial is the
  partial itself (gated), over several steps and slots (flag counters, parity buffers);
- two ranks on two GPUs (skipped with fewer): each rank decodes its half of the keys
  with flash_attn_ext and the peer merge must equal attention over all keys (oracle).
"""
import ctypes
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ATTN_TOL = 2e-3


def test_peer_merge_loopback_single_rank():
    import sqmix
    from sqmix._lib import PeerMergeArgs, check, lib

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    n_slots, rows = 2, 16
    own = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(64)
    check(lib().sqmix_peer_buffer_create(n_slots, ctypes.byref(own), handle), "create")
    try:
        ptrs = torch.tensor([own.value], dtype=torch.int64, device="cuda")
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        g = torch.Generator(device="cuda")
        g.manual_seed(3)
        for step in range(3):
            for slot in range(n_slots):
                o = torch.randn((rows, 256), generator=g, device="cuda")
                lse = torch.randn((rows,), generator=g, device="cuda")
                gate = torch.randn((rows, 256), generator=g, device="cuda")
                out = torch.empty_like(o)
                lse_out = torch.empty_like(lse)
                a = PeerMergeArgs(n_ranks=1, rank=0, slot=slot, n_slots=n_slots, rows=rows,
                                  buffers=ptrs.data_ptr(), o_local=o.data_ptr(), lse_local=lse.data_ptr(),
                                  gate=gate.data_ptr(), out=out.data_ptr(), lse_out=lse_out.data_ptr(),
                                  status=status.data_ptr())
                check(lib().sqmix_attn_merge_peers(ctypes.byref(a), None), "merge")
                torch.cuda.synchronize()
                want = o * torch.sigmoid(gate)
                assert torch.allclose(out, want, rtol=1e-5, atol=1e-6)
                assert torch.allclose(lse_out, lse, rtol=1e-6, atol=1e-6)
        assert int(status.item()) == 0
    finally:
        check(lib().sqmix_peer_buffer_destroy(own), "destroy")
    del sqmix


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, n_keys, seed):
    sys.path.insert(0, REPO)
    sys.path.insert(0, os.path.join(REPO, "sqwen-moe-3090_b200"))
    import datetime

    import torch.distributed as dist

    import oracle
    import sqmix
    from sqmix import split_kv

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    pm = None
    try:
        rng = np.random.default_rng(seed)
        k = rng.standard_normal((n_keys, 2, 256)).astype(np.float32)
        v = rng.standard_normal((n_keys, 2, 256)).astype(np.float32)
        sh = split_kv.plan(n_keys, world, rank)
        kc, vc = sqmix.new_kv_cache(sh.capacity, dev), sqmix.new_kv_cache(sh.capacity, dev)
        sqmix.set_rows_q4_0(torch.from_numpy(k[sh.start:sh.start + sh.length]).to(dev),
                            torch.from_numpy(v[sh.start:sh.start + sh.length]).to(dev),
                            torch.arange(sh.length, device=dev), kc, vc, sh.capacity, rope_n_rot=64,
                            rope_freq_base=1e7, rope_pos_offset=sh.start)
        n_loc, qp = sh.local_step(n_keys, n_keys - 1)
        d = torch.tensor([n_loc, qp], dtype=torch.int64, device=dev)
        kd = oracle.q4_0_dequantize(oracle.q4_0_quantize(oracle.rope_text(k, 0, 1e7, 64).reshape(n_keys, 512)),
                                    512).reshape(n_keys, 2, 256)
        vd = oracle.q4_0_dequantize(oracle.q4_0_quantize(v.reshape(n_keys, 512)), 512).reshape(n_keys, 2, 256)
        pm = split_kv.PeerMerge(n_slots=2, rows=16, device=dev)
        for step in range(3):
            for slot in range(2):
                q = rng.standard_normal((1, 16, 256)).astype(np.float32)
                gate = rng.standard_normal((1, 16, 256)).astype(np.float32)
                lse = torch.empty((1, 16), device=dev)
                o = sqmix.flash_attn_ext(torch.from_numpy(q).to(dev), kc, vc, sh.capacity, d[0:1], d[1:2],
                                         rope_n_rot=64, rope_freq_base=1e7, rope_pos_offset=sh.start, lse=lse)
                out = pm.merge(o, lse, slot, gate=torch.from_numpy(gate).to(dev))
                torch.cuda.synchronize()
                want = oracle.attn(oracle.rope_text(q, n_keys - 1, 1e7, 64), kd, vd, gate, q_pos0=n_keys - 1,
                                   scale=1 / 16)
                got = out.cpu().numpy().reshape(want.shape)
                err = np.abs(got - want).max() / np.abs(want).max()
                assert err <= ATTN_TOL, (rank, step, slot, err)
        assert pm.ok()
    finally:
        if pm is not None:
            pm.close()
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_merge_two_gpus(oracle):
    mp.spawn(_rank_main, args=(2, _free_port(), 3000, 11), nprocs=2, join=True)
