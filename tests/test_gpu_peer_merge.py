"""GPU tests of the cross-GPU split-KV exchange over peer memory (sqmix_attn_merge_peers
and the fused decode sqmix_fa_decode_peers).

- loopback (one rank, runs on any GPU box): publish + merge of a single partial is the
  partial itself (gated), over several steps and slots (counters, parity buffers);
- fused decode with one rank equals sqmix_fa_decode;
- two ranks' exchange on ONE GPU without any kernel waiting on another: rank 0's
  publication is written into rank 1's buffer by the test (exactly the tagged words
  rank 0's kernel would push), so rank 1's launch finds it and completes; rank 1's
  launch pushes into rank 0's buffer, so rank 0's launch then completes too.  Both
  results must equal the decode over all keys; three steps over two slots exercise the
  tags, parities and counters;
- a wait that runs out: rank 0 of two with a peer buffer nobody writes gives up after
  the 2 s bound, sets the status bit, writes nothing and leaves the GPU usable;
- two ranks on two GPUs (skipped with fewer): each rank decodes its half of the keys
  and the exchange must equal attention over all keys (oracle).
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


# peer buffer layout (csrc/peer.cuh): data [slot][parity 2][src 8][row 32][slice 8][33] u64
_SLOT_WORDS = 2 * 8 * 32 * 8 * 33


def _peer_word(slot, parity, src, row, slice_, j):
    return slot * _SLOT_WORDS + ((((parity * 8 + src) * 32 + row) * 8 + slice_) * 33 + j)


def _publish(buf_words, slot, tag, src, o, lse):
    """Write the words that rank `src` pushes for publication `tag` of `slot`: o [rows][256]
    normalised partial, lse [rows]; value bits in the low 32 bits, the tag in the high."""
    rows = o.shape[0]
    par = tag & 1
    vals = torch.empty((rows, 8, 33), dtype=torch.float32, device=o.device)
    vals[:, :, :32] = o.reshape(rows, 8, 32)
    vals[:, :, 32] = lse.reshape(rows, 1)
    words = vals.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    words = words | (int(tag) << 32)
    base = _peer_word(slot, par, src, 0, 0, 0)
    buf_words[base:base + rows * 8 * 33] = words.reshape(-1)


def _new_buffer(n_slots):
    from sqmix._lib import check, lib
    from sqmix.state import _device_tensor

    own = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(64)
    check(lib().sqmix_peer_buffer_create(n_slots, ctypes.byref(own), handle), "create")
    nbytes = lib().sqmix_peer_buffer_bytes(n_slots)
    return own.value, _device_tensor(own.value, nbytes // 8 * 8, dtype=torch.int64)


def test_fa_decode_peers_single_rank_equals_decode():
    import sqmix
    from sqmix._lib import FaArgs, PeerMergeArgs, check, lib
    from sqmix.ops import _fa_args

    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    n_kv, cap = 3000, 3072
    kc, vc = sqmix.new_kv_cache(cap), sqmix.new_kv_cache(cap)
    sqmix.set_rows_q4_0(torch.randn((n_kv, 2, 256), generator=g, device="cuda"),
                        torch.randn((n_kv, 2, 256), generator=g, device="cuda"),
                        torch.arange(n_kv, device="cuda"), kc, vc, cap, rope_n_rot=64, rope_freq_base=1e7)
    ptr, _ = _new_buffer(1)
    try:
        ptrs = torch.tensor([ptr], dtype=torch.int64, device="cuda")
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        for n_q in (1, 2):
            q = torch.randn((n_q, 16, 256), generator=g, device="cuda")
            gate = torch.randn((n_q, 16, 256), generator=g, device="cuda")
            d = torch.tensor([n_kv, n_kv - n_q], dtype=torch.int64, device="cuda")
            want_lse = torch.empty((n_q, 16), device="cuda")
            want = sqmix.flash_attn_ext(q, kc, vc, cap, d[0:1], d[1:2], gate=gate, rope_n_rot=64, lse=want_lse)
            for step in range(2):
                ws = sqmix.new_fa_workspace(n_q)
                lse = torch.empty((n_q, 16), device="cuda")
                a, out = _fa_args(q, kc, vc, cap, d[0:1], d[1:2], gate, 1 / 16, 64, 1e7, 0, None, lse, ws, 0, 0,
                                  None, None, 0)
                pm = PeerMergeArgs(n_ranks=1, rank=0, slot=0, n_slots=1, rows=16 * n_q, buffers=ptrs.data_ptr(),
                                   status=status.data_ptr())
                check(lib().sqmix_fa_decode_peers(ctypes.byref(a), ctypes.byref(pm), None), "fa_decode_peers")
                torch.cuda.synchronize()
                assert torch.allclose(out, want, rtol=1e-6, atol=1e-7)
                assert torch.allclose(lse, want_lse, rtol=1e-6, atol=1e-6)
        assert int(status.item()) == 0
    finally:
        check(lib().sqmix_peer_buffer_destroy(ctypes.c_void_p(ptr)), "destroy")


def test_fa_decode_peers_two_ranks_on_one_gpu(oracle):
    """Two ranks' slices of one cache, exchanged through two peer buffers on one GPU with
    no concurrent waiting (see the module docstring)."""
    import sqmix
    from sqmix import split_kv
    from sqmix._lib import PeerMergeArgs, check, lib
    from sqmix.ops import _fa_args

    rng = np.random.default_rng(17)
    n_keys, n_slots = 2500, 2
    k = rng.standard_normal((n_keys, 2, 256)).astype(np.float32)
    v = rng.standard_normal((n_keys, 2, 256)).astype(np.float32)
    shards = [split_kv.plan(n_keys, 2, r) for r in range(2)]
    caches = []
    for sh in shards:
        kc, vc = sqmix.new_kv_cache(sh.capacity), sqmix.new_kv_cache(sh.capacity)
        sqmix.set_rows_q4_0(torch.from_numpy(k[sh.start:sh.start + sh.length]).cuda(),
                            torch.from_numpy(v[sh.start:sh.start + sh.length]).cuda(),
                            torch.arange(sh.length, device="cuda"), kc, vc, sh.capacity, rope_n_rot=64,
                            rope_freq_base=1e7, rope_pos_offset=sh.start)
        caches.append((kc, vc))
    kd = oracle.q4_0_dequantize(oracle.q4_0_quantize(oracle.rope_text(k, 0, 1e7, 64).reshape(n_keys, 512)),
                                512).reshape(n_keys, 2, 256)
    vd = oracle.q4_0_dequantize(oracle.q4_0_quantize(v.reshape(n_keys, 512)), 512).reshape(n_keys, 2, 256)
    bufs = [_new_buffer(n_slots) for _ in range(2)]
    try:
        ptrs = torch.tensor([bufs[0][0], bufs[1][0]], dtype=torch.int64, device="cuda")
        status = torch.zeros(1, dtype=torch.int32, device="cuda")

        def decode(rank, q, gate, n_q, slot, fused=True, lse=None):
            sh = shards[rank]
            n_loc, qp = sh.local_step(n_keys, n_keys - n_q)
            d = torch.tensor([n_loc, qp], dtype=torch.int64, device="cuda")
            kc, vc = caches[rank]
            if not fused:
                return sqmix.flash_attn_ext(q, kc, vc, sh.capacity, d[0:1], d[1:2], rope_n_rot=64, rope_freq_base=1e7,
                                            rope_pos_offset=sh.start, lse=lse)
            a, out = _fa_args(q, kc, vc, sh.capacity, d[0:1], d[1:2], gate, 1 / 16, 64, 1e7, sh.start, None, lse,
                              sqmix.new_fa_workspace(n_q), 0, 0, None, None, 0)
            pm = PeerMergeArgs(n_ranks=2, rank=rank, slot=slot, n_slots=n_slots, rows=16 * n_q, buffers=ptrs.data_ptr(),
                               status=status.data_ptr())
            check(lib().sqmix_fa_decode_peers(ctypes.byref(a), ctypes.byref(pm), None), "fa_decode_peers")
            return out

        for step in range(3):
            for slot in range(n_slots):
                n_q = 1 + slot  # slot 1 carries the 2-token query: every row's counter advances per step
                tag = step + 1
                q = torch.from_numpy(rng.standard_normal((n_q, 16, 256)).astype(np.float32)).cuda()
                gate = torch.from_numpy(rng.standard_normal((n_q, 16, 256)).astype(np.float32)).cuda()
                # rank 0's publication, as its fused kernel would push it into rank 1's buffer
                lse0 = torch.empty((n_q, 16), device="cuda")
                o0 = decode(0, q, gate, n_q, slot, fused=False, lse=lse0)
                _publish(bufs[1][1], slot, tag, 0, o0.reshape(16 * n_q, 256), lse0.reshape(-1))
                torch.cuda.synchronize()
                lse1 = torch.empty((n_q, 16), device="cuda")
                out1 = decode(1, q, gate, n_q, slot, lse=lse1)   # finds rank 0's words, pushes its own
                out0 = decode(0, q, gate, n_q, slot)             # finds rank 1's words
                torch.cuda.synchronize()
                assert int(status.item()) == 0, (step, slot)
                want, wlse = oracle.attn(oracle.rope_text(q.cpu().numpy(), n_keys - n_q, 1e7, 64), kd, vd,
                                         gate.cpu().numpy(), q_pos0=n_keys - n_q, scale=1 / 16, want_lse=True)
                for got in (out0, out1):
                    err = np.abs(got.cpu().numpy() - want).max() / np.abs(want).max()
                    assert err <= ATTN_TOL, (step, slot, err)
                assert np.abs(lse1.cpu().numpy() - wlse).max() < 1e-3
                assert torch.equal(out0, out1)
    finally:
        for ptr, _ in bufs:
            check(lib().sqmix_peer_buffer_destroy(ctypes.c_void_p(ptr)), "destroy")


def test_peer_merge_wait_gives_up_and_gpu_stays_usable():
    """Rank 0 of two whose peer never publishes: the bounded wait ends after ~2 s, sets bit 1
    of the status word, writes nothing; the GPU keeps working; a reset clears the buffer."""
    import time

    from sqmix._lib import PeerMergeArgs, check, lib

    n_slots, rows = 1, 16
    bufs = [_new_buffer(n_slots) for _ in range(2)]
    try:
        ptrs = torch.tensor([bufs[0][0], bufs[1][0]], dtype=torch.int64, device="cuda")
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        o = torch.randn((rows, 256), device="cuda")
        lse = torch.randn((rows,), device="cuda")
        out = torch.full((rows, 256), float("nan"), device="cuda")
        a = PeerMergeArgs(n_ranks=2, rank=0, slot=0, n_slots=n_slots, rows=rows, buffers=ptrs.data_ptr(),
                          o_local=o.data_ptr(), lse_local=lse.data_ptr(), gate=None, out=out.data_ptr(),
                          lse_out=None, status=status.data_ptr())
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        check(lib().sqmix_attn_merge_peers(ctypes.byref(a), None), "merge")
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        assert 1.5 < dt < 30.0, dt
        assert int(status.item()) & 1
        assert torch.isnan(out).all()
        x = torch.arange(1000, device="cuda", dtype=torch.float32)
        assert float(x.sum().item()) == 499500.0  # the context is still usable
        check(lib().sqmix_peer_buffer_reset(ctypes.c_void_p(bufs[0][0]), n_slots, None), "reset")
        torch.cuda.synchronize()
        assert int(bufs[0][1].abs().sum().item()) == 0
    finally:
        for ptr, _ in bufs:
            check(lib().sqmix_peer_buffer_destroy(ctypes.c_void_p(ptr)), "destroy")


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
                if slot == 0:  # slot 0: decode then the standalone exchange; slot 1: the fused decode
                    o = sqmix.flash_attn_ext(torch.from_numpy(q).to(dev), kc, vc, sh.capacity, d[0:1], d[1:2],
                                             rope_n_rot=64, rope_freq_base=1e7, rope_pos_offset=sh.start, lse=lse)
                    out = pm.merge(o, lse, slot, gate=torch.from_numpy(gate).to(dev))
                else:
                    out = pm.decode(torch.from_numpy(q).to(dev), kc, vc, sh.capacity, d[0:1], d[1:2], slot,
                                    gate=torch.from_numpy(gate).to(dev), rope_n_rot=64, rope_freq_base=1e7,
                                    rope_pos_offset=sh.start)
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
