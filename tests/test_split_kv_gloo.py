"""Split-KV across ranks, host side: the shard plan and the gather + LSE merge
protocol, run as world_size-2 gloo process groups on the CPU.  Each rank computes its
partial attention with the CPU oracle over its key slice (the GPU kernel produces the
same (O, LSE) pair on a GPU rank); the merged result must equal attention over all keys.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(seed, n_keys, n_q):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((n_q, 16, 256)).astype(np.float32)
    k = rng.standard_normal((n_keys, 2, 256)).astype(np.float32)
    v = rng.standard_normal((n_keys, 2, 256)).astype(np.float32)
    gate = rng.standard_normal((n_q, 16, 256)).astype(np.float32)
    return q, k, v, gate


def _rank_main(rank, world, port, n_keys, n_q, q_pos0, seed):
    sys.path.insert(0, REPO)
    sys.path.insert(0, os.path.join(REPO, "sqwen-moe-3090_b200"))
    import datetime

    import torch.distributed as dist

    import oracle
    from sqmix import split_kv

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        q, k, v, gate = _case(seed, n_keys, n_q)
        sh = split_kv.plan(n_keys, world, rank)
        n_local, qp_local = sh.local_step(n_keys, q_pos0)
        ks, vs = k[sh.start:sh.start + n_local], v[sh.start:sh.start + n_local]
        if n_local > 0:
            o, lse = oracle.attn(q, ks, vs, None, q_pos0=qp_local, scale=1 / 16, want_lse=True)
        else:
            o = np.zeros((n_q, 16, 256), np.float32)
            lse = np.full((n_q, 16), -np.inf, np.float32)
        o_all, l_all = split_kv.gather(torch.from_numpy(o).reshape(n_q * 16, 256),
                                       torch.from_numpy(lse).reshape(n_q * 16))
        assert o_all.shape == (world, n_q * 16, 256) and l_all.shape == (world, n_q * 16)
        if rank == 0:
            got, _ = oracle.merge_lse(o_all.numpy(), l_all.numpy(), gate.reshape(n_q * 16, 256))
            want = oracle.attn(q, k, v, gate, q_pos0=q_pos0, scale=1 / 16)
            err = np.abs(got.reshape(want.shape) - want).max() / np.abs(want).max()
            assert err < 1e-5, err
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n_keys,world", [(172032, 8), (1000, 2), (17, 2), (4096, 3), (33, 4)])
def test_plan_covers_keys_once(n_keys, world):
    sys.path.insert(0, os.path.join(REPO, "sqwen-moe-3090_b200"))
    from sqmix import split_kv

    shards = [split_kv.plan(n_keys, world, r) for r in range(world)]
    covered = np.zeros(n_keys, np.int32)
    for sh in shards:
        assert sh.start % split_kv.GROUP == 0 or sh.length == 0
        covered[sh.start:sh.start + sh.length] += 1
    assert (covered == 1).all()
    for pos in (0, n_keys // 2, n_keys - 1):
        r = split_kv.owner(n_keys, world, pos)
        assert shards[r].owns(pos)
    # local causal bounds: a slice entirely after the query contributes nothing
    for sh in shards:
        n_local, qp = sh.local_step(n_keys, 0)
        assert n_local == sh.length and qp == -sh.start


@pytest.mark.parametrize("q_pos0", [1998, 700])
def test_split_kv_gather_merge_gloo_world2(oracle, q_pos0):
    """2 ranks over gloo: decode (q_pos0 at the end) and a query inside rank 0's slice,
    where rank 1 sees no key and contributes LSE -inf."""
    mp.spawn(_rank_main, args=(2, _free_port(), 2000, 2, q_pos0, 5), nprocs=2, join=True)
