"""GDN value-head sharding, host side, as world_size-2 gloo process groups on the CPU:
each rank runs the oracle recurrence over its value heads only (q/k head = the layer
index of the value head modulo H_k, as the kernels do with h_v_offset) and the gathered
outputs and states equal one whole-layer recurrence (gdn.rs:9-24, :436-441)."""
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


def _case(seed, T, h_k=16, h_v=32, d=128):
    import oracle

    rng = np.random.default_rng(seed)
    q = oracle.l2norm(rng.standard_normal((T, h_k, d)).astype(np.float32))
    k = oracle.l2norm(rng.standard_normal((T, h_k, d)).astype(np.float32))
    v = rng.standard_normal((T, h_v, d)).astype(np.float32)
    g = -rng.uniform(0.01, 1.0, (T, h_v)).astype(np.float32)
    b = rng.uniform(0.1, 0.9, (T, h_v)).astype(np.float32)
    S = (rng.standard_normal((h_v, d, d)) * 0.02).astype(np.float32)
    return q, k, v, g, b, S


def _local_gdn(oracle, q, k, v, g, b, S, h0, n, h_k):
    """The recurrence of value heads [h0, h0 + n) alone: the oracle over a layer whose q/k
    heads are re-indexed so that local head i reads layer q/k head (h0 + i) % h_k."""
    idx = [(h0 + i) % h_k for i in range(n)]
    return oracle.gdn(q[:, idx], k[:, idx], v[:, h0:h0 + n], g[:, h0:h0 + n], b[:, h0:h0 + n], S[h0:h0 + n],
                      n_snap=1)


def _rank_main(rank, world, port, T, seed):
    sys.path.insert(0, REPO)
    sys.path.insert(0, os.path.join(REPO, "sqwen-moe-3090_b200"))
    import datetime

    import torch.distributed as dist

    import oracle
    from sqmix import gdn_shard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        q, k, v, g, b, S = _case(seed, T)
        sh = gdn_shard.plan(32, world, rank)
        out, snaps = _local_gdn(oracle, q, k, v, g, b, S, sh.start, sh.count, 16)
        out_all = gdn_shard.gather_heads(torch.from_numpy(out), 32).numpy()
        st_all = gdn_shard.gather_heads(torch.from_numpy(snaps[0]).reshape(sh.count, 128 * 128, 1)
                                        .permute(2, 0, 1).reshape(1, sh.count, 128 * 128), 32).numpy()
        if rank == 0:
            want, wsnap = oracle.gdn(q, k, v, g, b, S, n_snap=1)
            assert np.abs(out_all - want).max() <= 1e-6 * np.abs(want).max()
            assert np.abs(st_all.reshape(32, 128, 128) - wsnap[0]).max() <= 1e-6 * np.abs(wsnap[0]).max()
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_head_plan_covers_every_head_once():
    sys.path.insert(0, os.path.join(REPO, "sqwen-moe-3090_b200"))
    from sqmix import gdn_shard

    for world in (1, 2, 3, 4, 5, 8):
        heads = [h for r in range(world) for h in gdn_shard.plan(32, world, r).heads()]
        assert heads == list(range(32))
    with pytest.raises(ValueError):
        gdn_shard.plan(4, 8, 0)


@pytest.mark.parametrize("T", [1, 5])
def test_value_head_sharding_world2(T):
    mp.spawn(_rank_main, args=(2, _free_port(), T, 90 + T), nprocs=2, join=True)
