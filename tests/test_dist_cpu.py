"""Multi-rank host logic on CPU with the gloo backend (world size 2): shards cover
the batch exactly once, each rank computes its shard independently (here with the
CPU oracle on the scaled-down model), and the gathered action chunks equal the
single-process result for the whole batch — the path needs no collective."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from vla_b200.dist import shard_bounds


def test_shard_bounds_cover_exactly_once():
    for n in (0, 1, 7, 8, 255, 256):
        for w in (1, 2, 3, 8):
            seen = []
            for r in range(w):
                a, b = shard_bounds(n, r, w)
                seen.extend(range(a, b))
                assert (b - a) in (n // w, n // w + 1)
            assert seen == list(range(n))
    with pytest.raises(ValueError):
        shard_bounds(4, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, batch, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "vla-to-npu_b200")]
    import torch.distributed as dist
    from oracle import smolvla_ref as R
    from vla_b200 import weights as W
    from vla_b200.configs import tiny_cfg
    from vla_b200.dist import gather_actions, shard
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.set_num_threads(1)
    cfg = tiny_cfg()
    params = W.smolvla_params(cfg, seed=0)
    obs = W.observation_batch(cfg, batch, seed=1)
    mine = shard(obs, rank, world)
    local = R.smolvla_chunk(mine, params, cfg, dt=torch.float32)
    full = gather_actions(local, batch)
    if rank == 0:
        q.put(full)
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_partition_matches_single_process():
    batch, world = 5, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, batch, q)) for r in range(world)]
    for p in procs:
        p.start()
    gathered = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    from oracle import smolvla_ref as R
    from vla_b200 import weights as W
    from vla_b200.configs import tiny_cfg
    cfg = tiny_cfg()
    ref = R.smolvla_chunk(W.observation_batch(cfg, batch, seed=1), W.smolvla_params(cfg, seed=0), cfg,
                          dt=torch.float32)
    torch.testing.assert_close(gathered, ref, atol=1e-5, rtol=1e-5)
