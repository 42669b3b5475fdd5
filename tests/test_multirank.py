"""Host logic of the data-parallel path on CPU: world_size-2 process groups over gloo.

The op shards by (b, h) with no collective inside it (every sequence is independent, the
reference folds heads into the batch, nope_gdn_mlx.py:833-838).  These tests check, without a
GPU, that the batch shards cover the global batch exactly once, that the per-rank oracle
results reassemble into the unsharded result (outputs and gradients), and that the step time
is the maximum over ranks."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mlx_vit_b200.shard import max_over_ranks, shard_batch, shard_range
from mlx_vit_b200.synthetic import make_inputs
from oracle.kda_oracle import fwd_bwd


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        B, T, H, D = 3, 20, 2, 8
        inp = make_inputs(B, T, H, D, seed=5, state_std=0.1)  # the same global batch everywhere
        mine = {k: shard_batch(torch.from_numpy(v), world, rank).numpy() for k, v in inp.items()}
        res = fwd_bwd(mine)
        # gather every rank's shard results on rank 0 (object collective over gloo)
        gathered = [None] * world
        dist.all_gather_object(gathered, res)
        step_ms = max_over_ranks(10.0 + rank)  # rank 1 is the slowest
        if rank == 0:
            out.put((gathered, step_ms))
    finally:
        dist.destroy_process_group()


def test_shard_range_covers_every_item_once():
    for n in range(0, 13):
        for world in range(1, 6):
            seen = []
            for r in range(world):
                a, b = shard_range(n, world, r)
                assert 0 <= a <= b <= n
                seen.extend(range(a, b))
            assert seen == list(range(n))
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def test_two_rank_gloo_shards_reassemble_to_the_global_result():
    world = 2
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    gathered, step_ms = out.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert step_ms == 11.0
    B, T, H, D = 3, 20, 2, 8
    inp = make_inputs(B, T, H, D, seed=5, state_std=0.1)
    full = fwd_bwd(inp)
    for name in full:
        parts = np.concatenate([g[name] for g in gathered], axis=0)
        np.testing.assert_allclose(parts, full[name], rtol=1e-6, atol=1e-7, err_msg=name)
