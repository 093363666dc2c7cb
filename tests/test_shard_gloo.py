"""Multi-rank host logic on CPU: world-size-2 gloo ranks shard 64 independent
streams, each computes its own (oracle) Snake+Conv1d outputs with no data
collective, and the whole-job time is the max over ranks."""
import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from sonata_b200.shard import shard_range


def test_shard_range_covers_everything_once():
    for total in (0, 1, 7, 64, 65, 1000):
        for world in (1, 2, 3, 4, 8):
            seen = []
            sizes = []
            for r in range(world):
                a, b = shard_range(total, world, r)
                seen.extend(range(a, b))
                sizes.append(b - a)
            assert seen == list(range(total))
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_dir):
    import datetime
    import torch.distributed as dist

    import oracle as O
    from sonata_b200.shard import max_over_ranks, shard_range, sum_over_ranks
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    streams, C, T = 8, 8, 64
    rng = np.random.default_rng(0)  # every rank draws the same full batch
    x = rng.standard_normal((streams, C, T)).astype(np.float32)
    alpha = (rng.random(C) + 0.5).astype(np.float32)
    W = (rng.standard_normal((C, C, 7)) / np.sqrt(7 * C)).astype(np.float32)
    b = rng.standard_normal(C).astype(np.float32)
    a, e = shard_range(streams, world, rank)
    dist.barrier()
    t0 = time.perf_counter()
    y = O.snake_conv1d_ref(x[a:e], alpha, W, b, padding=3, dilation=1)
    el = time.perf_counter() - t0
    t_max = max_over_ranks(el)
    n = sum_over_ranks(e - a)
    np.save(os.path.join(out_dir, f"y{rank}.npy"), y)
    with open(os.path.join(out_dir, f"meta{rank}.txt"), "w") as f:
        f.write(f"{a} {e} {t_max} {el} {n}\n")
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_shard_streams(tmp_path):
    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    import oracle as O
    metas = [open(tmp_path / f"meta{r}.txt").read().split() for r in range(world)]
    ys = [np.load(tmp_path / f"y{r}.npy") for r in range(world)]
    # shards are disjoint and complete, and each rank saw the same max time
    assert [(int(m[0]), int(m[1])) for m in metas] == [(0, 4), (4, 8)]
    assert float(metas[0][2]) == float(metas[1][2]) >= max(float(m[3]) for m in metas)
    assert int(float(metas[0][4])) == 8
    rng = np.random.default_rng(0)
    x = rng.standard_normal((8, 8, 64)).astype(np.float32)
    alpha = (rng.random(8) + 0.5).astype(np.float32)
    W = (rng.standard_normal((8, 8, 7)) / np.sqrt(56)).astype(np.float32)
    b = rng.standard_normal(8).astype(np.float32)
    full = O.snake_conv1d_ref(x, alpha, W, b, padding=3, dilation=1)
    np.testing.assert_array_equal(np.concatenate(ys), full)
