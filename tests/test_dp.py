"""Data-parallel sampling host logic (thinksound.cpp_b200/dp.py) on CPU with gloo ranks.

Sharding by prompt and the final gather to rank 0 are checked with a deterministic stand-in
sampler (the GPU sampler itself is covered by the gpu tests); world sizes 2 and 3 with even,
uneven and smaller-than-world prompt counts.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

# spawned ranks import this module without conftest: make the package importable here too
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)
import __graft_entry__  # noqa: E402

__graft_entry__.load_package()
from tsd_b200 import dp  # noqa: E402


def fake_sample(items, steps, cfg):
    # per prompt: a function of its own noise only, so the gathered order is checkable
    return np.stack([np.asarray(x, np.float32) * cfg + steps for x in items])


def make_items(n, C=4, T=6):
    rng = np.random.default_rng(7)
    return [rng.standard_normal((C, T)).astype(np.float32) for _ in range(n)]


def _worker(rank, world, port, n, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        out = dp.sample_sharded(fake_sample, make_items(n), 24, 5.0, rank, world)
        q.put((rank, None if out is None else out.tolist()))
    finally:
        dist.destroy_process_group()


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_ranges_cover_prompts_once():
    for n in range(0, 20):
        for world in (1, 2, 3, 8):
            got = [dp.shard_range(n, r, world) for r in range(world)]
            assert got[0][0] == 0 and got[-1][1] == n
            assert all(got[r][1] == got[r + 1][0] for r in range(world - 1))
            sizes = [hi - lo for lo, hi in got]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        dp.shard_range(4, 2, 2)


@pytest.mark.parametrize("world,n", [(2, 8), (2, 5), (3, 7), (2, 1)])
def test_sample_sharded_gathers_in_prompt_order(world, n):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref = fake_sample(make_items(n), 24, 5.0)
    assert np.allclose(np.asarray(results[0], np.float32), ref)
    assert all(results[r] is None for r in range(1, world))
