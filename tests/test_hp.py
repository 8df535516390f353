"""Head-parallel mode (include/tsd.h tsd_hp_*; thinksound.cpp_b200/dp.py head_parallel).

CPU: the head layout of every rank (tsd_hp_layout) and the handle exchange over gloo ranks.
GPU (two B200s of one box): a head-parallel forward and sampler on two ranks give bit-identical
results to the single-GPU path, for a width whose per-rank Q/K/V sections need padding rows.
"""
import os
import socket
import sys
import time

import numpy as np
import pytest
import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)
import __graft_entry__  # noqa: E402

__graft_entry__.load_package()
from tsd_b200 import dp, synth, tsd  # noqa: E402


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("H,nh", [(1536, 24), (1024, 16), (384, 6)])
def test_hp_layout_covers_every_head_once(H, nh):
    for world in range(1, 9):
        if nh % world:
            with pytest.raises(tsd.TsdError):
                tsd.hp_layout(H, nh, world, 0)
            continue
        heads = []
        for r in range(world):
            h0, nl, sec = tsd.hp_layout(H, nh, world, r)
            assert nl == nh // world and sec % 128 == 0 and nl * 64 <= sec < nl * 64 + 128
            heads += list(range(h0, h0 + nl))
        assert heads == list(range(nh))
    with pytest.raises(tsd.TsdError):
        tsd.hp_layout(H, nh, 9, 0)          # more ranks than one node's GPUs
    with pytest.raises(tsd.TsdError):
        tsd.hp_layout(H + 64, nh, 1, 0)     # head_dim must be 64


def _exchange_worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = bytes([rank]) * tsd.IPC_HANDLE_BYTES
        q.put((rank, dp.exchange_handles(mine, rank, world)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_handles_are_exchanged_in_rank_order(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = [bytes([r]) * tsd.IPC_HANDLE_BYTES for r in range(world)]
    assert all(got[r] == want for r in range(world))


# ---------------------------------------------------------------------------------------- GPU
HP = dict(hidden=384, n_head=6, depth=3, fused_depth=1, ffn=768)   # 3 heads per rank: padded sections
SHAPES = [dict(T=40, clip_S=16, sync_S=48, text_S=77, t5_S=20), dict(T=24, clip_S=8, sync_S=24, text_S=77, t5_S=9)]


def _hp_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    out = {}
    try:
        hp = synth.DitHParams(**HP)
        W = synth.make_weights(hp, seed=1234, wtype="bf16")
        m = tsd.DitModel.from_weights(hp, W, device=rank)
        dp.head_parallel(m, rank, world, arena_bytes=256 << 20)
        for k, sh in enumerate(SHAPES):           # two plans: the second carves fresh exchange buffers
            items = synth.make_inputs(hp, seed=4242 + k, batch=2, **sh)
            out[f"flow{k}"] = m.forward(items)
            out[f"flow{k}b"] = m.forward(items)   # a second forward of the same plan (next epoch)
        x = synth.make_inputs(hp, seed=77, batch=1, **SHAPES[0])[0]
        out["latent"] = m.sample([x], steps=3, cfg=5.0)
        dist.barrier()                            # no rank frees its exchange buffer while a peer maps it
        m.close()
        if rank == 0:                             # the single-GPU path on the same weights and inputs
            ref = tsd.DitModel.from_weights(hp, W, device=0)
            for k, sh in enumerate(SHAPES):
                out[f"ref{k}"] = ref.forward(synth.make_inputs(hp, seed=4242 + k, batch=2, **sh))
            out["ref_latent"] = ref.sample([x], steps=3, cfg=5.0)
            ref.close()
        q.put((rank, out, None))
    except Exception as e:  # report to the parent instead of leaving it waiting
        q.put((rank, None, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_head_parallel_two_gpus_equals_single_gpu():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs of one node")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_hp_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, out, err = q.get(timeout=600)
        assert err is None, f"rank {r}: {err}"
        res[r] = out
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for k in range(len(SHAPES)):
        ref = res[0][f"ref{k}"]
        for r in range(world):
            assert np.array_equal(res[r][f"flow{k}"], ref), (k, r)
            assert np.array_equal(res[r][f"flow{k}b"], ref), (k, r)
    for r in range(world):
        assert np.array_equal(res[r]["latent"], res[0]["ref_latent"])


def _hp_skip_worker(rank, world, port, q):
    """Both ranks set up head-parallel mode; rank 1 then skips the forward (it stays alive with
    nothing in flight). Rank 0's forward pushes its rows and waits for rank 1's, which never
    come: its bounded wait runs out and the forward returns TSD_ERR_DEVICE."""
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    out = {}
    try:
        hp = synth.DitHParams(**HP)
        W = synth.make_weights(hp, seed=1234, wtype="bf16")
        m = tsd.DitModel.from_weights(hp, W, device=rank)
        dp.head_parallel(m, rank, world, arena_bytes=256 << 20)
        tsd.set_wait_limit(rank, 200_000_000)      # 200 ms
        items = synth.make_inputs(hp, seed=4242, batch=2, **SHAPES[0])
        if rank == 0:
            t0 = time.perf_counter()
            try:
                m.forward(items)
                out["rc"] = 0
            except tsd.TsdError as e:
                out["rc"] = e.rc
            out["seconds"] = time.perf_counter() - t0
        dist.barrier()                            # rank 0's forward has returned; nothing is in flight
        tsd.set_wait_limit(rank, 2_000_000_000)
        m.close()
        if rank == 0:                             # the GPU still works: a plain single-GPU forward
            ref = tsd.DitModel.from_weights(hp, W, device=0)
            out["ok_after"] = bool(np.isfinite(ref.forward(items)).all())
            ref.close()
        q.put((rank, out, None))
    except Exception as e:  # report to the parent instead of leaving it waiting
        q.put((rank, None, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_head_parallel_missing_peer_ends_in_device_error():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs of one node")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_hp_skip_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, out, err = q.get(timeout=600)
        assert err is None, f"rank {r}: {err}"
        res[r] = out
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert res[0]["rc"] == -5                      # TSD_ERR_DEVICE
    assert res[0]["seconds"] < 30
    assert res[0]["ok_after"]
