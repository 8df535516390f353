"""Data-parallel CFG sampling over prompts: one process per GPU, torch.distributed for the plumbing.

The reference samples one prompt at a time (`ts_dit::sample`, src/mmdit.cpp:344-376: a cond and
an uncond forward per Euler step, the CFG combine and the Euler update on the host), called by
ts-generate once per prompt (src/generate.cpp:81-89). Prompts are independent and a prompt's
cond/uncond pair must stay together for the CFG combine, so the natural partition is by prompt:
rank r samples a contiguous block of prompts with `tsd_sample_batched` (all of its prompts'
cond + uncond passes as one batch per step) and nothing is exchanged while sampling. At the end
the latents ([prompts][latent_dim][T] f32, 3.2 MB for 64 prompts at T=194) are gathered to
rank 0 in prompt order.

The sampler is passed in as a function so that the sharding and the gather can run with any
backend: NCCL with the CUDA library on GPUs, gloo with a stand-in on CPU (tests).
"""
from __future__ import annotations

from typing import Callable, List, Optional, Sequence, Tuple

import numpy as np


def shard_range(n: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous prompt range [lo, hi) of `rank`: the first n % world ranks take one extra."""
    if world < 1 or not 0 <= rank < world or n < 0:
        raise ValueError(f"bad shard request n={n} rank={rank} world={world}")
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def sample_sharded(sample_fn: Callable[[Sequence, int, float], np.ndarray], items: Sequence, steps: int, cfg: float,
                   rank: int, world: int, device=None, group=None) -> Optional[np.ndarray]:
    """Sample this rank's share of `items` with sample_fn(items, steps, cfg) -> [n][C][T] f32, then
    gather every rank's latents to rank 0. Returns [len(items)][C][T] on rank 0, None elsewhere.

    Every rank takes the same collective steps (one gather), including ranks whose share is
    empty. `device`: where the gather buffers live (a CUDA device for NCCL, None = CPU)."""
    import torch
    import torch.distributed as dist

    lo, hi = shard_range(len(items), rank, world)
    if hi > lo:
        local = np.ascontiguousarray(sample_fn(items[lo:hi], steps, cfg), dtype=np.float32)
        if local.ndim != 3 or local.shape[0] != hi - lo:
            raise ValueError(f"sampler returned {local.shape} for {hi - lo} prompts")
        shape = local.shape[1:]
    else:
        local = None
        shape = None
    if world == 1:
        return local if local is not None else np.zeros((0,), np.float32)
    # every shard has the same per-prompt shape; ranks with no prompts learn it from the others
    shapes: List[Optional[Tuple[int, int]]] = [None] * world
    dist.all_gather_object(shapes, shape, group=group)
    shape = next(s for s in shapes if s is not None)
    cap = -(-len(items) // world)                       # largest shard
    buf = torch.zeros((cap,) + tuple(shape), dtype=torch.float32, device=device)
    if local is not None:
        buf[: hi - lo].copy_(torch.from_numpy(local))
    gathered = [torch.empty_like(buf) for _ in range(world)] if rank == 0 else None
    dist.gather(buf, gather_list=gathered, dst=0, group=group)
    if rank != 0:
        return None
    parts = []
    for r in range(world):
        rlo, rhi = shard_range(len(items), r, world)
        parts.append(gathered[r][: rhi - rlo].cpu().numpy())
    return np.concatenate(parts, axis=0)


def exchange_handles(handle: bytes, rank: int, world: int, group=None) -> List[bytes]:
    """Every rank's IPC handle in rank order (one all_gather_object; any backend)."""
    import torch.distributed as dist

    if world == 1:
        return [handle]
    out: List[Optional[bytes]] = [None] * world
    dist.all_gather_object(out, handle, group=group)
    if any(not isinstance(h, (bytes, bytearray)) or len(h) != len(handle) for h in out):
        raise RuntimeError("head-parallel set-up: a rank sent no handle")
    return [bytes(h) for h in out]


def head_parallel(model, rank: int, world: int, arena_bytes: int = 1 << 30, group=None) -> None:
    """Put `model` (this rank's copy of the DiT) into head-parallel mode: rank r computes heads
    [r * nh / world, (r + 1) * nh / world) of every block and exchanges its attention rows with
    the other ranks over peer memory (tsd_hp_init / tsd_hp_connect). Collective: every rank of
    the group calls it, then all ranks issue the same forwards. Before freeing the models, end
    with a barrier so that no rank frees its exchange buffer while a peer still maps it."""
    import torch.distributed as dist

    handle = model.hp_init(rank, world, arena_bytes)
    handles = exchange_handles(handle, rank, world, group)
    model.hp_connect(handles)
    if world > 1:
        dist.barrier(group=group)   # every rank has mapped every peer before any forward stores to it
