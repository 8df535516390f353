"""Failure detection on the GPU without a GPU fault.

Every device-side wait in the library is bounded (tsd_set_wait_limit, 2 s by default): a wait that
runs out records an error code in a device error word and its kernel returns, so the context
stays usable and the host reports TSD_ERR_DEVICE. Here the head-parallel arrival wait is made to
run out on purpose (its counters are a buffer nothing writes), with a short limit, and a normal
forward runs afterwards on the same GPU and gives the same result as before.
"""
import time

import numpy as np
import pytest
import torch

from tsd_b200 import synth, tsd

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
SMALL = dict(hidden=128, n_head=2, depth=3, fused_depth=1, ffn=256)
SHAPE = dict(T=20, clip_S=8, sync_S=24, text_S=77, t5_S=9)


@pytest.fixture
def short_wait_limit():
    tsd.set_wait_limit(0, 100_000_000)          # 100 ms
    yield 0.1
    tsd.set_wait_limit(0, 2_000_000_000)        # back to the default


def test_peer_wait_runs_out_and_reports(short_wait_limit):
    hp = synth.DitHParams(**SMALL)
    W = synth.make_weights(hp, seed=5, wtype="bf16")
    items = synth.make_inputs(hp, seed=6, batch=2, **SHAPE)
    m = tsd.DitModel.from_weights(hp, W)
    before = m.forward(items)

    counters = torch.zeros(8, dtype=torch.int32, device=DEV)   # rank 1's arrivals: never written
    epoch = torch.ones(1, dtype=torch.int32, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    tsd.op_peer_wait(counters, epoch, rank=0, world=2, ctas=1, err=err)
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    assert int(err.item()) != 0                       # the wait gave up and said so
    assert short_wait_limit * 0.9 <= dt < 1.5, dt     # after the short limit, not the 2 s default

    # arrivals that did happen satisfy the same wait at once
    counters[1] = 1
    err.zero_()
    tsd.op_peer_wait(counters, epoch, rank=0, world=2, ctas=1, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0

    # the GPU and the model are unaffected
    after = m.forward(items)
    assert np.array_equal(before, after)
    m.close()


def test_wait_limit_is_restored(short_wait_limit):
    tsd.set_wait_limit(0, 2_000_000_000)
    counters = torch.zeros(8, dtype=torch.int32, device=DEV)
    counters[1] = 3
    epoch = torch.full((1,), 3, dtype=torch.int32, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    tsd.op_peer_wait(counters, epoch, rank=0, world=2, ctas=1, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
