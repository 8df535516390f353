"""The no-allocation GEMM entry point, tsd_op_gemm_static.

Some callers cannot call cudaMalloc: a plugin that lives inside a host process which owns all
GPU memory through its own pool, or a real-time serving loop that may not take cudaMalloc's
implicit device synchronisation and unbounded latency once it is running. For them the
library keeps the GEMM's split-K scratch in fixed device arrays of its own; these tests call
that entry point through the C-ABI and check it against tsd_op_gemm (scratch from the caller)
on two calls in a row, which also shows that the second call is not disturbed by what the
first one left in the shared arrays.

This file is collected last so that a run stopping at the first failure has already run
every other test; it passes on its own in a fresh process as well.
"""
import pytest
import torch

from tsd_b200 import tsd

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def rel(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return float(((a - b).norm() / (b.norm() + 1e-30)).item())


def run_pair(mode, M, K, taps, nb, S, seed=0):
    """(tsd_op_gemm with caller scratch, [tsd_op_gemm_static twice]) on the same operands."""
    torch.manual_seed(seed)
    W = (0.02 * torch.randn(M, taps * K, device=DEV)).to(torch.bfloat16)
    X = torch.randn(nb, S, K, device=DEV).to(torch.bfloat16)
    bias = torch.randn(M, device=DEV)
    gate = torch.randn(nb * S, M, device=DEV)
    x0 = torch.randn(nb, S, M, device=DEV)
    ws = torch.empty(8 << 20, device=DEV)
    counters = torch.zeros(1 << 16, device=DEV, dtype=torch.int32)

    def run(static):
        out = torch.zeros(nb, S, M, device=DEV)
        resid = x0.clone()
        kw = dict(resid=resid, ldr=M, gate=gate, ldg=M, gate_div=1) if mode == tsd.EPI_GATE_RESID else {}
        args = (W, M, K, taps, (taps - 1) // 2, X, nb, S, K, S * K, mode, 0, bias,
                None if mode == tsd.EPI_GATE_RESID else out, 0, M)
        if static:
            tsd.op_gemm_static(*args, max_splits=8, **kw)
        else:
            tsd.op_gemm(*args, max_splits=8, ws=ws, counters=counters, **kw)
        torch.cuda.synchronize()
        return resid if mode == tsd.EPI_GATE_RESID else out

    ref = run(static=False)
    return ref, [run(static=True) for _ in range(2)]   # two calls in a row share the static arrays


@pytest.mark.parametrize("mode", [tsd.EPI_STORE, tsd.EPI_GATE_RESID])
def test_static_scratch_gemm_matches_caller_scratch_gemm(mode, monkeypatch):
    # Very long K, few tokens: the planner splits K. With the in-cluster reduction switched off
    # the splits reduce through global scratch, which for the static entry point is its device
    # arrays.
    monkeypatch.setenv("TSD_NO_CLUSTER_SPLIT", "1")
    M, K, taps, nb, S = 512, 8192, 3, 2, 40
    plan = tsd.op_gemm_plan(M, K, taps, nb, S, 8, tsd.GEMM_STATIC_WS_FLOATS, tsd.GEMM_STATIC_COUNTERS)
    assert plan["splits"] > 1 and not plan["csplit"] and 0 < plan["ws_floats"] <= tsd.GEMM_STATIC_WS_FLOATS, plan
    ref, got = run_pair(mode, M, K, taps, nb, S)
    for g in got:
        assert rel(g, ref) < 1e-5


def test_static_scratch_gemm_default_plan_matches():
    """Without the switch: the default plan (split-K inside a cluster where it fits, no scratch)."""
    ref, got = run_pair(tsd.EPI_GATE_RESID, 512, 1536, 3, 2, 40, seed=1)
    for g in got:
        assert rel(g, ref) < 1e-5


def test_static_scratch_gemm_large_outputs():
    """Outputs far larger than the scratch: plans that would need more scratch than the arrays
    hold split K less (or not at all), so every shape runs and matches tsd_op_gemm."""
    for M, K, taps, nb, S in ((4096, 128, 1, 1, 1024), (1536, 4096, 3, 2, 646)):
        plan = tsd.op_gemm_plan(M, K, taps, nb, S, 8, tsd.GEMM_STATIC_WS_FLOATS, tsd.GEMM_STATIC_COUNTERS)
        assert plan["ws_floats"] <= tsd.GEMM_STATIC_WS_FLOATS, plan
        ref, got = run_pair(tsd.EPI_STORE, M, K, taps, nb, S, seed=2)
        for g in got:
            assert rel(g, ref) < 1e-5
