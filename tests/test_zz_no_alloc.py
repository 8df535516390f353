"""The no-allocation GEMM entry point, tsd_op_gemm_static.

Some callers cannot call cudaMalloc: a plugin that lives inside a host process which owns all
GPU memory through its own pool, or a real-time serving loop that may not take cudaMalloc's
implicit device synchronisation and unbounded latency once it is running. For them the
library keeps the GEMM's split-K scratch in fixed device arrays of its own; this test calls
that entry point through the C-ABI and checks it against tsd_op_gemm (scratch from the
caller) on two calls in a row, which also shows that the second call is not disturbed by
what the first one left in the shared arrays.

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


@pytest.mark.parametrize("mode", [tsd.EPI_STORE, tsd.EPI_GATE_RESID])
def test_static_scratch_gemm_matches_caller_scratch_gemm(mode):
    torch.manual_seed(0)
    # long K, few tokens: the planner splits K, so the static scratch is in use
    M, K, taps, nb, S = 512, 1536, 3, 2, 40
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
        args = (W, M, K, taps, 1, X, nb, S, K, S * K, mode, 0, bias, None if mode == tsd.EPI_GATE_RESID else out, 0, M)
        if static:
            tsd.op_gemm_static(*args, max_splits=8, **kw)
        else:
            tsd.op_gemm(*args, max_splits=8, ws=ws, counters=counters, **kw)
        torch.cuda.synchronize()
        return resid if mode == tsd.EPI_GATE_RESID else out

    ref = run(static=False)
    for _ in range(2):                       # two calls in a row share the static arrays
        got = run(static=True)
        assert rel(got, ref) < 1e-5


def test_static_scratch_gemm_rejects_oversized_outputs():
    W = torch.zeros(4096, 128, device=DEV, dtype=torch.bfloat16)
    X = torch.zeros(1, 1024, 128, device=DEV, dtype=torch.bfloat16)
    out = torch.empty(1024, 4096, device=DEV)
    with pytest.raises(tsd.TsdError) as e:   # 4096 x 1024 outputs > the static limit
        tsd.op_gemm_static(W, 4096, 128, 1, 0, X, 1, 1024, 128, 1024 * 128, tsd.EPI_STORE, 0, None, out, 0, 4096)
    assert e.value.rc == -1
