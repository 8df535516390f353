"""GPU parity of the individual sm_100a kernels (through the C-ABI op entry points) against
plain PyTorch fp32 restatements of the same ops on the same bf16/fp16-rounded operands."""
import math

import numpy as np
import pytest
import torch

from tsd_b200 import synth, tsd

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def rel(a, b):
    a = a.double().flatten()
    b = b.double().flatten()
    return float(((a - b).norm() / (b.norm() + 1e-30)).item())


def ref_gemm(W, X, taps, pad):
    """X [nb][S][K] (bf16), W [M][taps*K] (bf16) -> fp32 [nb][S][M]."""
    nb, S, K = X.shape
    M = W.shape[0]
    Wf = W.float().view(M, taps, K)
    Xf = X.float()
    out = torch.zeros(nb, S, M, device=X.device)
    for tap in range(taps):
        sh = torch.zeros_like(Xf)
        off = tap - pad
        lo, hi = max(0, -off), min(S, S - off)
        if hi > lo:
            sh[:, lo:hi] = Xf[:, lo + off:hi + off]
        out += sh @ Wf[:, tap, :].T
    return out


def rnd(*shape, scale=1.0, dtype=torch.bfloat16, g=None):
    return (scale * torch.randn(*shape, generator=g, device=DEV)).to(dtype)


@pytest.fixture(autouse=True)
def _seed():
    torch.manual_seed(0)


@pytest.mark.parametrize("M,K,taps,pad,nb,S", [
    (256, 128, 1, 0, 1, 300),     # linear, two token tiles
    (128, 64, 3, 1, 2, 194),      # conv k3 with batch boundaries (latent input proj shape)
    (384, 256, 3, 1, 3, 17),      # ragged tiny sequence
    (128, 192, 7, 3, 2, 40),      # conv k7 (sync input proj / final conv)
    (128, 128, 1, 0, 1, 1),       # single token
    (512, 1536, 1, 0, 1, 388),    # QKV-like K
    (4096, 256, 1, 0, 1, 2000),   # > one tile per persistent CTA (TMEM double buffer cycles)
    (1024, 128, 3, 1, 4, 500),    # conv, many tiles per CTA, ragged last tile per item
])
def test_gemm_store(M, K, taps, pad, nb, S):
    W = rnd(M, taps * K, scale=0.05)
    X = rnd(nb, S, K)
    bias = torch.randn(M, device=DEV)
    out = torch.empty(nb, S, M, device=DEV)
    tsd.op_gemm(W, M, K, taps, pad, X, nb, S, K, S * K, tsd.EPI_STORE, tsd.ACT_NONE, bias, out, 0, M)
    torch.cuda.synchronize()
    ref = ref_gemm(W, X, taps, pad) + bias
    assert rel(out, ref) < 1e-5


def test_gemm_store_bf16_silu_and_m_valid():
    M, K, S = 128, 128, 50
    W = rnd(M, 3 * K, scale=0.05)
    X = rnd(2, S, K)
    bias = torch.randn(M, device=DEV)
    out = torch.zeros(2, S, 64, device=DEV, dtype=torch.bfloat16)
    tsd.op_gemm(W, M, K, 3, 1, X, 2, S, K, S * K, tsd.EPI_STORE, tsd.ACT_SILU, bias, out, 1, 64, m_valid=64)
    torch.cuda.synchronize()
    ref = torch.nn.functional.silu(ref_gemm(W, X, 3, 1) + bias)[..., :64]
    assert rel(out.float(), ref) < 4e-3
    assert rel(out.float(), ref.to(torch.bfloat16).float()) < 1e-3


@pytest.mark.parametrize("taps,F,S", [(1, 256, 100), (3, 256, 100), (3, 2048, 700)])
def test_gemm_swiglu(taps, F, S):
    K = 128
    W1, W3 = rnd(F, taps * K, scale=0.05), rnd(F, taps * K, scale=0.05)
    W13 = torch.empty(2 * F, taps * K, device=DEV, dtype=torch.bfloat16)
    W13[0::2] = W1                               # rows alternate: w1 row f, w3 row f
    W13[1::2] = W3
    X = rnd(2, S, K)
    out = torch.empty(2, S, F, device=DEV, dtype=torch.bfloat16)
    tsd.op_gemm(W13, 2 * F, K, taps, taps // 2, X, 2, S, K, S * K, tsd.EPI_SWIGLU, 0, None, out, 1, F)
    torch.cuda.synchronize()
    ref = torch.nn.functional.silu(ref_gemm(W1, X, taps, taps // 2)) * ref_gemm(W3, X, taps, taps // 2)
    assert rel(out.float(), ref) < 4e-3


@pytest.mark.parametrize("per_token,splits,taps,M,S", [(1, 1, 3, 256, 72), (1, 4, 3, 256, 72), (0, 1, 1, 256, 72),
                                                        (0, 4, 1, 256, 72), (1, 8, 3, 1536, 600)])
def test_gemm_gate_residual(per_token, splits, taps, M, S):
    K, nb = 512, 2
    W = rnd(M, taps * K, scale=0.03)
    X = rnd(nb, S, K)
    bias = torch.randn(M, device=DEV)
    gate = torch.randn(nb * S if per_token else nb, M, device=DEV)
    x0 = torch.randn(nb, S, M, device=DEV)
    ws = torch.empty(8 << 20, device=DEV) if splits > 1 else None
    counters = torch.zeros(1 << 16, device=DEV, dtype=torch.int32) if splits > 1 else None
    outs = []
    for _ in range(2):
        x = x0.clone()
        tsd.op_gemm(W, M, K, taps, taps // 2, X, nb, S, K, S * K, tsd.EPI_GATE_RESID, 0, bias, None, 0, 0,
                    resid=x, ldr=M, gate=gate, ldg=M, gate_div=1 if per_token else S, max_splits=splits,
                    ws=ws, counters=counters)
        outs.append(x)
    torch.cuda.synchronize()
    g = gate.view(nb, S, M) if per_token else gate.view(nb, 1, M)
    ref = x0 + g * (ref_gemm(W, X, taps, taps // 2) + bias)
    assert rel(outs[0], ref) < 1e-5
    assert torch.equal(outs[0], outs[1])          # split-K partials are summed in a fixed order
    if counters is not None:
        assert int(counters.abs().sum()) == 0     # the kernel leaves its arrival counters zero


@pytest.mark.parametrize("mode", [tsd.EPI_STORE, tsd.EPI_SWIGLU])
def test_gemm_split_k_store_and_swiglu(mode):
    """Long-K, few-token GEMMs split K across CTAs; the last CTA of a tile reduces and runs the epilogue."""
    M, K, nb, S, taps = 512, 1536, 2, 40, 3
    W = rnd(M, taps * K, scale=0.02)
    X = rnd(nb, S, K)
    bias = torch.randn(M, device=DEV)
    ws = torch.empty(8 << 20, device=DEV)
    counters = torch.zeros(1 << 16, device=DEV, dtype=torch.int32)
    Fo = M // 2 if mode == tsd.EPI_SWIGLU else M
    outs = []
    for _ in range(2):
        out = torch.empty(nb, S, Fo, device=DEV)
        tsd.op_gemm(W, M, K, taps, 1, X, nb, S, K, S * K, mode, 0, bias if mode == tsd.EPI_STORE else None, out, 0, Fo,
                    max_splits=8, ws=ws, counters=counters)
        outs.append(out)
    torch.cuda.synchronize()
    acc = ref_gemm(W, X, taps, 1)
    if mode == tsd.EPI_STORE:
        ref = acc + bias
    else:
        ref = torch.nn.functional.silu(acc[..., 0::2]) * acc[..., 1::2]   # rows alternate w1 / w3
    assert rel(outs[0], ref) < 1e-5
    assert torch.equal(outs[0], outs[1])
    assert int(counters.abs().sum()) == 0


@pytest.mark.parametrize("mode,gate_div", [(tsd.EPI_STORE, 1), (tsd.EPI_SWIGLU, 1), (tsd.EPI_GATE_RESID, 1),
                                           (tsd.EPI_GATE_RESID, 0)])
@pytest.mark.parametrize("S,nb,taps", [(72, 2, 3), (72, 5, 3), (40, 7, 7), (100, 3, 1)])
@pytest.mark.parametrize("pair", [0, 1])
def test_gemm_multi_item_tiles(monkeypatch, S, nb, taps, mode, gate_div, pair):
    """Several short batch items side by side in one token tile (each weight tile read once for all
    of them; the clip stream's 72-token items), on single CTAs or CTA pairs (each CTA of a pair
    loading whole items): the same sums in the same K order as one item per tile on single CTAs,
    so bit-identical to it (no split-K on either side), and within 1e-5 of the f32 reference.
    nb = 5 / 7 / 3 leave the last tile of items partly empty."""
    M, K = 512, 512
    W = rnd(M, taps * K, scale=0.03)
    X = rnd(nb, S, K)
    bias = torch.randn(M, device=DEV)
    gdiv = gate_div if gate_div else S
    gate = torch.randn(nb * S // gdiv, M, device=DEV)
    x0 = torch.randn(nb, S, M, device=DEV)
    Fo = M // 2 if mode == tsd.EPI_SWIGLU else M
    out = {}
    for form in ("multi", "single"):
        for v in ("TSD_FORCE_MULTI_ITEM", "TSD_NO_MULTI_ITEM", "TSD_FORCE_PAIR", "TSD_NO_PAIR"):
            monkeypatch.delenv(v, raising=False)
        monkeypatch.setenv("TSD_FORCE_MULTI_ITEM" if form == "multi" else "TSD_NO_MULTI_ITEM", "1")
        monkeypatch.setenv("TSD_FORCE_PAIR" if form == "multi" and pair else "TSD_NO_PAIR", "1")
        plan = tsd.op_gemm_plan(M, K, taps, nb, S, 1)
        assert (plan["BN"] > (S + 15) // 16 * 16) == (form == "multi"), (form, plan)
        assert plan["pair"] == (pair if form == "multi" else 0), (form, plan)
        if mode == tsd.EPI_GATE_RESID:
            x = x0.clone()
            tsd.op_gemm(W, M, K, taps, taps // 2, X, nb, S, K, S * K, mode, 0, bias, None, 0, 0, resid=x, ldr=M,
                        gate=gate, ldg=M, gate_div=gdiv, max_splits=1)
        else:
            x = torch.empty(nb, S, Fo, device=DEV)
            tsd.op_gemm(W, M, K, taps, taps // 2, X, nb, S, K, S * K, mode, 0, bias if mode == tsd.EPI_STORE else None,
                        x, 0, Fo, max_splits=1)
        out[form] = x
    torch.cuda.synchronize()
    acc = ref_gemm(W, X, taps, taps // 2)
    if mode == tsd.EPI_GATE_RESID:
        ref = x0 + gate.view(nb, S // gdiv, 1, M).expand(nb, S // gdiv, gdiv, M).reshape(nb, S, M) * (acc + bias)
    elif mode == tsd.EPI_STORE:
        ref = acc + bias
    else:
        ref = torch.nn.functional.silu(acc[..., 0::2]) * acc[..., 1::2]
    assert rel(out["multi"], ref) < 1e-5
    assert torch.equal(out["multi"], out["single"])


@pytest.mark.parametrize("gather", [1, 0])
@pytest.mark.parametrize("mode,gate_div", [(tsd.EPI_GATE_RESID, 1), (tsd.EPI_GATE_RESID, 0), (tsd.EPI_STORE, 1),
                                           (tsd.EPI_SWIGLU, 1)])
@pytest.mark.parametrize("M,K,taps,nb,S", [(512, 8192, 3, 2, 40), (1536, 4096, 3, 2, 194)])
def test_gemm_workspace_split_k(monkeypatch, M, K, taps, nb, S, mode, gate_div, gather):
    """Split-K through the workspace (the in-cluster reduction switched off), one tile per CTA:
    the split that completes a tile last either gathers the other partials into its shared memory
    and finishes the tile like an unsplit one (gather), or a reducer reads them from the
    workspace. Both sum the partials in split order (two runs bit-identical) and leave the
    arrival counters zero. (1536, 4096 x 3, 2 x 194) is the fused blocks' FFN down-projection.
    gate_div 0: one gate row per batch item (the joint blocks' clip / text streams)."""
    monkeypatch.setenv("TSD_NO_CLUSTER_SPLIT", "1")
    if not gather:
        monkeypatch.setenv("TSD_NO_GATHER_SPLIT", "1")
    ws = torch.empty(8 << 20, device=DEV)
    counters = torch.zeros(1 << 16, device=DEV, dtype=torch.int32)
    plan = tsd.op_gemm_plan(M, K, taps, nb, S, 8, ws.numel(), counters.numel())
    if not gather and plan["splits"] == 1:
        pytest.skip("the model does not split this shape without the gathering reduction")
    assert plan["splits"] > 1 and not plan["csplit"] and plan["gather"] == gather, plan
    W = rnd(M, taps * K, scale=0.02)
    X = rnd(nb, S, K)
    bias = torch.randn(M, device=DEV)
    gdiv = gate_div if gate_div else S
    gate = torch.randn(nb * S // gdiv, M, device=DEV)
    x0 = torch.randn(nb, S, M, device=DEV)
    Fo = M // 2 if mode == tsd.EPI_SWIGLU else M
    outs = []
    for _ in range(2):
        if mode == tsd.EPI_GATE_RESID:
            x = x0.clone()
            tsd.op_gemm(W, M, K, taps, taps // 2, X, nb, S, K, S * K, mode, 0, bias, None, 0, 0, resid=x, ldr=M,
                        gate=gate, ldg=M, gate_div=gdiv, max_splits=8, ws=ws, counters=counters)
        else:
            x = torch.empty(nb, S, Fo, device=DEV)
            tsd.op_gemm(W, M, K, taps, taps // 2, X, nb, S, K, S * K, mode, 0, bias if mode == tsd.EPI_STORE else None,
                        x, 0, Fo, max_splits=8, ws=ws, counters=counters)
        outs.append(x)
    torch.cuda.synchronize()
    acc = ref_gemm(W, X, taps, taps // 2)
    if mode == tsd.EPI_GATE_RESID:
        ref = x0 + gate.view(nb, S // gdiv, 1, M).expand(nb, S // gdiv, gdiv, M).reshape(nb, S, M) * (acc + bias)
    elif mode == tsd.EPI_STORE:
        ref = acc + bias
    else:
        ref = torch.nn.functional.silu(acc[..., 0::2]) * acc[..., 1::2]
    assert rel(outs[0], ref) < 1e-5
    assert torch.equal(outs[0], outs[1])
    assert int(counters.abs().sum()) == 0


@pytest.mark.parametrize("M,K,taps,nb,S,mode,splits", [
    (1536, 1536, 3, 2, 194, tsd.EPI_GATE_RESID, 2),  # linear1 / w2 shape class: pair tiles + cluster split-K
    (4608, 256, 1, 1, 388, tsd.EPI_STORE, 1),        # QKV-like: one pair tile per CTA pair
    (2048, 256, 3, 2, 194, tsd.EPI_SWIGLU, 1),       # w1/w3 SwiGLU conv
    (512, 128, 1, 1, 3000, tsd.EPI_STORE, 1),        # many pair tiles per pair (TMEM double buffer)
    (1536, 2048, 3, 2, 194, tsd.EPI_STORE, 4),       # cluster split-K of pair tiles, plain store
])
def test_gemm_cta_pairs_match_single_ctas(monkeypatch, capfd, M, K, taps, nb, S, mode, splits):
    """CTA pairs (cta_group::2: 256 weight rows per pair, each CTA loading half of the token
    tile) give the single-CTA kernel's results."""
    W = rnd(M, taps * K, scale=0.03)
    X = rnd(nb, S, K)
    bias = torch.randn(M, device=DEV) if mode != tsd.EPI_SWIGLU else None
    gate = torch.randn(nb * S, M, device=DEV)
    x0 = torch.randn(nb, S, M, device=DEV)
    ws = torch.empty(8 << 20, device=DEV)
    counters = torch.zeros(1 << 16, device=DEV, dtype=torch.int32)
    Fo = M // 2 if mode == tsd.EPI_SWIGLU else M
    outs = {}
    monkeypatch.setenv("TSD_DEBUG_PLAN", "1")
    for no_pair in ("1", "0"):
        monkeypatch.setenv("TSD_NO_PAIR", no_pair)
        if no_pair == "0":
            monkeypatch.setenv("TSD_FORCE_PAIR", "1")     # the model's best pair tiling, even if single CTAs win
        capfd.readouterr()
        if mode == tsd.EPI_GATE_RESID:
            out = x0.clone()
            tsd.op_gemm(W, M, K, taps, taps // 2, X, nb, S, K, S * K, mode, 0, bias, None, 0, 0, resid=out, ldr=M,
                        gate=gate, ldg=M, gate_div=1, max_splits=splits, ws=ws, counters=counters)
        else:
            out = torch.empty(nb, S, Fo, device=DEV, dtype=torch.bfloat16 if mode == tsd.EPI_SWIGLU else torch.float32)
            tsd.op_gemm(W, M, K, taps, taps // 2, X, nb, S, K, S * K, mode, 0, bias, out,
                        1 if mode == tsd.EPI_SWIGLU else 0, Fo, max_splits=splits, ws=ws, counters=counters)
        torch.cuda.synchronize()
        err = capfd.readouterr().err
        assert ("pair=1" in err) == (no_pair == "0"), err
        outs[no_pair] = out.float()
    acc = ref_gemm(W, X, taps, taps // 2)
    if mode == tsd.EPI_SWIGLU:
        ref, tol = torch.nn.functional.silu(acc[..., 0::2]) * acc[..., 1::2], 4e-3
    elif mode == tsd.EPI_GATE_RESID:
        ref, tol = x0 + gate.view(nb, S, M) * (acc + bias), 1e-5
    else:
        ref, tol = acc + bias, 1e-5
    assert rel(outs["1"], ref) < tol and rel(outs["0"], ref) < tol
    # the two tilings may split K differently (a different f32 summation order)
    assert rel(outs["0"], outs["1"]) < (2e-3 if mode == tsd.EPI_SWIGLU else 1e-5)
    assert int(counters.abs().sum()) == 0


def test_gemm_strided_slice_of_joint_buffer():
    """linear1 reads its stream's rows out of the joint attention output [B][Sj][H]."""
    H, B, Sj, off, S = 128, 2, 300, 194, 72
    ao = rnd(B, Sj, H)
    W = rnd(H, 3 * H, scale=0.05)
    out = torch.empty(B, S, H, device=DEV)
    tsd.op_gemm(W, H, H, 3, 1, ao[:, off:], B, S, H, Sj * H, tsd.EPI_STORE, 0, None, out, 0, H)
    torch.cuda.synchronize()
    ref = ref_gemm(W, ao[:, off:off + S].contiguous(), 3, 1)
    assert rel(out, ref) < 1e-5


def gemv_weights(wtype, M, K, seed=1, scale=0.02):
    w = (scale * np.random.default_rng(seed).standard_normal((M, K))).astype(np.float32)
    if wtype == synth.GGML_BF16:
        raw = synth.f32_to_bf16_bits(w)
    elif wtype == synth.GGML_Q8_0:
        raw = synth.quantize_q8_0(w)
    else:
        raw = w
    wt = synth.WTensor("w", (K, M), wtype, raw)
    Wd = torch.from_numpy(np.ascontiguousarray(raw).view(np.uint8).copy()).to(DEV)
    return Wd, torch.from_numpy(wt.dequant()).to(DEV)


# K % 256 == 0 takes the streaming form (a whole phase of the row in flight; 4096 = several
# phases), K = 288 the per-chunk form.
@pytest.mark.parametrize("K", [512, 4096, 288])
@pytest.mark.parametrize("wtype", [synth.GGML_BF16, synth.GGML_F32, synth.GGML_Q8_0])
@pytest.mark.parametrize("N", [1, 2, 5])
def test_gemv(wtype, N, K):
    M = 300
    Wd, wf = gemv_weights(wtype, M, K)
    x = torch.randn(N, K, device=DEV)
    bias = torch.randn(M, device=DEV)
    y = torch.empty(N, M, device=DEV)
    tsd.op_gemv(Wd, wtype, None, M, K, x, K, N, bias, tsd.ACT_SILU, int(wtype == synth.GGML_BF16), y, 0, M)
    torch.cuda.synchronize()
    xr = x.to(torch.bfloat16).float() if wtype == synth.GGML_BF16 else x
    ref = torch.nn.functional.silu(xr @ wf.T + bias)
    assert rel(y, ref) < 1e-5


def test_gemv_q8_streaming_equals_per_chunk_form():
    """Q8_0 rows read as 16-byte words through shared memory must sum exactly like the
    per-chunk form (taken for weights that are not 16-byte aligned): same chunks per lane in
    the same order."""
    M, K, N = 777, 1536, 2
    Wd, _ = gemv_weights(synth.GGML_Q8_0, M, K, seed=5)
    shifted = torch.zeros(Wd.numel() + 16, dtype=torch.uint8, device=DEV)
    shifted[2:2 + Wd.numel()] = Wd.flatten()
    x = torch.randn(N, K, device=DEV)
    y1, y2 = torch.empty(N, M, device=DEV), torch.empty(N, M, device=DEV)
    tsd.op_gemv(Wd, synth.GGML_Q8_0, None, M, K, x, K, N, None, 0, 0, y1, 0, M)
    tsd.op_gemv(shifted[2:], synth.GGML_Q8_0, None, M, K, x, K, N, None, 0, 0, y2, 0, M)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    # operands the kernels cannot read with their word sizes are rejected, not read
    with pytest.raises(tsd.TsdError):
        tsd.op_gemv(shifted[1:], synth.GGML_Q8_0, None, M, K, x, K, N, None, 0, 0, y2, 0, M)
    wb = torch.zeros(M * K + 8, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(tsd.TsdError):
        tsd.op_gemv(wb[1:], synth.GGML_BF16, None, M, K, x, K, N, None, 0, 1, y2, 0, M)
    with pytest.raises(tsd.TsdError):
        tsd.op_gemv(Wd, synth.GGML_Q8_0, None, M, K, x.flatten()[1:], K, N, None, 0, 0, y2, 0, M)


@pytest.mark.parametrize("wtype,K", [(synth.GGML_BF16, 256), (synth.GGML_BF16, 4096), (synth.GGML_Q8_0, 1536),
                                     (synth.GGML_F32, 2048), (synth.GGML_BF16, 96)])
def test_gemv_swiglu_pair(wtype, K):
    M, N = 256, 2
    w1, f1 = gemv_weights(wtype, M, K, seed=2, scale=0.05)
    w3, f3 = gemv_weights(wtype, M, K, seed=3, scale=0.05)
    x = torch.randn(N, K, device=DEV)
    y = torch.empty(N, M, device=DEV)
    rb = int(wtype == synth.GGML_BF16)
    tsd.op_gemv(w1, wtype, w3, M, K, x, K, N, None, 0, rb, y, 0, M)
    torch.cuda.synchronize()
    xr = x.to(torch.bfloat16).float() if rb else x
    ref = torch.nn.functional.silu(xr @ f1.T) * (xr @ f3.T)
    assert rel(y, ref) < 1e-5


def ref_attention(Q, K, V, B, nh, S):
    q, k, v = (t.float().view(B, nh, S, 64) for t in (Q, K, V))
    p = torch.softmax(q @ k.transpose(-1, -2) / 8.0, dim=-1)
    return (p @ v).permute(0, 2, 1, 3).reshape(B, S, nh * 64)


@pytest.mark.parametrize("B,nh,S", [(1, 1, 1), (1, 2, 63), (2, 3, 128), (2, 4, 194), (2, 24, 471), (1, 2, 700)])
def test_attention(B, nh, S):
    Q = rnd(B * nh, S, 64, scale=1.5, dtype=torch.float16)
    K = rnd(B * nh, S, 64, scale=1.5, dtype=torch.float16)
    V = rnd(B * nh, S, 64, dtype=torch.float16)
    out = torch.empty(B, S, nh * 64, device=DEV, dtype=torch.bfloat16)
    err = torch.zeros(1, device=DEV, dtype=torch.int32)
    tsd.op_attention(Q, K, V, B, nh, S, out, nh * 64, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = ref_attention(Q, K, V, B, nh, S)
    assert rel(out.float(), ref.to(torch.bfloat16).float()) < 2e-3
    assert rel(out.float(), ref) < 4e-3


def test_attention_row_stride_and_peaked_softmax():
    """Large logits (peaked softmax, running-max rescale across KV chunks) into a wider buffer."""
    B, nh, S = 1, 2, 300
    Q = rnd(B * nh, S, 64, scale=4.0, dtype=torch.float16)
    K = rnd(B * nh, S, 64, scale=4.0, dtype=torch.float16)
    V = rnd(B * nh, S, 64, dtype=torch.float16)
    out = torch.zeros(B, S, 512, device=DEV, dtype=torch.bfloat16)
    tsd.op_attention(Q, K, V, B, nh, S, out, 512)
    torch.cuda.synchronize()
    ref = ref_attention(Q, K, V, B, nh, S)
    assert rel(out[..., :128].float(), ref) < 4e-3
    assert float(out[..., 128:].abs().max()) == 0.0


@pytest.mark.parametrize("growth", [0.5, 12.0, 60.0])
def test_attention_running_max_grows_across_chunks(growth):
    """Logits whose row maximum rises from KV chunk to chunk: by less than 2^8 per chunk (the
    kernel keeps its stale running max and P exceeds 1) and by far more (O and the running sums
    are rescaled in TMEM), over 6 chunks of 128 keys."""
    B, nh, S = 1, 3, 700
    Q = rnd(B * nh, S, 64, scale=1.0, dtype=torch.float32)
    K = rnd(B * nh, S, 64, scale=1.0, dtype=torch.float32)
    # key t gets an extra component aligned with every query's mean direction, growing with t
    qdir = Q.mean(dim=1, keepdim=True)
    ramp = torch.linspace(0.0, 1.0, S, device=DEV).view(1, S, 1)
    K = K + growth * ramp * qdir / (qdir.norm(dim=-1, keepdim=True) + 1e-6) * 8.0
    Q, K = Q.half(), K.half()
    V = rnd(B * nh, S, 64, dtype=torch.float16)
    out = torch.empty(B, S, nh * 64, device=DEV, dtype=torch.bfloat16)
    err = torch.zeros(1, device=DEV, dtype=torch.int32)
    tsd.op_attention(Q, K, V, B, nh, S, out, nh * 64, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = ref_attention(Q, K, V, B, nh, S)
    assert torch.isfinite(out.float()).all()
    assert rel(out.float(), ref) < 4e-3


@pytest.mark.parametrize("per_token", [1, 0])
def test_ln_modulate(per_token):
    rows_per_item, nb, H = 50, 3, 384
    rows = rows_per_item * nb
    x = 3.0 * torch.randn(rows, H, device=DEV) + 1.0
    x[7] = 0.5                        # zero-variance row: eps decides
    nmod = rows if per_token else nb
    mod = torch.randn(nmod, 6 * H, device=DEV)
    y = torch.empty(rows, H, device=DEV, dtype=torch.bfloat16)
    tsd.op_ln_modulate(x, rows, H, mod[:, 0:], mod[:, H:], 6 * H, per_token, rows_per_item, y)
    torch.cuda.synchronize()
    idx = torch.arange(rows, device=DEV) if per_token else torch.arange(rows, device=DEV) // rows_per_item
    ln = torch.nn.functional.layer_norm(x, (H,), eps=1e-5)
    ref = ln * (1 + mod[idx, H:2 * H]) + mod[idx, :H]
    assert rel(y.float(), ref.to(torch.bfloat16).float()) < 1e-3


def test_qk_norm_rope():
    B, S, nh, Sj, off = 2, 40, 3, 100, 30
    H = nh * 64
    qkv = torch.randn(B, S, 3 * H, device=DEV)
    qg = 1 + 0.1 * torch.randn(64, device=DEV)
    kg = 1 + 0.1 * torch.randn(64, device=DEV)
    Q = torch.zeros(B * nh, Sj, 64, device=DEV, dtype=torch.float16)
    K, V = torch.zeros_like(Q), torch.zeros_like(Q)
    fs = 194.0 / 72.0
    tsd.op_qk_norm_rope(qkv, B, S, H, nh, qg, kg, 1, fs, 10000.0, Q, K, V, Sj, off)
    torch.cuda.synchronize()

    def ref(x, g):
        x = x.view(B, S, nh, 64)
        x = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * g
        i = torch.arange(32, device=DEV, dtype=torch.float32)
        ang = fs * (torch.arange(S, device=DEV, dtype=torch.float32)[:, None] * 10000.0 ** (-2 * i / 64))
        c, s = torch.cos(ang)[None, :, None], torch.sin(ang)[None, :, None]
        x0, x1 = x[..., 0::2], x[..., 1::2]
        return torch.stack([x0 * c - x1 * s, x0 * s + x1 * c], -1).view(B, S, nh, 64)

    def got(T):
        return T.view(B, nh, Sj, 64)[:, :, off:off + S].permute(0, 2, 1, 3).float()

    assert rel(got(Q), ref(qkv[..., :H], qg)) < 1e-3
    assert rel(got(K), ref(qkv[..., H:2 * H], kg)) < 1e-3
    assert rel(got(V), qkv[..., 2 * H:].reshape(B, S, nh, 64)) < 1e-3
    assert float(Q.view(B, nh, Sj, 64)[:, :, :off].abs().max()) == 0.0
