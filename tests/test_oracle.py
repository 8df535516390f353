"""CPU tests of the oracle (the checker the CUDA path is compared against).

The reference ships no golden vectors (its golden GGUFs were never committed), so the oracle is
pinned two ways: against an independent PyTorch restatement of src/mmdit.cpp
(tests/torch_ref.py) and against the committed fixtures in tests/golden/ (regression pin).
"""
import os

import numpy as np
import pytest
import torch

from tsd_b200 import synth
import oracle
import torch_ref

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "dit_small.npz")
HP = dict(hidden=128, n_head=2, depth=3, fused_depth=1, ffn=256)
SHAPE = dict(T=20, clip_S=8, sync_S=24, text_S=77, t5_S=9)


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


@pytest.mark.parametrize("wtype", ["f32", "bf16", "q8_0"])
def test_oracle_exact_matches_torch_restatement(wtype):
    hp = synth.DitHParams(**HP)
    W = synth.make_weights(hp, seed=7, wtype=wtype)
    x = synth.make_inputs(hp, seed=8, **SHAPE)[0]
    fo, do = oracle.OracleModel(hp, W).forward(x, mode=oracle.MODE_EXACT, dbg=True)
    dt = {}
    ft = torch_ref.TorchDiT(hp, W, dtype=torch.float64).forward(x, dbg=dt)
    assert oracle.rel_l2(fo, ft) < 2e-5
    for k in ("x_in", "t_emb", "clip_pp", "text_pp", "extended_c", "a0_q", "a0_k", "a0_v", "a0_out", "jb0_lat",
              "jb0_clip", "jb0_text", "after_joint", "after_fused"):
        assert oracle.rel_l2(do[k], dt[k]) < 2e-5, k


def test_oracle_ggml_mode_matches_torch_emulation():
    """Both restatements round at the reference's points (bf16 mul_mat operands, f16 Q/K/V)."""
    hp = synth.DitHParams(**HP)
    W = synth.make_weights(hp, seed=7, wtype="bf16")
    x = synth.make_inputs(hp, seed=8, **SHAPE)[0]
    fo, do = oracle.OracleModel(hp, W).forward(x, mode=oracle.MODE_GGML, dbg=True)
    dt = {}
    ft = torch_ref.TorchDiT(hp, W, dtype=torch.float32, emulate=True).forward(x, dbg=dt)
    # rounding-boundary flips between two f32 implementations compound over the blocks
    assert oracle.rel_l2(do["a0_out"], dt["a0_out"]) < 1e-3
    assert oracle.rel_l2(fo, ft) < 5e-3


def test_golden_fixtures_reproduce(golden):
    hp = synth.DitHParams(**HP)
    for wtype in ("bf16", "q8_0", "f32"):
        W = synth.make_weights(hp, seed=1234, wtype=wtype)
        x = synth.make_inputs(hp, seed=4242, **SHAPE)[0]
        om = oracle.OracleModel(hp, W)
        fg, dg = om.forward(x, mode=oracle.MODE_GGML, dbg=True)
        fe = om.forward(x, mode=oracle.MODE_EXACT)
        assert oracle.rel_l2(fg, golden[f"{wtype}/flow_ggml"]) < 1e-5, wtype
        assert oracle.rel_l2(fe, golden[f"{wtype}/flow_exact"]) < 1e-5, wtype
        if wtype == "bf16":
            for k in ("a0_q", "a0_out", "after_joint", "after_fused", "flow_cl"):
                assert oracle.rel_l2(dg[k], golden[f"bf16/stage/{k}"]) < 1e-5, k


def test_golden_sampler(golden):
    hp = synth.DitHParams(**HP)
    W = synth.make_weights(hp, seed=1234, wtype="bf16")
    x = synth.make_inputs(hp, seed=4242, **SHAPE)[0]
    lat, f0 = oracle.OracleModel(hp, W).sample(x, steps=3, cfg=5.0, mode=oracle.MODE_GGML, want_flow0=True)
    assert oracle.rel_l2(lat, golden["bf16/sample3_latent"]) < 1e-5
    assert oracle.rel_l2(f0, golden["bf16/sample3_flow0"]) < 1e-5


def test_sampler_is_euler_cfg_of_forward():
    """sample() == hand-rolled Euler + CFG over forward() (mmdit.cpp:359-375)."""
    hp = synth.DitHParams(**HP)
    W = synth.make_weights(hp, seed=3, wtype="f32")
    x = synth.make_inputs(hp, seed=5, **SHAPE)[0]
    om = oracle.OracleModel(hp, W)
    steps, cfg = 2, 3.0
    lat = om.sample(x, steps=steps, cfg=cfg, mode=oracle.MODE_EXACT)
    cur = x.latent.copy()
    es = W["empty_string_feat"].dequant()
    et = W["empty_t5_feat"].dequant()[: SHAPE["t5_S"]]
    for s in range(steps):
        t = 1.0 - s / steps
        dt = (1.0 - (s + 1) / steps) - t
        xc = synth.DitInputs(cur, x.clip_f, x.sync_f, x.text_f, x.t5, x.gtext, t)
        xu = synth.DitInputs(cur, x.clip_f, x.sync_f, es, et, np.zeros_like(x.gtext), t)
        fc = om.forward(xc, mode=oracle.MODE_EXACT)
        fu = om.forward(xu, mode=oracle.MODE_EXACT)
        v = (fu + (fc - fu) * cfg).T      # [T][L] -> [L][T]
        cur = cur + dt * v
    assert oracle.rel_l2(lat, cur) < 1e-6


def test_zero_variance_tokens_use_layernorm_eps_1e5():
    """Padding-like constant rows (zero variance): LayerNorm eps 1e-5 (docs/PROGRESS.md:40)."""
    hp = synth.DitHParams(**HP)
    W = synth.make_weights(hp, seed=11, wtype="f32")
    x = synth.make_inputs(hp, seed=12, **SHAPE)[0]
    x.text_f[40:] = 0.25            # constant MetaCLIP rows, like padded text features
    x.t5[:] = 0.0
    fo = oracle.OracleModel(hp, W).forward(x, mode=oracle.MODE_EXACT)
    ft = torch_ref.TorchDiT(hp, W, dtype=torch.float64).forward(x)
    assert oracle.rel_l2(fo, ft) < 2e-5


def test_rope_is_interleaved_pairs():
    """NORMAL-mode RoPE rotates adjacent pairs (2i, 2i+1) by pos * fs * theta^(-2i/64)."""
    hp = synth.DitHParams(**HP)
    ref = torch_ref.TorchDiT(hp, synth.make_weights(hp, seed=1, wtype="f32"), dtype=torch.float64)
    x = torch.randn(1, 1, 5, 64, dtype=torch.float64)
    y = ref.apply_rope(x, ref.rope_rot(5, 0.5))
    for n in range(5):
        for i in range(32):
            th = 0.5 * n * 10000.0 ** (-2 * i / 64)
            x0, x1 = x[0, 0, n, 2 * i].item(), x[0, 0, n, 2 * i + 1].item()
            assert abs(y[0, 0, n, 2 * i].item() - (x0 * np.cos(th) - x1 * np.sin(th))) < 1e-12
            assert abs(y[0, 0, n, 2 * i + 1].item() - (x0 * np.sin(th) + x1 * np.cos(th))) < 1e-12


def test_q8_0_round_trip_matches_gguf_py():
    """Our Q8_0 block writer agrees with gguf-py's reference quantiser."""
    import gguf
    from gguf import quants
    a = (0.02 * np.random.default_rng(0).standard_normal((4, 64))).astype(np.float32)
    ours = synth.quantize_q8_0(a)
    theirs = quants.quantize(a, gguf.GGMLQuantizationType.Q8_0)
    assert ours.shape == theirs.shape
    qa = synth.WTensor("w", (64, 4), synth.GGML_Q8_0, ours).dequant()
    qb = synth.WTensor("w", (64, 4), synth.GGML_Q8_0, np.asarray(theirs)).dequant()
    assert np.max(np.abs(qa - qb)) <= 1e-6 + 1e-3 * np.max(np.abs(a))
