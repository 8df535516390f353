"""GPU parity of the whole MM-DiT velocity evaluation and sampler (through the C-ABI)
against the CPU oracle on the same seeded inputs and weights.

Tolerances: the reference's own parity bars (src/tools/dit_test.cpp:19-20 stage rel-L2 2e-3,
dit_sample.cpp:18 5e-3) and the target's rel-L2 <= 1e-3 per attention layer, <= 2e-3 per BF16
flow step, <= 1e-2 for Q8_0. The oracle runs in GGML-emulating mode (bf16 mul_mat operands,
f16 Q/K/V) — the rounding the reference applies with BF16 weights.
"""
import os

import numpy as np
import pytest

from tsd_b200 import synth, tsd
import oracle

pytestmark = pytest.mark.gpu

SMALL = dict(hidden=128, n_head=2, depth=3, fused_depth=1, ffn=256)
SHAPE = dict(T=20, clip_S=8, sync_S=24, text_S=77, t5_S=9)


def bf16_round(a):
    return synth.bf16_bits_to_f32(synth.f32_to_bf16_bits(np.asarray(a, np.float32)))


@pytest.fixture(scope="module")
def small_bf16():
    hp = synth.DitHParams(**SMALL)
    W = synth.make_weights(hp, seed=1234, wtype="bf16")
    return hp, W, tsd.DitModel.from_weights(hp, W), oracle.OracleModel(hp, W)


STAGES = ("x_in", "t_emb", "clip_pp", "text_pp", "clip_fc", "text_fc", "gcmlp", "global_c", "extended_c", "text_xn",
          "a0_q", "a0_k", "a0_v", "a0_out", "jb0_lat", "jb0_clip", "jb0_text", "after_joint", "after_fused", "flow_cl")
BF16_STAGES = ("text_xn", "a0_out")   # stored bf16 on the GPU: the precision their consumer GEMM reads


def check_stages(dg, b, nb, x, hp, W, om, factor=2.5, floor_min=1e-3):
    """Per-stage parity with a measured noise floor.

    The reference rounds every mul_mat operand to bf16; two correct implementations of that
    arithmetic (the C++ oracle and the PyTorch emulation) already differ because 1e-7-level
    accumulation-order differences flip bf16 roundings, and the flips compound over the blocks.
    Each stage must be within `factor` x that floor (at least `floor_min`) of the oracle, and at
    least as close to the exact-f32 restatement as the reference arithmetic itself is.
    """
    import torch
    import torch_ref
    fo, do = om.forward(x, mode=oracle.MODE_GGML, dbg=True)
    fe, de = om.forward(x, mode=oracle.MODE_EXACT, dbg=True)
    dt = {}
    torch_ref.TorchDiT(hp, W, dtype=torch.float32, emulate=True).forward(x, dbg=dt)
    report = {}
    for name in STAGES:
        g = dg[name].reshape(nb, -1)[b]
        o, e, t = do[name], de[name], dt[name]
        if name in BF16_STAGES:
            o, t = bf16_round(o), bf16_round(t)
        floor = max(floor_min, oracle.rel_l2(t, o))
        err = oracle.rel_l2(g, o)
        report[name] = (err, floor)
        assert err <= factor * floor, (name, err, floor)
        if name not in BF16_STAGES and name != "t_emb":
            assert oracle.rel_l2(g, e) <= 1.1 * oracle.rel_l2(o, e) + 5e-4, (name, oracle.rel_l2(g, e), oracle.rel_l2(o, e))
    return report


def test_forward_stages_match_oracle(small_bf16):
    hp, W, m, om = small_bf16
    items = synth.make_inputs(hp, seed=4242, batch=2, **SHAPE)
    flow, dg = m.forward(items, dbg=True)
    for b, x in enumerate(items):
        check_stages(dg, b, 2, x, hp, W, om)
        assert oracle.rel_l2(flow[b], om.forward(x, mode=oracle.MODE_GGML)) < 5e-3


@pytest.mark.parametrize("wtype,tol", [("f32", 1e-2), ("q8_0", 1e-2)])
def test_forward_weight_types(wtype, tol):
    """F32 projection weights run as bf16 on the tensor cores (activations bf16, f32 accumulate);
    Q8_0 weights are dequantised exactly (q * fp16 scale) before the bf16 tensor-core path."""
    hp = synth.DitHParams(**SMALL)
    W = synth.make_weights(hp, seed=99, wtype=wtype)
    items = synth.make_inputs(hp, seed=5, batch=1, **SHAPE)
    m = tsd.DitModel.from_weights(hp, W)
    flow = m.forward(items)
    om = oracle.OracleModel(hp, W)
    assert oracle.rel_l2(flow[0], om.forward(items[0], mode=oracle.MODE_GGML)) < tol
    assert oracle.rel_l2(flow[0], om.forward(items[0], mode=oracle.MODE_EXACT)) < tol


@pytest.mark.parametrize("hidden,heads", [(128, 2), (256, 4)])
def test_q8_gemm_dequantises_in_kernel_bit_identically(monkeypatch, hidden, heads):
    """Planar Q8_0 projections are dequantised in shared memory by the GEMM's converter warps
    (w = q * scale rounded to bf16); the result must equal the load-time bf16 widening exactly."""
    hp = synth.DitHParams(hidden=hidden, n_head=heads, depth=3, fused_depth=1, ffn=2 * hidden)
    W = synth.make_weights(hp, seed=31, wtype="q8_0")
    items = synth.make_inputs(hp, seed=6, batch=2, **SHAPE)
    monkeypatch.setenv("TSD_Q8_IN_KERNEL", "1")
    in_kernel = tsd.DitModel.from_weights(hp, W).forward(items)
    monkeypatch.delenv("TSD_Q8_IN_KERNEL")
    at_load = tsd.DitModel.from_weights(hp, W).forward(items)
    assert np.isfinite(in_kernel).all()
    assert np.array_equal(in_kernel, at_load)


def test_forward_from_gguf_equals_from_weights(tmp_path, small_bf16):
    hp, W, m, _ = small_bf16
    path = str(tmp_path / "dit.gguf")
    synth.write_gguf(path, hp, W)
    m2 = tsd.DitModel.load(path)
    assert m2.hparams.hidden == hp.hidden and m2.hparams.depth == hp.depth
    items = synth.make_inputs(hp, seed=77, batch=1, **SHAPE)
    a, b = m.forward(items), m2.forward(items)
    assert oracle.rel_l2(a, b) < 1e-5
    es = m2.get_tensor("empty_string_feat")
    assert np.array_equal(es, W["empty_string_feat"].dequant())


def test_batched_equals_single(small_bf16):
    """Batch items are independent; a different batch size may tile the GEMMs (and order the
    f32 sums) differently, so agreement is at the bf16 rounding-noise level, while repeating
    the same call is bit-exact."""
    hp, W, m, _ = small_bf16
    items = synth.make_inputs(hp, seed=31, batch=3, **SHAPE)
    fb = m.forward(items)
    assert np.array_equal(fb, m.forward(items))
    for b in range(3):
        fs = m.forward([items[b]])
        assert oracle.rel_l2(fb[b], fs[0]) < 3e-3


def test_sampler_matches_oracle(small_bf16):
    hp, W, m, om = small_bf16
    x = synth.make_inputs(hp, seed=4242, batch=1, **SHAPE)[0]
    lat, f0 = m.sample([x], steps=3, cfg=5.0, want_flow0=True)
    lo, fo = om.sample(x, steps=3, cfg=5.0, mode=oracle.MODE_GGML, want_flow0=True)
    le, fe = om.sample(x, steps=3, cfg=5.0, mode=oracle.MODE_EXACT, want_flow0=True)
    # CFG 5 amplifies the cond/uncond rounding noise five-fold in the velocity
    assert oracle.rel_l2(f0[0], fo) < 1.5e-2 and oracle.rel_l2(lat[0], lo) < 1e-2
    assert oracle.rel_l2(f0[0], fe) <= 1.2 * oracle.rel_l2(fo, fe) + 2e-3
    assert oracle.rel_l2(lat[0], le) <= 1.2 * oracle.rel_l2(lo, le) + 2e-3


def test_sampler_batched_prompts(small_bf16):
    hp, W, m, _ = small_bf16
    items = synth.make_inputs(hp, seed=8, batch=3, **SHAPE)
    lat = m.sample(items, steps=2, cfg=5.0)
    assert np.array_equal(lat, m.sample(items, steps=2, cfg=5.0))
    for p in range(3):
        single = m.sample([items[p]], steps=2, cfg=5.0)
        assert oracle.rel_l2(lat[p], single[0]) < 1e-2


def test_sampler_step_loop_equals_forward_calls(small_bf16):
    """After step 0 the sampler replays the forward without its conditioning-only ops (clip /
    sync / text projections, global MLP) and reuses their step-0 results. Stepping by hand with
    full forward calls of the same cond / uncond pair (mmdit.cpp:344-376) must give the same
    latent, up to the rounding of the CFG + Euler update done here in numpy."""
    import dataclasses
    hp, W, m, _ = small_bf16
    x = synth.make_inputs(hp, seed=77, batch=1, **SHAPE)[0]
    steps, cfg = 4, 5.0
    lat = m.sample([x], steps=steps, cfg=cfg)[0]
    es = W["empty_string_feat"].dequant().reshape(-1, hp.text_dim)[:SHAPE["text_S"]]
    et = W["empty_t5_feat"].dequant().reshape(-1, hp.t5_dim)[:SHAPE["t5_S"]]
    cur = np.asarray(x.latent, np.float32).copy()
    for s in range(steps):
        tc, tp = np.float32(1 - s / steps), np.float32(1 - (s + 1) / steps)
        cond = dataclasses.replace(x, latent=cur, t=float(tc))
        unc = dataclasses.replace(x, latent=cur, text_f=es, t5=et, gtext=np.zeros_like(x.gtext), t=float(tc))
        fc, fu = m.forward([cond, unc])
        cur = cur + (tp - tc) * (fu + (fc - fu) * np.float32(cfg)).T
    assert oracle.rel_l2(lat, cur) < 1e-5
    # a second prompt through the same plan recomputes its own conditioning at step 0
    y = synth.make_inputs(hp, seed=78, batch=1, **SHAPE)[0]
    m.sample([x], steps=2, cfg=cfg)
    assert np.array_equal(m.sample([y], steps=2, cfg=cfg), m.sample([y], steps=2, cfg=cfg))
    assert oracle.rel_l2(m.sample([y], steps=2, cfg=cfg)[0], m.sample([x], steps=2, cfg=cfg)[0]) > 1e-3


def test_bad_shapes_are_rejected(small_bf16):
    hp, W, m, _ = small_bf16
    items = synth.make_inputs(hp, seed=1, batch=1, T=20, clip_S=8, sync_S=20, text_S=77, t5_S=9)  # sync_S % 8 != 0
    with pytest.raises(tsd.TsdError) as e:
        m.forward(items)
    assert e.value.rc == -1


def test_reference_model_width_h1024(tmp_path):
    """The reference's own thinksound_light widths: hidden 1024, 16 heads, FFN 2816."""
    hp = synth.DitHParams(hidden=1024, n_head=16, depth=2, fused_depth=1)
    assert hp.ffn == 2816
    W = synth.make_weights(hp, seed=2, wtype="bf16")
    items = synth.make_inputs(hp, seed=3, batch=1, T=44, clip_S=16, sync_S=48, text_S=77, t5_S=77)
    m = tsd.DitModel.from_weights(hp, W)
    flow, dg = m.forward(items, dbg=True)
    check_stages(dg, 0, 1, items[0], hp, W, oracle.OracleModel(hp, W))


def test_cfg1_joint_layer_shapes_h1536():
    """BASELINE config 1 shapes (H=1536, 24x64 heads, T=194, clip 72, text 77+128, joint S=471)
    through a model with one full joint block, per-stage against the oracle."""
    hp = synth.DitHParams(hidden=1536, n_head=24, depth=3, fused_depth=1)
    W = synth.make_weights(hp, seed=1234, wtype="bf16")
    items = synth.make_inputs(hp, seed=4242, batch=2, T=194, clip_S=72, sync_S=216, text_S=77, t5_S=128)
    m = tsd.DitModel.from_weights(hp, W)
    flow, dg = m.forward(items, dbg=True)
    rep = check_stages(dg, 0, 2, items[0], hp, W, oracle.OracleModel(hp, W))
    print({k: f"{e:.2e}/{f:.2e}" for k, (e, f) in rep.items()})
    m.close()


def test_ts_dit_shim_drop_in(tmp_path, small_bf16):
    """include/ts_dit.hpp (the mmdit.h drop-in) gives the same flow and latent as the C-ABI."""
    import subprocess
    from test_capi import build_shim_demo
    hp, W, m, _ = small_bf16
    path = str(tmp_path / "dit.gguf")
    synth.write_gguf(path, hp, W)
    exe = build_shim_demo(tmp_path)
    T, cS, yS, steps = 20, 8, 24, 2
    out = str(tmp_path / "out.bin")
    r = subprocess.run([exe, path, str(T), str(cS), str(yS), str(steps), out], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    for name in ("x_in", "a0_q", "a0_out", "after_joint", "after_fused", "flow_cl"):
        assert name in r.stdout
    data = np.fromfile(out, np.float32)
    flow_c, lat_c = data[:T * 64].reshape(T, 64), data[T * 64:].reshape(64, T)
    f32 = lambda a: np.asarray(a, np.float64).astype(np.float32)
    noise = f32(np.sin(0.37 * np.arange(64 * T))).reshape(64, T)
    text = f32(np.cos(0.11 * np.arange(77 * 1024))).reshape(77, 1024)
    t5 = f32(np.sin(0.05 * np.arange(77 * 2048) + 1.0)).reshape(77, 2048)
    gt = f32(np.cos(0.7 * np.arange(1024)))
    clip = np.tile(W["empty_clip_feat"].dequant().reshape(1, 1024), (cS, 1))
    sync = np.tile(W["empty_sync_feat"].dequant().reshape(1, 768), (yS, 1))
    item = synth.DitInputs(noise, clip, sync, text, t5, gt, 1.0)
    assert oracle.rel_l2(flow_c, m.forward([item])[0]) < 1e-5
    assert oracle.rel_l2(lat_c, m.sample([item], steps=steps, cfg=5.0)[0]) < 1e-5


def test_cfg4_q8_30s_shapes_h1536():
    """BASELINE config 4 shapes (30 s: T=646, clip 240, sync 720, T5 512; joint S=1475) with Q8_0
    weights, B=2, through a truncated model (2 joint + 1 fused blocks at H=1536, 24x64 heads).
    With Q8_0 weights the reference's CPU arithmetic quantises every mul_mat activation to
    Q8_0 blocks; that alone puts it ~1.4e-2 (rel-L2) from the exact restatement at these shapes,
    and the GPU path (bf16 activations, Q8_0 weights widened exactly and rounded to bf16) cannot
    reproduce that rounding. So each stage must be at least as close to the exact restatement as
    the reference arithmetic is, and within the Q8_0 bar (1e-2) plus that arithmetic's own
    distance from exact of the oracle's GGML-emulating output.

    The weights are the Q8_0 quantisation of N(0, 0.02^2) draws. Config 4's timing weights
    (random blocks: int8 ~U[-127,127] x fp16 scale ~U[1e-4,4e-3], ~7x larger) drive the
    activations past the f16 range the reference casts V to (V reaches ~1e9 in the first joint
    block), so the reference arithmetic itself yields inf/NaN there; they are used for timing
    only."""
    hp = synth.DitHParams(hidden=1536, n_head=24, depth=3, fused_depth=1)
    W = synth.make_weights(hp, seed=1234, wtype="q8_0")
    shape = dict(T=646, clip_S=240, sync_S=720, text_S=77, t5_S=512)
    items = synth.make_inputs(hp, seed=4242, batch=2, **shape)
    m = tsd.DitModel.from_weights(hp, W)
    flow, dg = m.forward(items, dbg=True)
    m.close()
    om = oracle.OracleModel(hp, W)
    fo, do = om.forward(items[0], mode=oracle.MODE_GGML, dbg=True)
    fe, de = om.forward(items[0], mode=oracle.MODE_EXACT, dbg=True)
    for name in ("a0_q", "a0_k", "a0_v", "a0_out", "jb0_lat", "jb0_text", "after_joint", "after_fused", "flow_cl"):
        g = dg[name].reshape(2, -1)[0]
        o, e = do[name], de[name]
        if name in BF16_STAGES:
            o, e = bf16_round(o), bf16_round(e)
        d_go, d_ge, d_oe = oracle.rel_l2(g, o), oracle.rel_l2(g, e), oracle.rel_l2(o, e)
        print(f"{name}: GPU vs GGML arithmetic {d_go:.2e}, GPU vs exact {d_ge:.2e}, GGML arithmetic vs exact {d_oe:.2e}")
        assert d_ge <= 1.2 * d_oe + 2e-3, (name, d_ge, d_oe)
        assert d_go <= 1e-2 + d_oe, (name, d_go, d_oe)
    fe1 = om.forward(items[1], mode=oracle.MODE_EXACT)
    fo1 = om.forward(items[1], mode=oracle.MODE_GGML)
    assert oracle.rel_l2(flow[1], fe1) <= 1.2 * oracle.rel_l2(fo1, fe1) + 2e-3


def test_many_item_batch_conditioning_gemms(small_bf16):
    """With more than 8 items the few-token projections (timestep MLP, conditioning projections,
    the stacked clip / text adaLN) run on the tensor-core GEMM instead of the GEMV; every item
    must still match its single-item forward and the oracle."""
    hp, W, m, om = small_bf16
    items = synth.make_inputs(hp, seed=91, batch=10, **SHAPE)
    fb = m.forward(items)
    for b in (0, 9):
        assert oracle.rel_l2(fb[b], m.forward([items[b]])[0]) < 3e-3
    fo = om.forward(items[9], mode=oracle.MODE_GGML)
    fe = om.forward(items[9], mode=oracle.MODE_EXACT)
    assert oracle.rel_l2(fb[9], fo) < 5e-3
    assert oracle.rel_l2(fb[9], fe) <= 1.2 * oracle.rel_l2(fo, fe) + 1e-3


@pytest.mark.parametrize("pair", [0, 1])
def test_multi_item_tiles_in_the_forward(monkeypatch, small_bf16, pair):
    """Every GEMM over short items (here the 20-token latent and 8-token clip streams) forced onto
    tiles that hold several batch items (pair = 1: on CTA pairs where the tiling allows): a
    5-item batch, whose last tile is partly empty, matches the oracle item by item and the same
    model's default tiling."""
    hp, W, m, om = small_bf16
    items = synth.make_inputs(hp, seed=77, batch=5, **SHAPE)
    ref = m.forward(items)
    monkeypatch.setenv("TSD_FORCE_MULTI_ITEM", "1")
    if pair:
        monkeypatch.setenv("TSD_FORCE_PAIR", "1")
    mf = tsd.DitModel.from_weights(hp, W)
    try:
        fm = mf.forward(items)
    finally:
        mf.close()
    for b in (0, 4):
        assert oracle.rel_l2(fm[b], ref[b]) < 3e-3
        assert oracle.rel_l2(fm[b], om.forward(items[b], mode=oracle.MODE_GGML)) < 5e-3


def test_ts_server_keeps_the_dit_resident(tmp_path, small_bf16):
    """tests/shim/ts_server_demo.cpp: the DiT part of ts-server's request path with the model
    loaded once and reused by every request (the reference reloads it per request,
    ts-server.cpp:74). Four requests over two input shapes: one load, and every request's
    latent equals a fresh model's sample of the same inputs."""
    import subprocess
    hp, W, m, _ = small_bf16
    path = str(tmp_path / "dit.gguf")
    synth.write_gguf(path, hp, W)
    libdir = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "thinksound.cpp_b200")
    incdir = os.path.join(os.path.dirname(libdir), "include")
    src = os.path.join(os.path.dirname(os.path.abspath(__file__)), "shim", "ts_server_demo.cpp")
    exe = str(tmp_path / "ts_server_demo")
    subprocess.run(["g++", "-std=c++17", "-O1", "-I", incdir, src, "-o", exe, "-L", libdir, "-ltsd_b200",
                    f"-Wl,-rpath,{libdir}"], check=True)
    reqs = [(20, 0.0), (20, 1.5), (40, 0.25), (20, 3.0)]
    out = str(tmp_path / "lat.bin")
    r = subprocess.run([exe, path, "2", out] + [f"{T}:{s}" for T, s in reqs], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    assert "loads=1" in r.stdout, r.stdout
    print(r.stdout)
    data = np.fromfile(out, np.float32)
    fresh = tsd.DitModel.load(path)
    off = 0
    for T, seed in reqs:
        lat = data[off:off + 64 * T].reshape(64, T)
        off += 64 * T
        i = np.arange
        f32 = lambda a: np.asarray(a, np.float64).astype(np.float32)
        cS, yS = 8 * ((T + 19) // 20), 24 * ((T + 19) // 20)
        noise = f32(np.sin(0.37 * i(64 * T) + seed)).reshape(64, T)
        text = f32(np.cos(0.11 * i(77 * 1024) + seed)).reshape(77, 1024)
        t5 = f32(np.sin(0.05 * i(77 * 2048) + 1.0 + seed)).reshape(77, 2048)
        gt = f32(np.cos(0.7 * i(1024) + seed))
        clip = np.tile(W["empty_clip_feat"].dequant().reshape(1, 1024), (cS, 1))
        sync = np.tile(W["empty_sync_feat"].dequant().reshape(1, 768), (yS, 1))
        ref = fresh.sample([synth.DitInputs(noise, clip, sync, text, t5, gt, 1.0)], steps=2, cfg=5.0)[0]
        assert oracle.rel_l2(lat, ref) < 1e-5, (T, seed)
    fresh.close()
