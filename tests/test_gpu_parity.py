"""Parity of the GPU path with the CPU oracle at the north-star bars, config by config.

(a) Attention alone (config 1 shapes: B=2, 24 heads x 64, joint S = 194 + 72 + 205 = 471): the
    oracle's Q / K / V of the first joint block, rounded to f16 as the reference casts them
    (src/mmdit.cpp:88-90), through the tcgen05 attention kernel; rel-L2 <= 1e-3 against the
    oracle's attention output (f32-output form of the kernel, so that bf16 output rounding,
    itself ~1.1e-3, does not mask the kernel's own error).
(b) Every block teacher-forced (the full model: 7 joint + 14 fused blocks at H=1536, config-3
    shapes, B=2): each block starts from the oracle's input to that block and the oracle's
    conditioning vectors (tsd_forward_inject), so per-block error is measured without
    compounding:
      - the attention half of each block (QKV projection with QK-norm / RoPE, joint attention,
        out-projection, gate): rel-L2 of its residual increment <= 1e-3 (the per attention
        layer bar; this increment is config 1's "per-stream attention output after out-proj");
      - the block's output residual stream: rel-L2 <= 2e-3;
      - the final layer from the oracle's last residual: rel-L2 <= 2e-3.
    Blocks 7-20 are config 2's stack of 14 fused blocks.
(c) The free-running full forward (config 3) against the oracle's GGML-emulating and exact
    restatements: the GPU must be at least as close to the exact restatement as the reference
    arithmetic itself is, and the measured gaps are printed.

The oracle runs in GGML-emulating mode (every mul_mat activation rounded to bf16, Q/K/V to f16):
the arithmetic the reference performs with BF16 weights.
"""
import numpy as np
import pytest

from tsd_b200 import synth, tsd
import oracle

pytestmark = pytest.mark.gpu

CFG3 = dict(T=194, clip_S=72, sync_S=216, text_S=77, t5_S=128)
STREAMS = ("lat", "clip", "text")


def rel(a, b):
    return oracle.rel_l2(np.asarray(a, np.float32).reshape(-1), np.asarray(b, np.float32).reshape(-1))


def bf16_round(a):
    return synth.bf16_bits_to_f32(synth.f32_to_bf16_bits(np.asarray(a, np.float32)))


def make_weights_gpu_rng(hp, seed):
    """Seeded BF16-GGUF weights drawn with torch's GPU generator (seconds for the full model,
    where numpy takes minutes), returned as host synth.WTensors for both the GPU model and the
    oracle. Same storage types and distributions as synth.make_weights."""
    import torch
    g = torch.Generator(device="cuda:0")
    g.manual_seed(seed)
    out = {}
    for name, ne, kind in synth.tensor_specs(hp):
        shp = tuple(reversed(ne))
        t = synth.storage_type(name, ne, "bf16")
        if kind == "zeros":
            a = torch.zeros(shp, device="cuda:0")
        elif kind == "gain":
            a = 1.0 + 0.1 * torch.randn(shp, generator=g, device="cuda:0")
        elif kind == "emb":
            a = torch.randn(shp, generator=g, device="cuda:0")
        else:
            a = 0.02 * torch.randn(shp, generator=g, device="cuda:0")
        if t == synth.GGML_BF16:
            data = a.to(torch.bfloat16).view(torch.int16).cpu().numpy().view(np.uint16)
        else:
            data = a.float().cpu().numpy()
        out[name] = synth.WTensor(name, ne, t, data)
    return out


# ------------------------------------------------------------------------------------- (a)
def head_major_f16(x, nh):
    """[S][H] (column d + 64 h) -> [nh][S][64] float16."""
    S = x.shape[0]
    return np.ascontiguousarray(np.asarray(x, np.float32).reshape(S, nh, 64).transpose(1, 0, 2)).astype(np.float16)


def test_attention_cfg1_isolated_within_1e3():
    import torch
    hp = synth.DitHParams(hidden=1536, n_head=24, depth=3, fused_depth=1)
    W = synth.make_weights(hp, seed=1234, wtype="bf16")
    om = oracle.OracleModel(hp, W)
    items = synth.make_inputs(hp, seed=4242, batch=2, T=194, clip_S=72, sync_S=216, text_S=77, t5_S=128)
    S = 194 + 72 + 205
    stages = [om.forward(x, mode=oracle.MODE_GGML, dbg=True)[1] for x in items]
    nh, B = hp.n_head, len(items)
    Q, K, V = (torch.from_numpy(np.stack([head_major_f16(d[n].reshape(S, -1), nh) for d in stages])).cuda()
               .reshape(B * nh, S, 64) for n in ("a0_q", "a0_k", "a0_v"))
    out32 = torch.zeros(B, S, hp.hidden, device="cuda:0")
    out16 = torch.zeros(B, S, hp.hidden, device="cuda:0", dtype=torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    tsd.op_attention_f32(Q, K, V, B, nh, S, out32, hp.hidden, err=err)
    tsd.op_attention(Q, K, V, B, nh, S, out16, hp.hidden, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    for b, d in enumerate(stages):
        ref = d["a0_out"].reshape(S, -1)
        e32 = rel(out32[b].cpu().numpy(), ref)
        e16 = rel(out16[b].float().cpu().numpy(), bf16_round(ref))
        print(f"attention cfg1 item {b}: f32 output {e32:.2e}; bf16 output vs bf16-rounded oracle {e16:.2e}")
        assert e32 <= 1e-3, e32
        assert e16 <= 2e-3, e16


# ------------------------------------------------------------------------------------- (b), (c)
@pytest.fixture(scope="module")
def full_model():
    hp = synth.DitHParams(hidden=1536, n_head=24, depth=21, fused_depth=14, text_seq=77, t5_seq=128)
    W = make_weights_gpu_rng(hp, seed=1234)
    m = tsd.DitModel.from_weights(hp, W)
    om = oracle.OracleModel(hp, W)
    del W
    items = synth.make_inputs(hp, seed=4242, batch=2, **CFG3)
    ggml = [om.forward(x, mode=oracle.MODE_GGML, dbg=True) for x in items]
    yield hp, m, om, items, ggml
    m.close()


def forced_inputs(hp, ggml, mid=False):
    """Injection map: every block's input streams (and with `mid`, the stream entering each
    block's FFN half) and the conditioning vectors, from the oracle's run of each item."""
    nj, depth = hp.depth - hp.fused_depth, hp.depth
    first = {"lat": "x_in", "clip": "clip_pp", "text": "text_pp"}
    inject = {}
    for i in range(depth):
        for s in (STREAMS if i < nj else ("lat",)):
            src = first[s] if i == 0 else f"blk{i - 1}_{s}"
            inject[f"blk{i}_in_{s}"] = np.stack([g[1][src] for g in ggml])
            if mid and not (i == nj - 1 and s != "lat"):
                inject[f"blk{i}_mid_{s}"] = np.stack([g[1][f"blk{i}_attn_{s}"] for g in ggml])
    inject["final_in_lat"] = np.stack([g[1][f"blk{depth - 1}_lat"] for g in ggml])
    # the conditioning every block's adaLN projection reads (mmdit.cpp:196-200, 209)
    inject["global_c"] = np.stack([g[1]["global_c"] for g in ggml])
    inject["extended_c"] = np.stack([g[1]["extended_c"] for g in ggml])
    return inject


def block_errors(hp, ggml, inject, dg, mid):
    """(block, stream, item, attention increment, FFN increment, block output) rel-L2 rows."""
    nj, depth = hp.depth - hp.fused_depth, hp.depth
    rows = []
    for i in range(depth):
        for s in (STREAMS if i < nj else ("lat",)):
            if i == nj - 1 and s != "lat":
                continue                               # pre_only: the clip / text streams are not updated
            x_in = inject[f"blk{i}_in_{s}"]
            g_attn = dg[f"blk{i}_attn_{s}"].reshape(x_in.shape)
            g_out = dg[f"blk{i}_{s}"].reshape(x_in.shape)
            for b in range(x_in.shape[0]):
                o = ggml[b][1]
                o_attn = o[f"blk{i}_attn_{s}"].reshape(x_in[b].shape)
                o_out = o[f"blk{i}_{s}"].reshape(x_in[b].shape)
                f_in = o_attn if mid else g_attn[b]       # what the GPU's FFN half started from
                rows.append((i, s, b, rel(g_attn[b] - x_in[b], o_attn - x_in[b]),
                             rel(g_out[b] - f_in, o_out - o_attn), rel(g_out[b], o_out)))
    return rows


def print_rows(title, rows):
    print(title)
    print("block stream item | attention increment | FFN increment | block output (rel-L2)")
    for r in rows:
        print(f"{r[0]:5d} {r[1]:6s} {r[2]:4d} | {r[3]:.2e} | {r[4]:.2e} | {r[5]:.2e}")
    print(f"worst: attention increment {max(r[3] for r in rows):.2e}, FFN increment {max(r[4] for r in rows):.2e}, "
          f"block output {max(r[5] for r in rows):.2e}")


def test_every_block_teacher_forced(full_model):
    """Each block from the oracle's block input: the attention half (QKV with QK-norm / RoPE,
    joint attention, out-projection, gate) within 1e-3 for every block and stream. The FFN half
    then starts from the GPU's own post-attention stream, whose ~6e-4 difference the FFN's two
    bf16 roundings amplify (a value that differs by d flips its rounding with probability
    ~d / 2^-8, each flip worth 2^-8); the whole block is held to 3e-3 here and each half to the
    north-star bars in test_every_half_block_teacher_forced."""
    hp, m, om, items, ggml = full_model
    inject = forced_inputs(hp, ggml, mid=False)
    _, dg = m.forward_inject(items, inject)
    rows = block_errors(hp, ggml, inject, dg, mid=False)
    print_rows("teacher-forced at every block input", rows)
    B = len(items)
    for b in range(B):
        d_fin = rel(dg["flow_cl"].reshape(B, -1)[b], ggml[b][1]["flow_cl"])
        print(f"final layer (teacher-forced) item {b}: {d_fin:.2e}")
        assert d_fin <= 2e-3, d_fin
    bad = [r for r in rows if r[3] > 1e-3 or r[5] > 3e-3]
    assert not bad, bad[:8]


def test_every_half_block_teacher_forced(full_model):
    """Both halves of every block from the oracle's inputs (block input, and the stream entering
    the FFN half): attention increment <= 1e-3, FFN increment <= 1e-3, block output <= 2e-3."""
    hp, m, om, items, ggml = full_model
    inject = forced_inputs(hp, ggml, mid=True)
    _, dg = m.forward_inject(items, inject)
    rows = block_errors(hp, ggml, inject, dg, mid=True)
    print_rows("teacher-forced at every block input and before every FFN half", rows)
    bad = [r for r in rows if r[3] > 1e-3 or r[4] > 1e-3 or r[5] > 2e-3]
    assert not bad, bad[:8]


def test_full_depth_free_running(full_model):
    hp, m, om, items, ggml = full_model
    flow, dg = m.forward(items, dbg=True)
    B = len(items)
    for b, x in enumerate(items):
        fe, de = om.forward(x, mode=oracle.MODE_EXACT, dbg=True)
        do = ggml[b][1]
        for name in ("a0_out", "jb0_lat", "after_joint", "after_fused", "flow_cl"):
            g = dg[name].reshape(B, -1)[b]
            o, e = do[name], de[name]
            if name == "a0_out":
                o, e = bf16_round(o), bf16_round(e)
            d_go, d_ge, d_oe = rel(g, o), rel(g, e), rel(o, e)
            print(f"item {b} {name}: GPU vs reference arithmetic {d_go:.2e}; GPU vs exact {d_ge:.2e}; "
                  f"reference arithmetic vs exact {d_oe:.2e}")
            # as accurate as the reference's own BF16 arithmetic
            assert d_ge <= 1.1 * d_oe + 1e-3, (name, d_ge, d_oe)
        d = rel(flow[b], ggml[b][0])
        print(f"item {b} flow: GPU vs reference arithmetic {d:.2e}")
        assert d <= 3e-2, d
