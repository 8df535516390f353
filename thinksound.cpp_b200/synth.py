"""Synthetic MM-DiT weights and GGUF files with the reference's tensor schema.

The reference ships no checkpoint, so tests and the benchmark use random-initialised weights
with the exact tensor names, ggml shapes and per-tensor storage types of the reference's DiT
GGUF files:

* names and shapes: ``convert/convert_thinksound.py:36-52`` (checkpoint keys with the
  ``model.model.`` prefix stripped) as consumed by ``src/mmdit.cpp:150-290``;
* storage types: ``convert/quantize_gguf.py:11-15`` — BF16 files cast 2-D and 3-D weights
  except names containing ``norm``/``empty``/``_emb``; Q8_0 files quantise only 2-D weights
  whose ne0 is a multiple of 32 (conv weights stay F32).

Shapes are in ggml ``ne`` order (ne0 fastest); a numpy array holding a tensor has the reversed
shape. Matrices and biases are N(0, std^2) (std 0.02 by default), QK-norm gains 1 + 0.1 N(0,1),
``empty_t5_feat`` zeros (it is an untrained zero buffer upstream).
"""
from __future__ import annotations

import dataclasses
from typing import Dict, List, Optional, Tuple

import numpy as np

GGML_F32, GGML_F16, GGML_Q8_0, GGML_BF16 = 0, 1, 8, 30
TYPE_NAMES = {GGML_F32: "f32", GGML_F16: "f16", GGML_Q8_0: "q8_0", GGML_BF16: "bf16"}


def multiple_of(m: int, x: int) -> int:
    return m * ((x + m - 1) // m)


@dataclasses.dataclass
class DitHParams:
    hidden: int = 1536
    n_head: int = 24
    depth: int = 21
    fused_depth: int = 14
    latent_dim: int = 64
    ffn: int = 0                 # 0: SwiGLU width multiple_of(256, int(2 * 4 * hidden / 3))
    clip_dim: int = 1024
    sync_dim: int = 768
    text_dim: int = 1024         # MetaCLIP-text width (padded to t5_dim, mmdit.cpp:179)
    t5_dim: int = 2048
    text_seq: int = 77           # rows of empty_string_feat
    t5_seq: int = 77             # rows of empty_t5_feat
    rope_theta: float = 10000.0
    t_max_period: float = 1.0

    def __post_init__(self):
        if not self.ffn:
            self.ffn = multiple_of(256, int(2 * 4 * self.hidden / 3))

    @property
    def head_dim(self) -> int:
        return self.hidden // self.n_head

    @property
    def n_joint(self) -> int:
        return self.depth - self.fused_depth


# (name, ne, kind) with kind in {"mat", "conv", "bias", "gain", "emb", "zeros"}
Spec = Tuple[str, Tuple[int, ...], str]


def tensor_specs(hp: DitHParams) -> List[Spec]:
    H, F, L = hp.hidden, hp.ffn, hp.latent_dim
    hd = hp.head_dim
    s: List[Spec] = []

    def lin(p, i, o, bias=True):
        s.append((p + ".weight", (i, o), "mat"))
        if bias:
            s.append((p + ".bias", (o,), "bias"))

    def conv(p, k, i, o, bias=True):
        s.append((p + ".weight", (k, i, o), "conv"))
        if bias:
            s.append((p + ".bias", (o,), "bias"))

    def convmlp(p):
        conv(p + ".w1", 3, H, F, False)
        conv(p + ".w3", 3, H, F, False)
        conv(p + ".w2", 3, F, H, False)

    def mlp(p):
        lin(p + ".w1", H, F, False)
        lin(p + ".w3", H, F, False)
        lin(p + ".w2", F, H, False)

    conv("audio_input_proj.0", 3, L, H)
    convmlp("audio_input_proj.2")
    lin("t_embed.mlp.0", H, H)
    lin("t_embed.mlp.2", H, H)
    lin("clip_input_proj.0", hp.clip_dim, H)
    convmlp("clip_input_proj.2")
    s.append(("sync_pos_emb", (hp.sync_dim, 8, 1, 1), "emb"))
    conv("sync_input_proj.0", 7, hp.sync_dim, H)
    convmlp("sync_input_proj.2")
    lin("text_input_proj.0", hp.t5_dim, H)
    mlp("text_input_proj.2")
    lin("text_cond_proj", hp.text_dim, H)
    lin("clip_cond_proj", H, H)
    mlp("global_cond_mlp")
    lin("final_layer.adaLN_modulation.1", H, 2 * H)
    conv("final_layer.conv", 7, H, L)
    s.append(("empty_clip_feat", (hp.clip_dim, 1), "emb"))
    s.append(("empty_sync_feat", (hp.sync_dim, 1), "emb"))
    s.append(("empty_string_feat", (hp.text_dim, hp.text_seq), "emb"))
    s.append(("empty_t5_feat", (hp.t5_dim, hp.t5_seq), "zeros"))

    def block(p, kind, pre_only):
        lin(p + ".adaLN_modulation.1", H, (2 if pre_only else 6) * H)
        lin(p + ".attn.qkv", H, 3 * H)
        s.append((p + ".attn.q_norm.weight", (hd,), "gain"))
        s.append((p + ".attn.k_norm.weight", (hd,), "gain"))
        if pre_only:
            return
        if kind == "text":
            lin(p + ".linear1", H, H)
            mlp(p + ".ffn")
        else:
            conv(p + ".linear1", 3, H, H)
            convmlp(p + ".ffn")

    for i in range(hp.n_joint):
        pre_only = i == hp.n_joint - 1
        block(f"joint_blocks.{i}.latent_block", "latent", False)
        block(f"joint_blocks.{i}.clip_block", "clip", pre_only)
        block(f"joint_blocks.{i}.text_block", "text", pre_only)
    for i in range(hp.fused_depth):
        block(f"fused_blocks.{i}", "latent", False)
    return s


def storage_type(name: str, ne: Tuple[int, ...], wtype: str) -> int:
    """Per-tensor ggml type of a converted file (quantize_gguf.py:11-15)."""
    if wtype == "f32":
        return GGML_F32
    blocked = ("empty" in name or "_emb" in name or "norm" in name)
    if wtype == "bf16":
        return GGML_BF16 if (not blocked and len(ne) in (2, 3)) else GGML_F32
    if wtype == "q8_0":
        return GGML_Q8_0 if (not blocked and len(ne) == 2 and ne[0] % 32 == 0) else GGML_F32
    raise ValueError(wtype)


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        r[nan] = 0x7FC0
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def quantize_q8_0(a: np.ndarray) -> np.ndarray:
    """ggml Q8_0 blocks along ne0: fp16 d = amax/127, int8 q = round(x/d). 34 bytes / 32."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    rows = a.reshape(-1, 32)
    amax = np.abs(rows).max(axis=1, keepdims=True)
    d = amax / 127.0
    with np.errstate(divide="ignore", invalid="ignore"):
        idv = np.where(d > 0, 1.0 / d, 0.0)
    q = np.rint(rows * idv).astype(np.int8)
    out = np.empty((rows.shape[0], 34), np.uint8)
    out[:, :2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.reshape(*a.shape[:-1], a.shape[-1] // 32 * 34)


def random_q8_0(shape_np: Tuple[int, ...], rng: np.random.Generator) -> np.ndarray:
    """Q8_0 blocks with int8 ~ U[-127, 127] and fp16 scale ~ U[1e-4, 4e-3] (BASELINE cfg 4)."""
    nblk = int(np.prod(shape_np)) // 32
    out = np.empty((nblk, 34), np.uint8)
    out[:, :2] = rng.uniform(1e-4, 4e-3, size=(nblk, 1)).astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = rng.integers(-127, 128, size=(nblk, 32), dtype=np.int8).view(np.uint8)
    return out.reshape(*shape_np[:-1], shape_np[-1] // 32 * 34)


@dataclasses.dataclass
class WTensor:
    name: str
    ne: Tuple[int, ...]
    type: int
    data: np.ndarray       # raw ggml bytes (uint8 / uint16 / float32), numpy shape = reversed ne

    def raw(self) -> np.ndarray:
        return np.ascontiguousarray(self.data)

    def dequant(self) -> np.ndarray:
        """float32 array with numpy shape = reversed ne."""
        shp = tuple(reversed(self.ne))
        if self.type == GGML_F32:
            return self.data.astype(np.float32).reshape(shp)
        if self.type == GGML_BF16:
            return bf16_bits_to_f32(self.data).reshape(shp)
        if self.type == GGML_F16:
            return self.data.view(np.float16).astype(np.float32).reshape(shp)
        if self.type == GGML_Q8_0:
            blk = self.data.reshape(-1, 34)
            d = blk[:, :2].copy().view(np.float16).astype(np.float32)
            q = blk[:, 2:].view(np.int8).astype(np.float32)
            return (q * d).reshape(shp)
        raise ValueError(self.type)


def make_weights(hp: DitHParams, seed: int = 1234, wtype: str = "bf16", std: float = 0.02,
                 q8_random_blocks: bool = False) -> Dict[str, WTensor]:
    """Seeded synthetic DiT weights. ``wtype`` in {"f32", "bf16", "q8_0"}."""
    rng = np.random.default_rng(seed)
    out: Dict[str, WTensor] = {}
    for name, ne, kind in tensor_specs(hp):
        shp = tuple(reversed(ne))
        t = storage_type(name, ne, wtype)
        if kind == "zeros":
            a = np.zeros(shp, np.float32)
        elif kind == "gain":
            a = (1.0 + 0.1 * rng.standard_normal(shp)).astype(np.float32)
        elif kind == "emb":
            a = rng.standard_normal(shp).astype(np.float32)
        else:
            if t == GGML_Q8_0 and q8_random_blocks:
                out[name] = WTensor(name, ne, t, random_q8_0(shp, rng))
                continue
            a = (std * rng.standard_normal(shp)).astype(np.float32)
        if t == GGML_F32:
            data = a
        elif t == GGML_BF16:
            data = f32_to_bf16_bits(a).reshape(shp)
        elif t == GGML_Q8_0:
            data = quantize_q8_0(a)
        else:
            raise ValueError(t)
        out[name] = WTensor(name, ne, t, data)
    return out


def write_gguf(path: str, hp: DitHParams, weights: Dict[str, WTensor]) -> None:
    """Write a DiT GGUF with the reference's metadata keys (convert_thinksound.py:37-46)."""
    import gguf
    w = gguf.GGUFWriter(path, arch="thinksound-mmdit")
    for k, v in dict(latent_dim=hp.latent_dim, clip_dim=hp.clip_dim, sync_dim=hp.sync_dim,
                     text_dim=hp.t5_dim, hidden_dim=hp.hidden, depth=hp.depth,
                     fused_depth=hp.fused_depth, num_heads=hp.n_head, text_seq_len=hp.text_seq,
                     kernel_size=3, sync_kernel=7).items():
        w.add_uint32(f"dit.{k}", int(v))
    w.add_float32("dit.rope_theta", float(hp.rope_theta))
    w.add_float32("dit.t_embed_max_period", float(hp.t_max_period))
    w.add_uint32("dit.sample_rate", 44100)
    w.add_string("dit.diffusion_objective", "rectified_flow")
    qt = {GGML_BF16: gguf.GGMLQuantizationType.BF16, GGML_Q8_0: gguf.GGMLQuantizationType.Q8_0,
          GGML_F16: gguf.GGMLQuantizationType.F16}
    for name, t in weights.items():
        if t.type == GGML_F32:
            w.add_tensor(name, np.ascontiguousarray(t.data, dtype=np.float32))
        else:
            raw = np.ascontiguousarray(t.data).view(np.uint8)
            w.add_tensor(name, raw, raw_dtype=qt[t.type])
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


@dataclasses.dataclass
class DitInputs:
    """One batch item of forward() inputs in the reference's host layouts (mmdit.h:19-29)."""
    latent: np.ndarray    # [latent_dim][T] (t fastest)
    clip_f: np.ndarray    # [clip_S][clip_dim]
    sync_f: np.ndarray    # [sync_S][sync_dim]
    text_f: np.ndarray    # [text_S][text_dim]
    t5: np.ndarray        # [t5_S][t5_dim]
    gtext: np.ndarray     # [text_dim]
    t: float


def make_inputs(hp: DitHParams, T: int, clip_S: int, sync_S: int, text_S: int, t5_S: int,
                seed: int = 4242, batch: int = 1) -> List[DitInputs]:
    rng = np.random.default_rng(seed)
    items = []
    for _ in range(batch):
        items.append(DitInputs(
            latent=rng.standard_normal((hp.latent_dim, T)).astype(np.float32),
            clip_f=rng.standard_normal((clip_S, hp.clip_dim)).astype(np.float32),
            sync_f=rng.standard_normal((sync_S, hp.sync_dim)).astype(np.float32),
            text_f=rng.standard_normal((text_S, hp.text_dim)).astype(np.float32),
            t5=rng.standard_normal((t5_S, hp.t5_dim)).astype(np.float32),
            gtext=rng.standard_normal((hp.text_dim,)).astype(np.float32),
            t=float(rng.uniform(0.0, 1.0))))
    return items


def step_flops(hp: DitHParams, B: int, T: int, clip_S: int, sync_S: int, text_S: int, t5_S: int) -> Dict[str, float]:
    """Algorithmic FLOPs of one forward over B items (2*M*N*K per GEMM, 4*S*S*H per attention)."""
    H, F, L = hp.hidden, hp.ffn, hp.latent_dim
    St = text_S + t5_S
    Sj = T + clip_S + St
    f = dict(adaln=0.0, qkv=0.0, attn=0.0, out=0.0, ffn=0.0, pre=0.0)

    def g(n, k, m):
        return 2.0 * B * n * k * m

    def sub(S, conv, pre_only, per_token_cond):
        f["adaln"] += g(S if per_token_cond else 1, H, (2 if pre_only else 6) * H)
        f["qkv"] += g(S, H, 3 * H)
        if pre_only:
            return
        kk = 3 if conv else 1
        f["out"] += g(S, kk * H, H)
        f["ffn"] += 2 * g(S, kk * H, F) + g(S, kk * F, H)

    for i in range(hp.n_joint):
        po = i == hp.n_joint - 1
        sub(T, True, False, True)
        sub(clip_S, True, po, False)
        sub(St, False, po, False)
        f["attn"] += 4.0 * B * Sj * Sj * H
    for _ in range(hp.fused_depth):
        sub(T, True, False, True)
        f["attn"] += 4.0 * B * T * T * H
    # pre-processing + final layer (mmdit.cpp:150-200, 284-290)
    f["pre"] += g(T, 3 * L, H) + 2 * g(T, 3 * H, F) + g(T, 3 * F, H)
    f["pre"] += g(1, H, H) * 2
    f["pre"] += g(clip_S, hp.clip_dim, H) + 2 * g(clip_S, 3 * H, F) + g(clip_S, 3 * F, H)
    f["pre"] += g(sync_S, 7 * hp.sync_dim, H) + 2 * g(sync_S, 3 * H, F) + g(sync_S, 3 * F, H)
    f["pre"] += g(St, hp.t5_dim, H) + 2 * g(St, H, F) + g(St, F, H)
    f["pre"] += g(1, hp.text_dim, H) + g(1, H, H) + 2 * g(1, H, F) + g(1, F, H)
    f["pre"] += g(T, H, 2 * H) + g(T, 7 * H, L)
    f["total"] = sum(f.values())
    f["attn_proj"] = f["qkv"] + f["attn"] + f["out"]
    return f
