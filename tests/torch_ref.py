"""Independent PyTorch (CPU, fp32/fp64) restatement of the reference DiT forward.

Test infrastructure: it cross-checks the C++ oracle (oracle/tsd_oracle.cpp), which is the
checker the GPU path is compared against. It is written in the module style of the upstream
MMAudio/ThinkSound PyTorch model the reference ports (ChannelLastConv1d, ConvMLP, SelfAttention
with `b n (h d j)` qkv split, FLUX-style rotation matrices) and follows the reference's
numerics where they differ from upstream: LayerNorm eps 1e-5 (src/mmdit.cpp:59), QK RMSNorm
eps 1e-6 (:10,78-80), RoPE on the latent and clip streams with clip freq_scale T/clip_S
(:237,245-246), text stream = [MetaCLIP-text padded to the T5 width | T5] (:178-183).

``emulate=True`` reproduces the reference's rounding points: every linear/conv input is
rounded to the weight's storage type (bf16 for BF16 weights), and Q/K/V are rounded to fp16
before attention (:88-90).
"""
from __future__ import annotations

import math
from typing import Dict, Optional

import numpy as np
import torch
import torch.nn.functional as F

GGML_F32, GGML_F16, GGML_Q8_0, GGML_BF16 = 0, 1, 8, 30


class TorchDiT:
    def __init__(self, hp, weights, dtype=torch.float32, emulate=False):
        self.hp = hp
        self.dtype = dtype
        self.emulate = emulate
        self.w = {n: torch.from_numpy(t.dequant().copy()).to(dtype) for n, t in weights.items()}
        self.wt = {n: t.type for n, t in weights.items()}

    # --- rounding of activations at a linear/conv input (reference mul_mat src1 conversion)
    def _act(self, x, wname):
        if not self.emulate:
            return x
        t = self.wt[wname]
        if t == GGML_BF16:
            return x.to(torch.bfloat16).to(self.dtype)
        if t == GGML_F16:
            return x.to(torch.float16).to(self.dtype)
        if t == GGML_Q8_0:
            xs = x.reshape(-1, 32)
            d = xs.abs().amax(dim=1, keepdim=True) / 127.0
            idv = torch.where(d > 0, 1.0 / d, torch.zeros_like(d))
            q = torch.round(xs * idv)
            return (q * d.to(torch.float16).to(self.dtype)).reshape(x.shape)
        return x

    def linear(self, p, x, bias=True):
        w = self.w[p + ".weight"]
        return F.linear(self._act(x, p + ".weight"), w, self.w[p + ".bias"] if bias else None)

    def conv_cl(self, p, x, pad, bias=True):   # ChannelLastConv1d: x [B, N, C]
        w = self.w[p + ".weight"]                 # [OC, IC, K]
        y = F.conv1d(self._act(x, p + ".weight").transpose(1, 2), w,
                     self.w[p + ".bias"] if bias else None, padding=pad)
        return y.transpose(1, 2)

    def conv_mlp(self, p, x):
        return self.conv_cl(p + ".w2", F.silu(self.conv_cl(p + ".w1", x, 1, False)) *
                            self.conv_cl(p + ".w3", x, 1, False), 1, False)

    def mlp(self, p, x):
        return self.linear(p + ".w2", F.silu(self.linear(p + ".w1", x, False)) *
                           self.linear(p + ".w3", x, False), False)

    @staticmethod
    def modulate(x, shift, scale):
        return x * (1 + scale) + shift

    def rope_rot(self, L, freq_scaling):
        hd = self.hp.head_dim
        freqs = freq_scaling * self.hp.rope_theta ** (-torch.arange(0, hd, 2, dtype=torch.float64) / hd)
        ang = torch.arange(L, dtype=torch.float64)[:, None] * freqs[None, :]
        return torch.cos(ang).to(self.dtype), torch.sin(ang).to(self.dtype)

    @staticmethod
    def apply_rope(x, rot):   # x [B, h, N, d]; pairs (2i, 2i+1)
        c, s = rot
        x2 = x.reshape(*x.shape[:-1], -1, 2)
        x0, x1 = x2[..., 0], x2[..., 1]
        return torch.stack([c * x0 - s * x1, s * x0 + c * x1], dim=-1).reshape(x.shape)

    def rms(self, x, g):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * g

    def pre_attention(self, p, x, c, rot, pre_only):
        H, nh = self.hp.hidden, self.hp.n_head
        mod = self.linear(p + ".adaLN_modulation.1", F.silu(c))
        chunks = mod.chunk(2 if pre_only else 6, dim=-1)
        xn = self.modulate(F.layer_norm(x, (H,), eps=1e-5), chunks[0], chunks[1])
        qkv = self.linear(p + ".attn.qkv", xn)
        B, N, _ = qkv.shape
        qkv = qkv.view(B, N, nh, H // nh, 3).permute(0, 2, 1, 3, 4)   # b h n d j
        q, k, v = qkv[..., 0], qkv[..., 1], qkv[..., 2]
        q = self.rms(q, self.w[p + ".attn.q_norm.weight"])
        k = self.rms(k, self.w[p + ".attn.k_norm.weight"])
        if rot is not None:
            q, k = self.apply_rope(q, rot), self.apply_rope(k, rot)
        return q, k, v, chunks, xn

    def attention(self, q, k, v):
        if self.emulate:
            q, k, v = (t.to(torch.float16).to(self.dtype) for t in (q, k, v))
        s = (q @ k.transpose(-1, -2)) / math.sqrt(q.shape[-1])
        o = torch.softmax(s, dim=-1) @ v                  # [B, h, N, d]
        B, h, N, d = o.shape
        return o.permute(0, 2, 1, 3).reshape(B, N, h * d)

    def post_attention(self, p, x, ao, chunks, is_text):
        H = self.hp.hidden
        _, _, gate_msa, shift_mlp, scale_mlp, gate_mlp = chunks
        l1 = self.linear(p + ".linear1", ao) if is_text else self.conv_cl(p + ".linear1", ao, 1)
        x = x + l1 * gate_msa
        r = self.modulate(F.layer_norm(x, (H,), eps=1e-5), shift_mlp, scale_mlp)
        f = self.mlp(p + ".ffn", r) if is_text else self.conv_mlp(p + ".ffn", r)
        return x + f * gate_mlp

    def forward(self, inp, dbg: Optional[Dict[str, np.ndarray]] = None):
        hp, H = self.hp, self.hp.hidden
        tt = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(self.dtype)[None]
        latent = tt(inp.latent).transpose(1, 2)           # [1, T, 64]
        T = latent.shape[1]
        clip_f, sync_f = tt(inp.clip_f), tt(inp.sync_f)
        text_f, t5, gtext = tt(inp.text_f), tt(inp.t5), tt(inp.gtext)
        clip_S, sync_S = clip_f.shape[1], sync_f.shape[1]

        x = self.conv_mlp("audio_input_proj.2", F.silu(self.conv_cl("audio_input_proj.0", latent, 1)))
        half = H // 2
        # the reference computes the sinusoid on the host in float32 (mmdit.cpp:306-313)
        f32 = torch.float32
        fr = torch.tensor(10000.0 / hp.t_max_period, dtype=f32) * torch.pow(
            torch.tensor(10000.0, dtype=f32), -2.0 * torch.arange(half, dtype=f32) / H)
        ang = torch.tensor(inp.t, dtype=f32) * fr
        temb = torch.cat([torch.cos(ang), torch.sin(ang)]).to(self.dtype)[None]
        te = self.linear("t_embed.mlp.2", F.silu(self.linear("t_embed.mlp.0", temb)))

        clip = self.conv_mlp("clip_input_proj.2", F.silu(self.linear("clip_input_proj.0", clip_f)))
        spe = self.w["sync_pos_emb"].reshape(1, 1, 8, hp.sync_dim)
        sy = (sync_f.view(1, sync_S // 8, 8, hp.sync_dim) + spe).reshape(1, sync_S, hp.sync_dim)
        sy = self.conv_mlp("sync_input_proj.2", F.silu(self.conv_cl("sync_input_proj.0", sy, 3)))
        idx = torch.floor((torch.arange(T, dtype=torch.float32) + 0.5) * sync_S / T).long()
        sy = sy[:, idx]
        text_cat = torch.cat([F.pad(text_f, (0, hp.t5_dim - text_f.shape[-1])), t5], dim=1)
        text = self.mlp("text_input_proj.2", F.silu(self.linear("text_input_proj.0", text_cat)))
        text_fc = self.linear("text_cond_proj", gtext)
        clip_fc = self.linear("clip_cond_proj", clip.mean(dim=1))
        gc = self.mlp("global_cond_mlp", clip_fc + text_fc)
        if dbg is not None:
            dbg.update(x_in=x, t_emb=te, clip_pp=clip, text_pp=text, clip_fc=clip_fc, text_fc=text_fc, gcmlp=gc)
        global_c = (gc + te)[:, None]                     # [1, 1, H]
        extended_c = sy + global_c
        if dbg is not None:
            dbg.update(global_c=global_c, extended_c=extended_c)

        lat_rot = self.rope_rot(T, 1.0)
        clip_rot = self.rope_rot(clip_S, T / clip_S)
        for i in range(hp.n_joint):
            jb = f"joint_blocks.{i}"
            po = i == hp.n_joint - 1
            ql, kl, vl, cl, _ = self.pre_attention(jb + ".latent_block", x, extended_c, lat_rot, False)
            qc, kc, vc, cc, _ = self.pre_attention(jb + ".clip_block", clip, global_c, clip_rot, po)
            qt, kt, vt, ct, xnt = self.pre_attention(jb + ".text_block", text, global_c, None, po)
            q = torch.cat([ql, qc, qt], dim=2)
            k = torch.cat([kl, kc, kt], dim=2)
            v = torch.cat([vl, vc, vt], dim=2)
            ao = self.attention(q, k, v)
            if dbg is not None and i == 0:
                flat = lambda z: z.permute(0, 2, 1, 3).reshape(1, z.shape[2], H)
                dbg.update(text_xn=xnt, a0_q=flat(q), a0_k=flat(k), a0_v=flat(v), a0_out=ao)
            nl, nc = x.shape[1], clip.shape[1]
            x = self.post_attention(jb + ".latent_block", x, ao[:, :nl], cl, False)
            if not po:
                clip = self.post_attention(jb + ".clip_block", clip, ao[:, nl:nl + nc], cc, False)
                text = self.post_attention(jb + ".text_block", text, ao[:, nl + nc:], ct, True)
            if dbg is not None and i == 0:
                dbg.update(jb0_lat=x, jb0_clip=clip, jb0_text=text)
        if dbg is not None:
            dbg["after_joint"] = x
        for i in range(hp.fused_depth):
            fb = f"fused_blocks.{i}"
            q, k, v, c, _ = self.pre_attention(fb, x, extended_c, lat_rot, False)
            x = self.post_attention(fb, x, self.attention(q, k, v), c, False)
        if dbg is not None:
            dbg["after_fused"] = x
        shift, scale = self.linear("final_layer.adaLN_modulation.1", F.silu(extended_c)).chunk(2, dim=-1)
        fx = self.modulate(F.layer_norm(x, (H,), eps=1e-5), shift, scale)
        flow = self.conv_cl("final_layer.conv", fx, 3)   # [1, T, 64]
        if dbg is not None:
            dbg["flow_cl"] = flow
            for k_ in list(dbg):
                dbg[k_] = dbg[k_].detach().to(torch.float32).numpy().ravel()
        return flow[0].detach().to(torch.float32).numpy()
