"""Generate tests/golden/dit_small.npz: seeded small-model fixtures for the MM-DiT hot path.

The reference's own golden GGUFs (convert/dump_dit_golden.py, dump_dit_debug*.py) were never
committed and its PyTorch upstream is absent, so these fixtures come from this repository's CPU
oracle (oracle/tsd_oracle.cpp, a restatement of src/mmdit.cpp) and are cross-checked here
against the independent PyTorch restatement (tests/torch_ref.py) before being written. They pin
the oracle against regressions; they do not pin it against the reference (parity unpinned).

Run from the repository root:  python tests/golden/make_golden.py
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [REPO, os.path.join(REPO, "oracle"), os.path.join(REPO, "tests")]

import __graft_entry__  # noqa: E402

__graft_entry__.load_package()
from tsd_b200 import synth  # noqa: E402
import oracle  # noqa: E402
import torch_ref  # noqa: E402

HP = dict(hidden=128, n_head=2, depth=3, fused_depth=1, ffn=256)
SHAPE = dict(T=20, clip_S=8, sync_S=24, text_S=77, t5_S=9)
STAGES = ["x_in", "t_emb", "clip_pp", "text_pp", "global_c", "extended_c", "a0_q", "a0_k", "a0_v", "a0_out",
          "jb0_lat", "after_joint", "after_fused", "flow_cl"]


def weights_digest(W) -> str:
    h = hashlib.sha256()
    for name in sorted(W):
        h.update(name.encode())
        h.update(np.ascontiguousarray(W[name].data).tobytes())
    return h.hexdigest()


def main():
    import torch
    hp = synth.DitHParams(**HP)
    out = {}
    for wtype in ("bf16", "q8_0", "f32"):
        W = synth.make_weights(hp, seed=1234, wtype=wtype)
        x = synth.make_inputs(hp, seed=4242, **SHAPE)[0]
        om = oracle.OracleModel(hp, W)
        flow_g, dbg_g = om.forward(x, mode=oracle.MODE_GGML, dbg=True)
        flow_e = om.forward(x, mode=oracle.MODE_EXACT)
        tref = torch_ref.TorchDiT(hp, W, dtype=torch.float64).forward(x)
        r = oracle.rel_l2(flow_e, tref)
        assert r < 1e-5, f"oracle vs torch restatement ({wtype}) rel-L2 {r}"
        out[f"{wtype}/digest"] = np.frombuffer(weights_digest(W).encode(), np.uint8)
        out[f"{wtype}/flow_ggml"] = flow_g
        out[f"{wtype}/flow_exact"] = flow_e
        if wtype == "bf16":
            for k in STAGES:
                out[f"{wtype}/stage/{k}"] = dbg_g[k]
            lat, f0 = om.sample(x, steps=3, cfg=5.0, mode=oracle.MODE_GGML, want_flow0=True)
            out["bf16/sample3_latent"] = lat
            out["bf16/sample3_flow0"] = f0
        print(wtype, "oracle vs torch", r)
    np.savez_compressed(os.path.join(HERE, "dit_small.npz"), **out)
    print("wrote", os.path.join(HERE, "dit_small.npz"))


if __name__ == "__main__":
    main()
