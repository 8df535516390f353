"""CPU tests of the drop-in boundary: the C-ABI library loads and exports every declared
symbol, argument validation that needs no GPU, and the host-side helpers."""
import ctypes
import os
import re

import numpy as np
import pytest

from tsd_b200 import synth, tsd

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in ("tsd.h", "tsd_ops.h"):
        src = open(os.path.join(REPO, "include", h)).read()
        names |= set(re.findall(r"TSD_API\s+[\w\s\*]*?\b(tsd_\w+)\s*\(", src))
    return names


def test_library_loads_and_exports_every_declared_symbol():
    lib = tsd.lib()
    decl = declared_symbols()
    assert len(decl) >= 20
    missing = [n for n in sorted(decl) if not hasattr(lib, n)]
    assert not missing, missing
    assert set(tsd.EXPORTS) == decl


def test_version_string():
    assert b"sm_100a" in tsd.lib().tsd_version()


def test_load_gguf_rejects_missing_and_non_gguf_files(tmp_path):
    h = ctypes.c_void_p()
    rc = tsd.lib().tsd_load_gguf(str(tmp_path / "nope.gguf").encode(), 0, ctypes.byref(h))
    assert rc == -3
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"NOTGGUF" + b"\0" * 64)
    rc = tsd.lib().tsd_load_gguf(str(bad).encode(), 0, ctypes.byref(h))
    assert rc == -3


def test_load_gguf_rejects_truncated_data_without_touching_the_gpu(tmp_path):
    """A GGUF whose header and tensor table are intact but whose data section was cut short
    (an interrupted download or copy) is rejected as TSD_ERR_IO before any device work."""
    hp = synth.DitHParams(hidden=128, n_head=2, depth=2, fused_depth=1, ffn=256)
    W = synth.make_weights(hp, seed=3, wtype="bf16")
    path = tmp_path / "dit.gguf"
    synth.write_gguf(str(path), hp, W)
    data = path.read_bytes()
    h = ctypes.c_void_p()
    for keep in (len(data) - 1, len(data) - 4096, len(data) // 2):
        cut = tmp_path / f"cut{keep}.gguf"
        cut.write_bytes(data[:keep])
        rc = tsd.lib().tsd_load_gguf(str(cut).encode(), 0, ctypes.byref(h))
        assert rc == -3, (keep, rc)
    # a header cut inside the tensor table is reported the same way
    short = tmp_path / "short.gguf"
    short.write_bytes(data[:200])
    assert tsd.lib().tsd_load_gguf(str(short).encode(), 0, ctypes.byref(h)) == -3


def test_wait_limit_range_is_checked_without_touching_the_gpu():
    L = tsd.lib()
    assert L.tsd_set_wait_limit(0, 10) == -1                 # below 1 ms
    assert L.tsd_set_wait_limit(0, 120 * 10**9) == -1        # above 60 s


def test_null_arguments_are_rejected_without_touching_the_gpu():
    L = tsd.lib()
    assert L.tsd_model_get_hparams(None, None) == -1
    assert L.tsd_get_tensor_f32(None, b"x", None, 0, None) == -1
    assert L.tsd_sync_check(None, None) == -1
    assert L.tsd_op_attention(None, None, None, 1, 1, 1, None, 64, None, None) == -1


def test_tensor_specs_follow_reference_schema():
    hp = synth.DitHParams()
    specs = {n: ne for n, ne, _ in synth.tensor_specs(hp)}
    H, F = 1536, 4096
    assert hp.ffn == F
    assert specs["joint_blocks.0.latent_block.attn.qkv.weight"] == (H, 3 * H)
    assert specs["joint_blocks.0.latent_block.linear1.weight"] == (3, H, H)
    assert specs["joint_blocks.0.text_block.linear1.weight"] == (H, H)
    assert specs["joint_blocks.6.clip_block.adaLN_modulation.1.weight"] == (H, 2 * H)
    assert "joint_blocks.6.clip_block.linear1.weight" not in specs
    assert specs["fused_blocks.13.ffn.w2.weight"] == (3, F, H)
    assert specs["final_layer.conv.weight"] == (7, H, 64)
    assert specs["sync_input_proj.0.weight"] == (7, 768, H)


def test_storage_types_follow_quantize_rules():
    assert synth.storage_type("t_embed.mlp.0.weight", (8, 8), "bf16") == synth.GGML_F32      # "_emb"
    assert synth.storage_type("x.attn.q_norm.weight", (64,), "bf16") == synth.GGML_F32
    assert synth.storage_type("x.linear1.weight", (3, 64, 64), "bf16") == synth.GGML_BF16
    assert synth.storage_type("x.linear1.weight", (3, 64, 64), "q8_0") == synth.GGML_F32     # conv stays F32
    assert synth.storage_type("x.attn.qkv.weight", (64, 192), "q8_0") == synth.GGML_Q8_0


def test_step_flops_match_reference_accounting():
    hp = synth.DitHParams()
    f = synth.step_flops(hp, B=2, T=194, clip_S=72, sync_S=216, text_S=77, t5_S=128)
    assert abs(f["total"] / 1e9 - 1819) / 1819 < 0.03
    assert abs(f["attn"] / 1e9 - 25.6) / 25.6 < 0.05


def test_gguf_writer_round_trip(tmp_path):
    import gguf
    hp = synth.DitHParams(hidden=128, n_head=2, depth=2, fused_depth=1, ffn=256)
    W = synth.make_weights(hp, seed=1, wtype="q8_0")
    path = str(tmp_path / "m.gguf")
    synth.write_gguf(path, hp, W)
    r = gguf.GGUFReader(path)
    assert int(r.fields["dit.hidden_dim"].contents()) == 128
    got = {t.name: t for t in r.tensors}
    assert set(got) == set(W)
    t = got["joint_blocks.0.latent_block.attn.qkv.weight"]
    assert int(t.tensor_type) == synth.GGML_Q8_0
    assert np.array_equal(np.asarray(t.data).view(np.uint8).ravel(), W[t.name].data.view(np.uint8).ravel())


SHIM_SRC = os.path.join(REPO, "tests", "shim", "ts_dit_demo.cpp")


def build_shim_demo(out_dir):
    """Compile the ts_dit drop-in demo against include/ and libtsd_b200.so (g++, C++17)."""
    import subprocess
    exe = os.path.join(str(out_dir), "ts_dit_demo")
    libdir = os.path.join(REPO, "thinksound.cpp_b200")
    subprocess.run(["g++", "-std=c++17", "-O1", "-I", os.path.join(REPO, "include"), SHIM_SRC, "-o", exe,
                    "-L", libdir, "-ltsd_b200", f"-Wl,-rpath,{libdir}"], check=True)
    return exe


def test_ts_dit_shim_compiles_and_reports_load_failure(tmp_path):
    import subprocess
    exe = build_shim_demo(tmp_path)
    r = subprocess.run([exe, str(tmp_path / "missing.gguf"), "20", "8", "24", "1"], capture_output=True, text=True)
    assert r.returncode == 1 and "load failed" in r.stderr
