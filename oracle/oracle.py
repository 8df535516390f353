"""ctypes binding of the CPU oracle (oracle/_build/libtsd_oracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's CPU
baseline leg, never by the product package. Parity unpinned (see tsd_oracle.cpp header).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Dict, List, Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libtsd_oracle.so")

EMU_ACT = 1
EMU_KV16 = 2
MODE_GGML = EMU_ACT | EMU_KV16
MODE_EXACT = 0

_DBG_CB = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_float), ctypes.c_int64)
_lib = None


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        fp = ctypes.POINTER(ctypes.c_float)
        L.tso_model_new.restype = ctypes.c_void_p
        L.tso_model_new.argtypes = [ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_float]
        L.tso_model_free.argtypes = [ctypes.c_void_p]
        L.tso_model_set.restype = ctypes.c_int
        L.tso_model_set.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int,
                                    ctypes.POINTER(ctypes.c_int64), ctypes.c_void_p]
        L.tso_forward.restype = ctypes.c_int
        L.tso_forward.argtypes = [ctypes.c_void_p, ctypes.c_int, fp, ctypes.c_int64, ctypes.c_float,
                                  fp, ctypes.c_int64, fp, ctypes.c_int64, fp, ctypes.c_int64,
                                  fp, ctypes.c_int64, fp, fp, _DBG_CB, ctypes.c_void_p]
        L.tso_sample.restype = ctypes.c_int
        L.tso_sample.argtypes = [ctypes.c_void_p, ctypes.c_int, fp, ctypes.c_int64,
                                 fp, ctypes.c_int64, fp, ctypes.c_int64, fp, ctypes.c_int64,
                                 fp, ctypes.c_int64, fp, ctypes.c_int, ctypes.c_float, fp, fp]
        L.tso_num_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _fp(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


class OracleModel:
    """The oracle's DiT: hparams + named ggml tensors (dequantised to f32 inside)."""

    def __init__(self, hp, weights):
        L = lib()
        self.hp = hp
        self.h = L.tso_model_new(hp.hidden, hp.n_head, hp.depth, hp.fused_depth, hp.latent_dim,
                                 hp.rope_theta, hp.t_max_period)
        for name, t in weights.items():
            ne = (ctypes.c_int64 * 4)(*(list(t.ne) + [1] * (4 - len(t.ne))))
            raw = t.raw()
            rc = L.tso_model_set(self.h, name.encode(), t.type, ne, raw.ctypes.data_as(ctypes.c_void_p))
            if rc != 0:
                raise RuntimeError(f"tso_model_set({name}) -> {rc}")

    def __del__(self):
        try:
            if getattr(self, "h", None) and _lib is not None:
                _lib.tso_model_free(self.h)
                self.h = None
        except Exception:
            pass

    def forward(self, x, mode: int = MODE_GGML, dbg: bool = False):
        """One batch item (synth.DitInputs). Returns flow [T][latent] (and dbg dict)."""
        L = lib()
        lat = np.ascontiguousarray(x.latent, np.float32)
        T = lat.shape[1]
        out = np.zeros((T, self.hp.latent_dim), np.float32)
        store: Dict[str, np.ndarray] = {}

        def cb(_ud, name, ptr, n):
            store[name.decode()] = np.ctypeslib.as_array(ptr, shape=(n,)).copy()

        cbf = _DBG_CB(cb) if dbg else _DBG_CB()
        arrs = [np.ascontiguousarray(a, np.float32) for a in (x.clip_f, x.sync_f, x.text_f, x.t5, x.gtext)]
        rc = L.tso_forward(self.h, mode, _fp(lat), T, float(x.t),
                           _fp(arrs[0]), arrs[0].shape[0], _fp(arrs[1]), arrs[1].shape[0],
                           _fp(arrs[2]), arrs[2].shape[0], _fp(arrs[3]), arrs[3].shape[0],
                           _fp(arrs[4]), _fp(out), cbf, None)
        if rc != 0:
            raise RuntimeError(f"tso_forward -> {rc}")
        return (out, store) if dbg else out

    def sample(self, x, steps: int, cfg: float, mode: int = MODE_GGML, want_flow0: bool = False):
        L = lib()
        noise = np.ascontiguousarray(x.latent, np.float32)
        T = noise.shape[1]
        out = np.zeros_like(noise)
        flow0 = np.zeros_like(noise) if want_flow0 else None
        arrs = [np.ascontiguousarray(a, np.float32) for a in (x.clip_f, x.sync_f, x.text_f, x.t5, x.gtext)]
        rc = L.tso_sample(self.h, mode, _fp(noise), T,
                          _fp(arrs[0]), arrs[0].shape[0], _fp(arrs[1]), arrs[1].shape[0],
                          _fp(arrs[2]), arrs[2].shape[0], _fp(arrs[3]), arrs[3].shape[0],
                          _fp(arrs[4]), steps, cfg, _fp(out),
                          _fp(flow0) if flow0 is not None else ctypes.POINTER(ctypes.c_float)())
        if rc != 0:
            raise RuntimeError(f"tso_sample -> {rc}")
        return (out, flow0) if want_flow0 else out


def num_threads() -> int:
    return lib().tso_num_threads()


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.sqrt(((a - b) ** 2).sum() / ((b ** 2).sum() + 1e-30)))
