"""ctypes binding of libtsd_b200.so (include/tsd.h, include/tsd_ops.h).

Host-side mirror of the reference's ``ts_dit`` interface (src/mmdit.h:9-42): ``DitModel.load``
(ts_dit::load), ``forward`` (ts_dit::forward, with the ``dbg`` stage map of mmdit.cpp:333-337)
and ``sample`` (ts_dit::sample). There is no fallback: if the CUDA library is not built or no
GPU is visible the calls raise.
"""
from __future__ import annotations

import ctypes
import os
from typing import Dict, List, Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libtsd_b200.so")

TSD_OK = 0
ERRORS = {-1: "TSD_ERR_ARG", -2: "TSD_ERR_CUDA", -3: "TSD_ERR_IO", -4: "TSD_ERR_MISSING",
          -5: "TSD_ERR_DEVICE", -6: "TSD_ERR_UNSUPPORTED", -7: "TSD_ERR_STATE"}

EPI_STORE, EPI_SWIGLU, EPI_GATE_RESID = 0, 1, 2
ACT_NONE, ACT_SILU = 0, 1

# Every symbol include/tsd.h and include/tsd_ops.h declare.
EXPORTS = [
    "tsd_load_gguf", "tsd_model_create", "tsd_model_set_tensor", "tsd_model_finalize", "tsd_model_free",
    "tsd_model_get_hparams", "tsd_get_tensor_f32", "tsd_forward", "tsd_forward_batched",
    "tsd_forward_device", "tsd_sync_check", "tsd_sample", "tsd_sample_batched", "tsd_version",
    "tsd_device_count", "tsd_op_gemm", "tsd_op_gemv", "tsd_op_attention", "tsd_op_ln_modulate",
    "tsd_op_qk_norm_rope", "tsd_forward_profile", "tsd_plan_op_label", "tsd_op_gemm_static",
    "tsd_hp_layout", "tsd_hp_init", "tsd_hp_connect", "tsd_op_gemm_plan",
    "tsd_set_wait_limit", "tsd_op_peer_wait", "tsd_op_attention_f32", "tsd_forward_inject",
]


class TsdError(RuntimeError):
    def __init__(self, fn: str, rc: int):
        super().__init__(f"{fn} failed: {ERRORS.get(rc, rc)}")
        self.rc = rc


class HParams(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int32), ("n_head", ctypes.c_int32), ("depth", ctypes.c_int32),
                ("fused_depth", ctypes.c_int32), ("latent_dim", ctypes.c_int32),
                ("rope_theta", ctypes.c_float), ("t_max_period", ctypes.c_float)]


DBG_FN = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_float), ctypes.c_int64)
INJECT_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_float),
                             ctypes.c_int64)

_lib = None


def lib() -> ctypes.CDLL:
    """Load libtsd_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} not built: run `make -C thinksound.cpp_b200` (or __graft_entry__.build())")
    L = ctypes.CDLL(LIB_PATH)
    vp, i64, i32, f32, fp = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.POINTER(ctypes.c_float)
    sig = {
        "tsd_load_gguf": [ctypes.c_char_p, i32, ctypes.POINTER(vp)],
        "tsd_model_create": [ctypes.POINTER(HParams), i32, ctypes.POINTER(vp)],
        "tsd_model_set_tensor": [vp, ctypes.c_char_p, i32, ctypes.POINTER(i64), vp, ctypes.c_size_t],
        "tsd_model_finalize": [vp],
        "tsd_model_free": [vp],
        "tsd_model_get_hparams": [vp, ctypes.POINTER(HParams)],
        "tsd_get_tensor_f32": [vp, ctypes.c_char_p, fp, i64, ctypes.POINTER(i64)],
        "tsd_forward": [vp, fp, i64, f32, fp, i64, fp, i64, fp, i64, fp, i64, fp, fp],
        "tsd_forward_batched": [vp, i32, fp, i64, fp, fp, i64, fp, i64, fp, i64, fp, i64, fp, fp, DBG_FN, vp],
        "tsd_forward_device": [vp, i32, vp, i64, vp, vp, i64, vp, i64, vp, i64, vp, i64, vp, vp, vp],
        "tsd_sync_check": [vp, vp],
        "tsd_sample": [vp, fp, i64, fp, i64, fp, i64, fp, i64, fp, i64, fp, i32, f32, fp, fp],
        "tsd_sample_batched": [vp, i32, fp, i64, fp, i64, fp, i64, fp, i64, fp, i64, fp, i32, f32, fp, fp],
        "tsd_version": [],
        "tsd_device_count": [],
        "tsd_op_gemm": [vp, i32, i32, i32, i32, vp, i32, i32, i64, i64, i32, i32, vp, i32, vp, i32, i64, vp, i64, vp,
                        i64, i32, i32, vp, i64, vp, i32, vp, vp],
        "tsd_op_gemm_static": [vp, i32, i32, i32, i32, vp, i32, i32, i64, i64, i32, i32, vp, i32, vp, i32, i64, vp,
                               i64, vp, i64, i32, i32, vp, vp],
        "tsd_op_gemv": [vp, i32, vp, i32, i32, vp, i64, i32, vp, i32, i32, vp, i32, i64, vp],
        "tsd_op_gemm_plan": [i32, i32, i32, i32, i32, i32, i64, i32, ctypes.POINTER(i64)],
        "tsd_set_wait_limit": [i32, ctypes.c_uint64],
        "tsd_op_peer_wait": [vp, vp, i32, i32, ctypes.c_uint32, vp, vp],
        "tsd_op_attention": [vp, vp, vp, i32, i32, i32, vp, i64, vp, vp],
        "tsd_op_attention_f32": [vp, vp, vp, i32, i32, i32, vp, i64, vp, vp],
        "tsd_forward_inject": [vp, i32, fp, i64, fp, fp, i64, fp, i64, fp, i64, fp, i64, fp, fp, DBG_FN, INJECT_FN, vp],
        "tsd_hp_layout": [i32, i32, i32, i32, ctypes.POINTER(i32)],
        "tsd_hp_init": [vp, i32, i32, ctypes.c_size_t, vp],
        "tsd_hp_connect": [vp, vp],
        "tsd_op_ln_modulate": [vp, i32, i32, vp, vp, i64, i32, i32, vp, vp],
        "tsd_op_qk_norm_rope": [vp, i32, i32, i32, i32, vp, vp, i32, f32, f32, vp, vp, vp, i32, i32, vp],
        "tsd_forward_profile": [vp, i32, vp, i64, vp, vp, i64, vp, i64, vp, i64, vp, i64, vp, vp, vp, i32,
                                ctypes.POINTER(i32), ctypes.POINTER(i32), ctypes.POINTER(i32), ctypes.POINTER(f32),
                                ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)],
    }
    for name, args in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = ctypes.c_int
    L.tsd_plan_op_label.argtypes = [vp, i32]
    L.tsd_plan_op_label.restype = ctypes.c_char_p
    L.tsd_model_free.restype = None
    L.tsd_version.restype = ctypes.c_char_p
    _lib = L
    return L


def check(fn: str, rc: int) -> None:
    if rc != TSD_OK:
        raise TsdError(fn, rc)


def _fp(a: Optional[np.ndarray]):
    if a is None:
        return ctypes.POINTER(ctypes.c_float)()
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"], "float32 C-contiguous arrays expected"
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _stack(items, attr) -> np.ndarray:
    return np.ascontiguousarray(np.stack([np.asarray(getattr(x, attr), np.float32) for x in items]))


IPC_HANDLE_BYTES = 64


def hp_layout(hidden: int, n_head: int, world: int, rank: int):
    """(first head, heads, rows per Q/K/V section) of `rank` in a head-parallel group."""
    out = (ctypes.c_int32 * 3)()
    check("tsd_hp_layout", lib().tsd_hp_layout(hidden, n_head, world, rank, out))
    return int(out[0]), int(out[1]), int(out[2])


class DitModel:
    """A loaded DiT on one GPU (the reference's ts_dit)."""

    def hp_init(self, rank: int, world: int, arena_bytes: int) -> bytes:
        """Head-parallel set-up, step 1: returns this rank's exchange-buffer IPC handle."""
        buf = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
        check("tsd_hp_init", lib().tsd_hp_init(self.h, rank, world, arena_bytes, buf))
        return buf.raw

    def hp_connect(self, handles) -> None:
        """Head-parallel set-up, step 2: every rank's handle, in rank order."""
        blob = b"".join(handles)
        assert len(blob) == IPC_HANDLE_BYTES * len(handles)
        check("tsd_hp_connect", lib().tsd_hp_connect(self.h, ctypes.create_string_buffer(blob, len(blob))))

    def __init__(self, handle: int):
        self.h = ctypes.c_void_p(handle)
        hp = HParams()
        check("tsd_model_get_hparams", lib().tsd_model_get_hparams(self.h, ctypes.byref(hp)))
        self.hparams = hp
        self.latent_dim = hp.latent_dim

    @classmethod
    def load(cls, path: str, device: int = 0) -> "DitModel":
        h = ctypes.c_void_p()
        check("tsd_load_gguf", lib().tsd_load_gguf(path.encode(), device, ctypes.byref(h)))
        return cls(h.value)

    @classmethod
    def from_weights(cls, hp, weights: Dict[str, object], device: int = 0) -> "DitModel":
        """hp: synth.DitHParams; weights: name -> synth.WTensor (ggml bytes, host or torch cuda)."""
        L = lib()
        h = ctypes.c_void_p()
        chp = HParams(hp.hidden, hp.n_head, hp.depth, hp.fused_depth, hp.latent_dim, hp.rope_theta, hp.t_max_period)
        check("tsd_model_create", L.tsd_model_create(ctypes.byref(chp), device, ctypes.byref(h)))
        try:
            for name, t in weights.items():
                ne = (ctypes.c_int64 * 4)(*(list(t.ne) + [1] * (4 - len(t.ne))))
                data = t.data
                if hasattr(data, "data_ptr"):          # torch tensor (device or host)
                    ptr, nbytes = data.data_ptr(), data.numel() * data.element_size()
                else:
                    raw = np.ascontiguousarray(data)
                    ptr, nbytes = raw.ctypes.data, raw.nbytes
                check("tsd_model_set_tensor", L.tsd_model_set_tensor(h, name.encode(), t.type, ne, ctypes.c_void_p(ptr), nbytes))
            check("tsd_model_finalize", L.tsd_model_finalize(h))
        except Exception:
            L.tsd_model_free(h)
            raise
        return cls(h.value)

    def close(self) -> None:
        if self.h:
            lib().tsd_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def get_tensor(self, name: str) -> np.ndarray:
        ne = (ctypes.c_int64 * 4)()
        check("tsd_get_tensor_f32", lib().tsd_get_tensor_f32(self.h, name.encode(), None, 0, ne))
        n = int(np.prod(list(ne)))
        out = np.empty(n, np.float32)
        check("tsd_get_tensor_f32", lib().tsd_get_tensor_f32(self.h, name.encode(), _fp(out), n, ne))
        dims = [int(v) for v in ne]
        while len(dims) > 1 and dims[-1] == 1:      # ggml pads unused trailing dims with 1
            dims.pop()
        return out.reshape(tuple(reversed(dims)))

    def forward(self, items: Sequence, dbg: bool = False):
        """Batched velocity evaluation of synth.DitInputs items -> flow [B][T][latent_dim]."""
        lat = _stack(items, "latent")
        B, _, T = lat.shape
        t = np.asarray([x.t for x in items], np.float32)
        clip, sync, text, t5, gt = (_stack(items, a) for a in ("clip_f", "sync_f", "text_f", "t5", "gtext"))
        out = np.zeros((B, T, self.latent_dim), np.float32)
        store: Dict[str, np.ndarray] = {}

        def cb(_ud, name, ptr, n):
            store[name.decode()] = np.ctypeslib.as_array(ptr, shape=(n,)).copy()

        cbf = DBG_FN(cb) if dbg else DBG_FN()
        rc = lib().tsd_forward_batched(self.h, B, _fp(lat), T, _fp(t), _fp(clip), clip.shape[1], _fp(sync),
                                       sync.shape[1], _fp(text), text.shape[1], _fp(t5), t5.shape[1], _fp(gt),
                                       _fp(out), cbf, None)
        check("tsd_forward_batched", rc)
        return (out, store) if dbg else out

    def forward_inject(self, items: Sequence, inject: Dict[str, np.ndarray]):
        """Teacher-forced forward (tsd_forward_inject): `inject` maps boundary names
        ("blk<i>_in_lat", ..., "final_in_lat") to [B][S][hidden] f32 arrays that replace the
        residual stream before that block. Returns (flow, stages) like forward(dbg=True)."""
        lat = _stack(items, "latent")
        B, _, T = lat.shape
        t = np.asarray([x.t for x in items], np.float32)
        clip, sync, text, t5, gt = (_stack(items, a) for a in ("clip_f", "sync_f", "text_f", "t5", "gtext"))
        out = np.zeros((B, T, self.latent_dim), np.float32)
        store: Dict[str, np.ndarray] = {}

        def cb(_ud, name, ptr, n):
            store[name.decode()] = np.ctypeslib.as_array(ptr, shape=(n,)).copy()

        def inj(_ud, name, ptr, n):
            v = inject.get(name.decode())
            if v is None:
                return 0
            v = np.ascontiguousarray(v, np.float32).reshape(-1)
            assert v.size == n, (name, v.size, n)
            np.ctypeslib.as_array(ptr, shape=(n,))[:] = v
            return 1

        cbf, injf = DBG_FN(cb), INJECT_FN(inj)
        rc = lib().tsd_forward_inject(self.h, B, _fp(lat), T, _fp(t), _fp(clip), clip.shape[1], _fp(sync),
                                      sync.shape[1], _fp(text), text.shape[1], _fp(t5), t5.shape[1], _fp(gt),
                                      _fp(out), cbf, injf, None)
        check("tsd_forward_inject", rc)
        return out, store

    def forward_host(self, B: int, T: int, clip_S: int, sync_S: int, text_S: int, t5_S: int,
                     ptrs: Dict[str, int]) -> None:
        """tsd_forward_batched on caller-owned host buffers given as raw addresses (e.g. pinned
        memory, whose copies the GPU's copy engines run without staging); flow written to
        ptrs["flow"] ([B][T][latent_dim]) before returning."""
        fp = ctypes.POINTER(ctypes.c_float)
        c = lambda k: ctypes.cast(ctypes.c_void_p(ptrs[k]), fp)
        rc = lib().tsd_forward_batched(self.h, B, c("latent"), T, c("t"), c("clip_f"), clip_S, c("sync_f"), sync_S,
                                       c("text_f"), text_S, c("t5"), t5_S, c("gtext"), c("flow"), DBG_FN(), None)
        check("tsd_forward_batched", rc)

    def forward_device(self, B: int, T: int, clip_S: int, sync_S: int, text_S: int, t5_S: int, ptrs: Dict[str, int],
                       stream: int = 0) -> None:
        """Enqueue a forward on device-resident inputs (raw device pointers)."""
        rc = lib().tsd_forward_device(self.h, B, ptrs["latent"], T, ptrs["t"], ptrs["clip_f"], clip_S, ptrs["sync_f"],
                                      sync_S, ptrs["text_f"], text_S, ptrs["t5"], t5_S, ptrs["gtext"], ptrs["flow"],
                                      ctypes.c_void_p(stream))
        check("tsd_forward_device", rc)

    def forward_profile(self, B: int, T: int, clip_S: int, sync_S: int, text_S: int, t5_S: int,
                        ptrs: Dict[str, int], stream: int = 0, max_ops: int = 4096):
        """Per-op kind / launches / ms / FLOPs / bytes of one forward on device-resident inputs."""
        n = ctypes.c_int(0)
        kind = (ctypes.c_int * max_ops)()
        launches = (ctypes.c_int * max_ops)()
        ms = (ctypes.c_float * max_ops)()
        flops = (ctypes.c_double * max_ops)()
        nbytes = (ctypes.c_double * max_ops)()
        rc = lib().tsd_forward_profile(self.h, B, ptrs["latent"], T, ptrs["t"], ptrs["clip_f"], clip_S, ptrs["sync_f"],
                                       sync_S, ptrs["text_f"], text_S, ptrs["t5"], t5_S, ptrs["gtext"], ptrs["flow"],
                                       ctypes.c_void_p(stream), max_ops, ctypes.byref(n), kind, launches, ms, flops,
                                       nbytes)
        check("tsd_forward_profile", rc)
        k = min(n.value, max_ops)
        labels = [(lib().tsd_plan_op_label(self.h, i) or b"").decode() for i in range(k)]
        return dict(kind=np.array(kind[:k]), launches=np.array(launches[:k]), ms=np.array(ms[:k]),
                    flops=np.array(flops[:k]), bytes=np.array(nbytes[:k]), labels=labels)

    def sync_check(self, stream: int = 0) -> None:
        check("tsd_sync_check", lib().tsd_sync_check(self.h, ctypes.c_void_p(stream)))

    def sample(self, items: Sequence, steps: int, cfg: float, want_flow0: bool = False):
        """CFG rectified-flow sampling of P prompts -> latents [P][latent_dim][T] (+ flow0)."""
        noise = _stack(items, "latent")
        P, _, T = noise.shape
        clip, sync, text, t5, gt = (_stack(items, a) for a in ("clip_f", "sync_f", "text_f", "t5", "gtext"))
        out = np.zeros_like(noise)
        f0 = np.zeros_like(noise) if want_flow0 else None
        rc = lib().tsd_sample_batched(self.h, P, _fp(noise), T, _fp(clip), clip.shape[1], _fp(sync), sync.shape[1],
                                      _fp(text), text.shape[1], _fp(t5), t5.shape[1], _fp(gt), steps, cfg, _fp(out),
                                      _fp(f0))
        check("tsd_sample_batched", rc)
        return (out, f0) if want_flow0 else out


# ----------------------------- operator-level wrappers (torch tensors) -----------------------------
def _ptr(t) -> Optional[int]:
    return None if t is None else t.data_ptr()


def op_gemm(W, M, K_in, taps, pad, X, nbatch, S, x_row_stride, x_batch_stride, mode, act, bias, out, out_bf16, ldo,
            resid=None, ldr=0, gate=None, ldg=0, gate_div=1, max_splits=1, m_valid=0, ws=None, counters=None,
            err=None, stream=0):
    """ws: float32 tensor of split-K partials; counters: int32 tensor, zero before first use."""
    rc = lib().tsd_op_gemm(_ptr(W), M, K_in, taps, pad, _ptr(X), nbatch, S, x_row_stride, x_batch_stride, mode, act,
                           _ptr(bias), m_valid, _ptr(out), out_bf16, ldo, _ptr(resid), ldr, _ptr(gate), ldg, gate_div,
                           max_splits, _ptr(ws), 0 if ws is None else ws.numel(), _ptr(counters),
                           0 if counters is None else counters.numel(), _ptr(err), stream)
    check("tsd_op_gemm", rc)


def op_gemm_static(W, M, K_in, taps, pad, X, nbatch, S, x_row_stride, x_batch_stride, mode, act, bias, out, out_bf16,
                   ldo, resid=None, ldr=0, gate=None, ldg=0, gate_div=1, max_splits=8, m_valid=0, err=None, stream=0):
    """op_gemm whose split-K scratch is the library's static device arrays (no allocation)."""
    rc = lib().tsd_op_gemm_static(_ptr(W), M, K_in, taps, pad, _ptr(X), nbatch, S, x_row_stride, x_batch_stride, mode,
                                  act, _ptr(bias), m_valid, _ptr(out), out_bf16, ldo, _ptr(resid), ldr, _ptr(gate), ldg,
                                  gate_div, max_splits, _ptr(err), stream)
    check("tsd_op_gemm_static", rc)


def set_wait_limit(device: int, ns: int) -> None:
    """Deadline of every bounded device-side wait on `device` (default 2 s)."""
    check("tsd_set_wait_limit", lib().tsd_set_wait_limit(device, ns))


def op_peer_wait(counters, epoch, rank, world, ctas, err=None, stream=0):
    check("tsd_op_peer_wait", lib().tsd_op_peer_wait(_ptr(counters), _ptr(epoch), rank, world, ctas, _ptr(err), stream))


GEMM_STATIC_WS_FLOATS, GEMM_STATIC_COUNTERS = 2097152, 8192   # include/tsd_ops.h


def op_gemm_plan(M, K_in, taps, nbatch, S, max_splits=8, ws_floats=0, n_counters=0):
    """The tiling tsd_op_gemm chooses for a shape: dict(BN, splits, pair, csplit, ws_floats, gather)."""
    out = (ctypes.c_int64 * 6)()
    check("tsd_op_gemm_plan", lib().tsd_op_gemm_plan(M, K_in, taps, nbatch, S, max_splits, ws_floats, n_counters, out))
    return dict(BN=int(out[0]), splits=int(out[1]), pair=int(out[2]), csplit=int(out[3]), ws_floats=int(out[4]),
                gather=int(out[5]))


def op_gemv(W, ggml_type, W2, M, K, x, ldx, N, bias, act, round_bf16, y, y_bf16, ldy, stream=0):
    rc = lib().tsd_op_gemv(_ptr(W), ggml_type, _ptr(W2), M, K, _ptr(x), ldx, N, _ptr(bias), act, round_bf16, _ptr(y),
                           y_bf16, ldy, stream)
    check("tsd_op_gemv", rc)


def op_attention(Q, K, V, B, nh, S, out, ldo, err=None, stream=0):
    check("tsd_op_attention", lib().tsd_op_attention(_ptr(Q), _ptr(K), _ptr(V), B, nh, S, _ptr(out), ldo, _ptr(err), stream))


def op_attention_f32(Q, K, V, B, nh, S, out, ldo, err=None, stream=0):
    check("tsd_op_attention_f32",
          lib().tsd_op_attention_f32(_ptr(Q), _ptr(K), _ptr(V), B, nh, S, _ptr(out), ldo, _ptr(err), stream))


def op_ln_modulate(x, rows, H, shift, scale, ld_mod, per_token, rows_per_item, y, stream=0):
    check("tsd_op_ln_modulate", lib().tsd_op_ln_modulate(_ptr(x), rows, H, _ptr(shift), _ptr(scale), ld_mod, per_token,
                                                         rows_per_item, _ptr(y), stream))


def op_qk_norm_rope(qkv, B, S, H, nh, qg, kg, rope, fscale, theta, Q, K, V, Sj, s_off, stream=0):
    check("tsd_op_qk_norm_rope", lib().tsd_op_qk_norm_rope(_ptr(qkv), B, S, H, nh, _ptr(qg), _ptr(kg), rope, fscale,
                                                           theta, _ptr(Q), _ptr(K), _ptr(V), Sj, s_off, stream))
