"""Python binding of the C ABI in include/amoe.h (ctypes over libamoe.so).

The methods mirror the reference's MoE seam (internal/model/gptoss/layer.go:94-123):
``upload_layer`` takes the GGUF-layout tensors that ``loadDecoderLayer`` reads
(weights.go:52-116) and ``forward`` returns the block output plus the routing
that ``MoERouterTopK`` (internal/backend/cpuref/moe.go:12-41) produces.
Errors are raised as ``AmoeError`` carrying the library's message, the way the
Go code returns ``error`` values.  There is no CPU fallback: if libamoe.so is
missing or fails to load, constructing a block raises.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import build as _build

AMOE_OK = 0
AMOE_ERR_INVALID = -1
AMOE_ERR_CUDA = -2
AMOE_ERR_NCCL = -3
AMOE_ERR_TIMEOUT = -4
AMOE_ERR_STATE = -5
AMOE_ERR_NOMEM = -6

PATH_AUTO, PATH_GEMV, PATH_TENSOR = 0, 1, 2

_vp = ctypes.c_void_p
_i32 = ctypes.c_int32


class AmoeConfig(ctypes.Structure):
    _fields_ = [
        ("hidden", _i32),
        ("intermediate", _i32),
        ("experts", _i32),
        ("top_k", _i32),
        ("layers", _i32),
        ("rms_eps", ctypes.c_float),
        ("swiglu_alpha", ctypes.c_float),
        ("swiglu_limit", ctypes.c_float),
        ("max_tokens", _i32),
        ("device", _i32),
        ("stream_slots", _i32),
        ("ep_size", _i32),
        ("ep_rank", _i32),
        ("nccl_id", _vp),
        ("path", _i32),
        ("stream_experts", _i32),
    ]


AMOE_STAGES = 8
STAGE_NAMES = ["route", "scan", "gate_up", "down", "combine", "scatter_gather", "decode_experts", "reserved7"]


class AmoeStats(ctypes.Structure):
    _fields_ = [
        ("launches", ctypes.c_int64),
        ("forwards", ctypes.c_int64),
        ("timed_forwards", ctypes.c_int64),
        ("stage_ms", ctypes.c_double * AMOE_STAGES),
        ("last_path", _i32),
        ("layer_bytes", ctypes.c_int64),
    ]


# Every entry point declared in include/amoe.h: name -> (restype, argtypes)
SIGNATURES = {
    "amoe_abi_version": (ctypes.c_int, []),
    "amoe_create": (ctypes.c_int, [ctypes.POINTER(AmoeConfig), ctypes.POINTER(_vp)]),
    "amoe_destroy": (None, [_vp]),
    "amoe_last_error": (ctypes.c_char_p, [_vp]),
    "amoe_upload_layer": (ctypes.c_int, [_vp, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "amoe_forward": (ctypes.c_int, [_vp, _i32, _vp, _i32, _vp, _vp, _vp]),
    "amoe_forward_device": (ctypes.c_int, [_vp, _i32, _vp, _i32, _vp, _vp, _vp, _vp]),
    "amoe_synchronize": (ctypes.c_int, [_vp]),
    "amoe_prefetch_layer": (ctypes.c_int, [_vp, _i32]),
    "amoe_last_routing": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp]),
    "amoe_set_profiling": (ctypes.c_int, [_vp, _i32]),
    "amoe_get_stats": (ctypes.c_int, [_vp, ctypes.POINTER(AmoeStats), _i32]),
    "amoe_ep_unique_id": (ctypes.c_int, [_vp]),
    "amoe_ep_layout": (ctypes.c_int, [_i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp]),
    "amoe_decode_schedule": (ctypes.c_int, [_i32, _i32, _i32, _i32, _i32, _vp]),
    "amoe_route_noalloc": (ctypes.c_int, [_i32, _i32, _i32, _i32, ctypes.c_float, _vp, _i32, _vp, _vp, _vp,
                                          _vp, _vp, _vp, _vp]),
    "amoe_gguf_open": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(_vp)]),
    "amoe_gguf_close": (None, [_vp]),
    "amoe_gguf_tensor": (ctypes.c_int, [_vp, ctypes.c_char_p, _vp, _vp, _vp, _vp, _vp]),
    "amoe_gguf_moe_config": (ctypes.c_int, [_vp, ctypes.POINTER(AmoeConfig)]),
    "amoe_upload_layer_gguf": (ctypes.c_int, [_vp, _vp, _i32]),
    "amoe_head_create": (ctypes.c_int, [_i32, _i32, ctypes.c_float, _i32, ctypes.POINTER(_vp)]),
    "amoe_head_destroy": (None, [_vp]),
    "amoe_head_last_error": (ctypes.c_char_p, [_vp]),
    "amoe_head_upload": (ctypes.c_int, [_vp, _vp, _vp, _i32]),
    "amoe_head_upload_gguf": (ctypes.c_int, [_vp, _vp]),
    "amoe_head_next_token": (ctypes.c_int, [_vp, _vp, _i32, _vp, _vp]),
    "amoe_head_next_token_device": (ctypes.c_int, [_vp, _vp, _i32, _vp, _vp, _vp]),
}

GGUF_F32, GGUF_F16, GGUF_BF16, GGUF_MXFP4 = 0, 1, 30, 39

_lib = None


def library_path() -> str:
    return _build.LIB


def load_library(build_if_missing: bool = True):
    """Load libamoe.so (building it in-tree with nvcc if it is absent or stale)."""
    global _lib
    if _lib is None:
        path = _build.build() if build_if_missing else _build.LIB
        if not os.path.exists(path):
            raise RuntimeError(f"libamoe.so not found at {path}; run airllm_b200/build.py")
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


class AmoeError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"amoe error {code}: {message}")
        self.code = code


def _ptr(a) -> int | None:
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    return a.data_ptr()  # torch tensor


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def ep_unique_id() -> bytes:
    """A fresh 128-byte NCCL unique id for an expert-parallel group (rank 0 makes it)."""
    lib = load_library()
    buf = ctypes.create_string_buffer(128)
    rc = lib.amoe_ep_unique_id(buf)
    if rc != AMOE_OK:
        raise AmoeError(rc, lib.amoe_last_error(None).decode())
    return buf.raw


def ep_layout(n_ranks: int, experts_per_rank: int, rank: int, table) -> dict:
    """Layout of one expert-parallel exchange from the count table [N][E]
    (amoe_ep_layout; the arithmetic the device runs, here on the host)."""
    lib = load_library()
    N, El = n_ranks, experts_per_rank
    tab = np.ascontiguousarray(table, np.int32)
    if tab.shape != (N, N * El):
        raise AmoeError(AMOE_ERR_INVALID, f"table must be [{N}][{N * El}]")
    out = {"send_base": np.zeros(N * El, np.int32), "offsets_loc": np.zeros(El + 1, np.int32),
           "seg_start": np.zeros(El * N, np.int32), "src_pos": np.zeros(El * N, np.int32)}
    rc = lib.amoe_ep_layout(N, El, rank, tab.ctypes.data, *[out[k].ctypes.data for k in
                            ("send_base", "offsets_loc", "seg_start", "src_pos")])
    if rc != AMOE_OK:
        raise AmoeError(rc, lib.amoe_last_error(None).decode())
    out["seg_start"] = out["seg_start"].reshape(El, N)
    out["src_pos"] = out["src_pos"].reshape(El, N)
    return out


DECODE_SCHED_WORDS = 1024


def decode_schedule(hidden: int, intermediate: int, experts: int, top_k: int, ctas: int) -> np.ndarray:
    """The fused decode kernel's work table [ctas][DECODE_SCHED_WORDS]
    (amoe_decode_schedule; host arithmetic, no GPU needed)."""
    lib = load_library()
    rows = np.zeros((ctas, DECODE_SCHED_WORDS), np.int32)
    rc = lib.amoe_decode_schedule(hidden, intermediate, experts, top_k, ctas, rows.ctypes.data)
    if rc != AMOE_OK:
        raise AmoeError(rc, lib.amoe_last_error(None).decode())
    return rows


class GGUFFile:
    """An open GGUF file (amoe_gguf_open): the tensor index and the MoE metadata of a
    GPT-OSS model, as internal/gguf/reader.go and gptoss.go read them."""

    def __init__(self, path: str):
        self._lib = load_library()
        h = _vp()
        rc = self._lib.amoe_gguf_open(os.fsencode(path), ctypes.byref(h))
        if rc != AMOE_OK:
            raise AmoeError(rc, self._lib.amoe_last_error(None).decode())
        self._h = h

    @property
    def handle(self):
        return self._h

    def tensor(self, name: str) -> dict:
        """{"type", "shape", "offset", "bytes"} of one tensor (shape[0] varies fastest)."""
        t, nd = _i32(), _i32()
        dims = (ctypes.c_int64 * 4)()
        off, nbytes = ctypes.c_int64(), ctypes.c_int64()
        rc = self._lib.amoe_gguf_tensor(self._h, name.encode(), ctypes.byref(t), ctypes.byref(nd), dims,
                                        ctypes.byref(off), ctypes.byref(nbytes))
        if rc != AMOE_OK:
            raise AmoeError(rc, self._lib.amoe_last_error(None).decode())
        return {"type": t.value, "shape": [dims[i] for i in range(min(nd.value, 4))], "offset": off.value,
                "bytes": nbytes.value}

    def moe_config(self) -> dict:
        """hidden, intermediate, experts, top_k, layers, rms_eps from the GPT-OSS metadata."""
        cfg = AmoeConfig()
        rc = self._lib.amoe_gguf_moe_config(self._h, ctypes.byref(cfg))
        if rc != AMOE_OK:
            raise AmoeError(rc, self._lib.amoe_last_error(None).decode())
        return {k: getattr(cfg, k) for k in ("hidden", "intermediate", "experts", "top_k", "layers", "rms_eps")}

    def close(self):
        if self._h:
            self._lib.amoe_gguf_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class MoEBlock:
    """One B200 MoE-block context (amoe_ctx): weights for `layers` layers plus scratch."""

    def __init__(self, hidden: int, intermediate: int, experts: int, top_k: int, layers: int = 1,
                 max_tokens: int = 4096, eps: float = 1e-5, device: int = 0, stream_slots: int = 0,
                 path: int = PATH_AUTO, ep_size: int = 1, ep_rank: int = 0, nccl_id: bytes | None = None,
                 stream_experts: int = 0):
        self._lib = load_library()
        self.hidden, self.intermediate, self.experts, self.top_k = hidden, intermediate, experts, top_k
        self.layers, self.max_tokens = layers, max_tokens
        self._nccl_id = ctypes.create_string_buffer(nccl_id, 128) if nccl_id is not None else None
        cfg = AmoeConfig(hidden, intermediate, experts, top_k, layers, eps, 1.702, 7.0, max_tokens, device,
                         stream_slots, ep_size, ep_rank,
                         ctypes.cast(self._nccl_id, _vp) if self._nccl_id is not None else None, path,
                         stream_experts)
        h = _vp()
        rc = self._lib.amoe_create(ctypes.byref(cfg), ctypes.byref(h))
        if rc != AMOE_OK:
            raise AmoeError(rc, self._lib.amoe_last_error(None).decode())
        self._h = h

    @classmethod
    def for_layer(cls, layer: dict, **kw) -> "MoEBlock":
        blk = cls(layer["hidden"], layer["intermediate"], layer["experts"], layer["top_k"],
                  eps=layer.get("eps", 1e-5), **kw)
        return blk

    def _check(self, rc: int):
        if rc != AMOE_OK:
            raise AmoeError(rc, self._lib.amoe_last_error(self._h).decode())

    def close(self):
        if getattr(self, "_h", None):
            self._lib.amoe_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def upload_layer(self, index: int, layer: dict):
        arrs = [
            _c(layer["norm_gain"], np.float32), _c(layer["router_w"], np.float32),
            _c(layer["router_b"], np.float32), _c(layer["gate_up"], np.uint8),
            _c(layer["gate_up_b"], np.float32), _c(layer["down"], np.uint8), _c(layer["down_b"], np.float32),
        ]
        H, I, E = self.hidden, self.intermediate, self.experts
        want = [H, E * H, E, E * 2 * I * (H // 32) * 17, E * 2 * I, E * H * (I // 32) * 17, E * H]
        for a, n in zip(arrs, want):
            if a.size != n:
                raise AmoeError(AMOE_ERR_INVALID, f"tensor length {a.size}, want {n}")
        self._check(self._lib.amoe_upload_layer(self._h, index, *[a.ctypes.data for a in arrs]))

    def upload_layer_gguf(self, index: int, gguf: "GGUFFile"):
        """Layer `index` of a GGUF file into slot `index` (amoe_upload_layer_gguf)."""
        self._check(self._lib.amoe_upload_layer_gguf(self._h, gguf.handle, index))

    def forward(self, residual, layer: int = 0):
        """Host-buffer forward (amoe_forward).  Returns (out, topk_idx, topk_w)."""
        x = _c(residual, np.float32)
        T = x.shape[0]
        out = np.empty_like(x)
        idx = np.empty((T, self.top_k), np.int32)
        w = np.empty((T, self.top_k), np.float32)
        self._check(self._lib.amoe_forward(self._h, layer, x.ctypes.data, T, out.ctypes.data,
                                           idx.ctypes.data, w.ctypes.data))
        return out, idx, w

    def forward_into(self, residual, out, layer: int = 0, topk_idx=None, topk_w=None):
        """Host-buffer forward into caller-owned (e.g. pinned) arrays."""
        T = residual.shape[0]
        self._check(self._lib.amoe_forward(self._h, layer, _ptr(residual), T, _ptr(out),
                                           _ptr(topk_idx), _ptr(topk_w)))

    def forward_device(self, residual, out, layer: int = 0, topk_idx=None, topk_w=None, stream=None):
        """Device-buffer forward on torch CUDA tensors (amoe_forward_device); asynchronous."""
        T = residual.shape[0]
        st = None
        if stream is not None:
            st = stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)
            if st == 0:
                st = 1  # torch's default stream is the legacy stream (cudaStreamLegacy); NULL means "own stream"
        self._check(self._lib.amoe_forward_device(self._h, layer, _ptr(residual), T, _ptr(out),
                                                  _ptr(topk_idx), _ptr(topk_w), st))

    def synchronize(self):
        self._check(self._lib.amoe_synchronize(self._h))

    def prefetch_layer(self, index: int):
        self._check(self._lib.amoe_prefetch_layer(self._h, index))

    def set_profiling(self, on: bool):
        self._check(self._lib.amoe_set_profiling(self._h, 1 if on else 0))

    def stats(self, reset: bool = False) -> dict:
        st = AmoeStats()
        self._check(self._lib.amoe_get_stats(self._h, ctypes.byref(st), 1 if reset else 0))
        return {
            "launches": st.launches, "forwards": st.forwards, "timed_forwards": st.timed_forwards,
            "stage_ms": {STAGE_NAMES[i]: st.stage_ms[i] for i in range(AMOE_STAGES)},
            "last_path": st.last_path,
            "layer_bytes": st.layer_bytes,
        }

    def last_routing(self, T: int):
        """(logits [T,E], perm_pair [T*k], counts [E], offsets [E+1]) of the last forward."""
        logits = np.empty((T, self.experts), np.float32)
        perm = np.empty(T * self.top_k, np.int32)
        counts = np.empty(self.experts, np.int32)
        offsets = np.empty(self.experts + 1, np.int32)
        self._check(self._lib.amoe_last_routing(self._h, logits.ctypes.data, perm.ctypes.data,
                                                counts.ctypes.data, offsets.ctypes.data))
        return logits, perm, counts, offsets


class Head:
    """The model head (amoe_head): final RMSNorm, lm_head and greedy token choice,
    as Runtime.nextToken does it (internal/model/gptoss/runtime.go:234-250)."""

    MAX_TOKENS = 16

    def __init__(self, hidden: int, vocab: int, eps: float = 1e-5, device: int = 0):
        self._lib = load_library()
        self.hidden, self.vocab = hidden, vocab
        h = _vp()
        rc = self._lib.amoe_head_create(hidden, vocab, eps, device, ctypes.byref(h))
        if rc != AMOE_OK:
            raise AmoeError(rc, self._lib.amoe_head_last_error(None).decode())
        self._h = h

    def _check(self, rc: int):
        if rc != AMOE_OK:
            raise AmoeError(rc, self._lib.amoe_head_last_error(self._h).decode())

    def upload(self, final_norm, lm_head, gguf_type: int = GGUF_F32):
        """final_norm [H] f32; lm_head [V, H] as f32 (GGUF_F32), or its raw 16-bit words
        (uint16/float16 array) for GGUF_F16 / GGUF_BF16."""
        g = _c(final_norm, np.float32)
        if g.size != self.hidden:
            raise AmoeError(AMOE_ERR_INVALID, f"final norm length {g.size}, want {self.hidden}")
        w = np.ascontiguousarray(lm_head)
        want = 4 if gguf_type == GGUF_F32 else 2
        if w.size != self.vocab * self.hidden or w.itemsize != want:
            raise AmoeError(AMOE_ERR_INVALID, "lm head must hold vocab x hidden elements of its encoding")
        self._check(self._lib.amoe_head_upload(self._h, g.ctypes.data, w.ctypes.data, gguf_type))

    def upload_gguf(self, gguf: "GGUFFile"):
        self._check(self._lib.amoe_head_upload_gguf(self._h, gguf.handle))

    def next_token(self, hidden, want_logits: bool = False):
        """hidden [T, H] host rows -> tokens [T] (and logits [T, V])."""
        x = _c(hidden, np.float32).reshape(-1, self.hidden)
        T = x.shape[0]
        tokens = np.empty(T, np.int32)
        logits = np.empty((T, self.vocab), np.float32) if want_logits else None
        self._check(self._lib.amoe_head_next_token(self._h, x.ctypes.data, T, tokens.ctypes.data,
                                                   logits.ctypes.data if want_logits else None))
        return (tokens, logits) if want_logits else tokens

    def next_token_device(self, hidden, tokens, logits=None, stream=None):
        """Device-buffer call on torch tensors; asynchronous."""
        st = None
        if stream is not None:
            st = stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)
            if st == 0:
                st = 1
        self._check(self._lib.amoe_head_next_token_device(self._h, _ptr(hidden), hidden.shape[0], _ptr(tokens),
                                                          _ptr(logits), st))

    def close(self):
        if getattr(self, "_h", None):
            self._lib.amoe_head_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
