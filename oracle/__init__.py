"""CPU oracle for the GPT-OSS MoE block -- TEST INFRASTRUCTURE ONLY.

A C restatement (moe_oracle.c) of the reference Go CPU path, loaded through
ctypes.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline and
reference legs import this package; the product library never does.

Reference functions restated (paths relative to the reference project root):
  RMSNorm            internal/backend/cpuref/primitives.go:50-72
  Linear/LinearBias  internal/backend/cpuref/primitives.go:11-47
  MoERouterTopK      internal/backend/cpuref/moe.go:12-41
  GPTOSSSwiGLU       internal/backend/cpuref/primitives.go:138-149
  MXFP4 decode       internal/model/gptoss/tensor.go:145-170, gguf/reader.go:442-449
  MoE block          internal/model/gptoss/layer.go:94-188 (token by token, or
                     expert-major with the same arithmetic: moe_block_grouped)
  FP4 activation terms  no reference counterpart: the bit-exact E2M1-term operand of a
                     block-scaled FP4 GEMM (oracle_e2m1_terms in moe_oracle.c)
  Runtime.nextToken  internal/model/gptoss/runtime.go:234-250 (final RMSNorm,
                     lm_head Linear, first-max argmax)
  RoPE / YaRNRoPE    internal/backend/cpuref/rope.go:10-86           (attn_oracle.c)
  KVCache            internal/backend/cpuref/attention.go:8-59       (KVCache below)
  CausalAttention    internal/backend/cpuref/attention.go:61-171     (attn_oracle.c)
  attention half     internal/model/gptoss/layer.go:31-92, 189-207   (attn_oracle.c)
  layer window       internal/model/gptoss/weights.go:118-122
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lock = threading.Lock()
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)
_u8p = ctypes.POINTER(ctypes.c_uint8)


class OracleLayer(ctypes.Structure):
    _fields_ = [
        ("hidden", ctypes.c_int32),
        ("intermediate", ctypes.c_int32),
        ("experts", ctypes.c_int32),
        ("top_k", ctypes.c_int32),
        ("eps", ctypes.c_float),
        ("norm_gain", _f32p),
        ("router_w", _f32p),
        ("router_b", _f32p),
        ("gate_up", _u8p),
        ("gate_up_b", _f32p),
        ("down", _u8p),
        ("down_b", _f32p),
    ]


class OracleAttnLayer(ctypes.Structure):
    _fields_ = [
        ("hidden", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("eps", ctypes.c_float),
        ("theta", ctypes.c_double),
        ("norm1", _f32p),
        ("qkv_w", _f32p),
        ("qkv_b", _f32p),
        ("out_w", _f32p),
        ("out_b", _f32p),
        ("sinks", _f32p),
    ]


def build() -> str:
    """Compile liboracle.so with the committed Makefile (gcc, OpenMP)."""
    src = [os.path.join(_HERE, f) for f in ("moe_oracle.c", "moe_oracle.h", "attn_oracle.c", "attn_oracle.h",
                                            "Makefile")]
    if os.path.exists(_LIB_PATH) and all(
        os.path.getmtime(_LIB_PATH) >= os.path.getmtime(s) for s in src
    ):
        return _LIB_PATH
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    with _lock:
        if _lib is None:
            build()
            L = ctypes.CDLL(_LIB_PATH)
            L.oracle_rmsnorm.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_float, _f32p]
            L.oracle_linear_bias.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int, _f32p]
            L.oracle_router_topk.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, _i32p, _f32p]
            L.oracle_swiglu.argtypes = [_f32p, _f32p, ctypes.c_int, _f32p]
            L.oracle_mxfp4_decode.argtypes = [_u8p, ctypes.c_int64, ctypes.c_int64, _f32p]
            L.oracle_mxfp4_encoded_size.argtypes = [ctypes.c_int64]
            L.oracle_mxfp4_encoded_size.restype = ctypes.c_int64
            L.oracle_moe_block.argtypes = [
                ctypes.POINTER(OracleLayer), _f32p, ctypes.c_int, _f32p, _i32p, _f32p, _f32p,
                _i32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
            ]
            L.oracle_moe_block_grouped.argtypes = [
                ctypes.POINTER(OracleLayer), _f32p, ctypes.c_int, _f32p, _i32p, _f32p, _f32p,
                _i32p, ctypes.c_int, ctypes.c_int,
            ]
            L.oracle_route.argtypes = [
                ctypes.POINTER(OracleLayer), _f32p, ctypes.c_int, _f32p, _i32p, _f32p, ctypes.c_int,
            ]
            L.oracle_expert_rows.argtypes = [ctypes.POINTER(OracleLayer), ctypes.c_int, _f32p, ctypes.c_int,
                                             _f32p, ctypes.c_int]
            L.oracle_permute.argtypes = [_i32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                         _i32p, _i32p, _i32p, _i32p]
            L.oracle_next_token.argtypes = [_f32p, ctypes.c_int, _f32p, ctypes.c_float, _f32p, ctypes.c_int, _f32p,
                                            _i32p]
            L.oracle_e2m1_terms.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int, _u8p, _u8p]
            L.oracle_rope.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_double,
                                      ctypes.c_int, _f32p]
            L.oracle_causal_attention.argtypes = [
                _f32p, ctypes.c_int64, ctypes.c_int, _f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_double, ctypes.c_double, _f32p,
            ]
            L.oracle_attention_half.argtypes = [
                ctypes.POINTER(OracleAttnLayer), _f32p, ctypes.c_int, _f32p, _f32p, ctypes.POINTER(ctypes.c_int),
                ctypes.c_int, ctypes.c_int, _f32p,
            ]
            _lib = L
    return _lib


def _p(a: np.ndarray, ty):
    return a.ctypes.data_as(ty) if a is not None else None


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


class OracleError(RuntimeError):
    pass


def _check(rc: int, what: str):
    if rc != 0:
        raise OracleError(f"oracle {what} rejected its arguments")


def rmsnorm(x, g, eps):
    x, g = _c(x, np.float32), _c(g, np.float32)
    out = np.empty_like(x)
    _check(lib().oracle_rmsnorm(_p(x, _f32p), _p(g, _f32p), x.size, eps, _p(out, _f32p)), "rmsnorm")
    return out


def linear_bias(x, w, b, in_dim, out_dim):
    x, w = _c(x, np.float32), _c(w, np.float32)
    b = _c(b, np.float32) if b is not None else None
    if x.size != in_dim or w.size != in_dim * out_dim or (b is not None and b.size != out_dim):
        raise OracleError("linear length mismatch")
    y = np.empty(out_dim, np.float32)
    _check(lib().oracle_linear_bias(_p(x, _f32p), _p(w, _f32p), _p(b, _f32p) if b is not None else None,
                                    in_dim, out_dim, _p(y, _f32p)), "linear")
    return y


def router_topk(logits, k):
    logits = _c(logits, np.float32)
    idx = np.empty(max(k, 0), np.int32)
    w = np.empty(max(k, 0), np.float32)
    _check(lib().oracle_router_topk(_p(logits, _f32p), logits.size, k, _p(idx, _i32p), _p(w, _f32p)),
           "router_topk")
    return idx, w


def swiglu(gate, up):
    gate, up = _c(gate, np.float32), _c(up, np.float32)
    if gate.size != up.size:
        raise OracleError("swiglu lengths differ")
    out = np.empty_like(gate)
    lib().oracle_swiglu(_p(gate, _f32p), _p(up, _f32p), gate.size, _p(out, _f32p))
    return out


def mxfp4_encoded_size(elements: int) -> int:
    n = lib().oracle_mxfp4_encoded_size(elements)
    if n < 0:
        raise OracleError("MXFP4 element count must be divisible by 32")
    return n


def mxfp4_decode(data, elements):
    data = _c(np.frombuffer(bytes(data), np.uint8) if isinstance(data, (bytes, bytearray)) else data, np.uint8)
    out = np.empty(elements, np.float32)
    _check(lib().oracle_mxfp4_decode(_p(data, _u8p), data.size, elements, _p(out, _f32p)), "mxfp4_decode")
    return out


class _Layer:
    """Keeps the numpy arrays alive for as long as the ctypes struct is used."""

    def __init__(self, layer: dict):
        self.arrays = {
            "norm_gain": _c(layer["norm_gain"], np.float32),
            "router_w": _c(layer["router_w"], np.float32),
            "router_b": _c(layer["router_b"], np.float32),
            "gate_up": _c(layer["gate_up"], np.uint8),
            "gate_up_b": _c(layer["gate_up_b"], np.float32),
            "down": _c(layer["down"], np.uint8),
            "down_b": _c(layer["down_b"], np.float32),
        }
        a = self.arrays
        self.s = OracleLayer(
            layer["hidden"], layer["intermediate"], layer["experts"], layer["top_k"], layer["eps"],
            _p(a["norm_gain"], _f32p), _p(a["router_w"], _f32p), _p(a["router_b"], _f32p),
            _p(a["gate_up"], _u8p), _p(a["gate_up_b"], _f32p), _p(a["down"], _u8p),
            _p(a["down_b"], _f32p),
        )


def moe_block(layer: dict, residual, tokens=None, faithful=False, threads=None):
    """Run the reference MoE block.  Returns (out, topk_idx, topk_w, logits).

    tokens: optional row indices to compute (others stay NaN / -1)."""
    L = _Layer(layer)
    res = _c(residual, np.float32)
    T = res.shape[0]
    H, k, E = layer["hidden"], layer["top_k"], layer["experts"]
    out = np.full((T, H), np.nan, np.float32)
    idx = np.full((T, k), -1, np.int32)
    w = np.full((T, k), np.nan, np.float32)
    logits = np.full((T, E), np.nan, np.float32)
    tok = _c(tokens, np.int32) if tokens is not None else None
    threads = threads or os.cpu_count() or 1
    rc = lib().oracle_moe_block(ctypes.byref(L.s), _p(res, _f32p), T, _p(out, _f32p), _p(idx, _i32p),
                                _p(w, _f32p), _p(logits, _f32p), _p(tok, _i32p) if tok is not None else None,
                                0 if tok is None else tok.size, 1 if faithful else 0, threads)
    _check(rc, "moe_block")
    return out, idx, w, logits


def moe_block_grouped(layer: dict, residual, tokens=None, threads=None):
    """moe_block evaluated expert by expert (oracle_moe_block_grouped): the same
    (out, topk_idx, topk_w, logits), bit for bit, fast enough for full prefill
    outputs.  tokens: optional row indices to compute (others stay NaN / -1)."""
    L = _Layer(layer)
    res = _c(residual, np.float32)
    T = res.shape[0]
    H, k, E = layer["hidden"], layer["top_k"], layer["experts"]
    out = np.full((T, H), np.nan, np.float32)
    idx = np.full((T, k), -1, np.int32)
    w = np.full((T, k), np.nan, np.float32)
    logits = np.full((T, E), np.nan, np.float32)
    tok = _c(tokens, np.int32) if tokens is not None else None
    rc = lib().oracle_moe_block_grouped(ctypes.byref(L.s), _p(res, _f32p), T, _p(out, _f32p), _p(idx, _i32p),
                                        _p(w, _f32p), _p(logits, _f32p),
                                        _p(tok, _i32p) if tok is not None else None,
                                        0 if tok is None else tok.size, threads or os.cpu_count() or 1)
    _check(rc, "moe_block_grouped")
    return out, idx, w, logits


def route(layer: dict, residual, threads=None):
    """Router only for all rows: (logits, topk_idx, topk_w)."""
    L = _Layer(layer)
    res = _c(residual, np.float32)
    T = res.shape[0]
    k, E = layer["top_k"], layer["experts"]
    logits = np.empty((T, E), np.float32)
    idx = np.empty((T, k), np.int32)
    w = np.empty((T, k), np.float32)
    rc = lib().oracle_route(ctypes.byref(L.s), _p(res, _f32p), T, _p(logits, _f32p), _p(idx, _i32p),
                            _p(w, _f32p), threads or os.cpu_count() or 1)
    _check(rc, "route")
    return logits, idx, w


def expert_rows(layer: dict, expert: int, x_norm, threads=None):
    """forwardExpert of `expert` on normalized rows x_norm [n, H] -> y [n, H]."""
    L = _Layer(layer)
    x = _c(x_norm, np.float32).reshape(-1, layer["hidden"])
    y = np.empty_like(x)
    _check(lib().oracle_expert_rows(ctypes.byref(L.s), expert, _p(x, _f32p), x.shape[0], _p(y, _f32p),
                                    threads or os.cpu_count() or 1), "expert_rows")
    return y


def normalize_rows(layer: dict, residual):
    """RMSNorm of every row with the layer's gain (primitives.go:50-72)."""
    res = _c(residual, np.float32)
    return np.stack([rmsnorm(r, layer["norm_gain"], layer["eps"]) for r in res]) if len(res) else res


def permute(topk_idx, experts):
    """Stable (expert, token, slot) order: (perm_pair, counts, offsets, inv)."""
    idx = _c(topk_idx, np.int32)
    T, k = idx.shape
    perm = np.empty(T * k, np.int32)
    counts = np.empty(experts, np.int32)
    offsets = np.empty(experts + 1, np.int32)
    inv = np.empty(T * k, np.int32)
    _check(lib().oracle_permute(_p(idx, _i32p), T, k, experts, _p(perm, _i32p), _p(counts, _i32p),
                                _p(offsets, _i32p), _p(inv, _i32p)), "permute")
    return perm, counts, offsets, inv


# ---- the model head -------------------------------------------------------------------

def next_token(hidden, gain, eps, lm_head):
    """Runtime.nextToken (runtime.go:234-250) on one hidden row: (token, logits).
    lm_head [V, H] float32 (decoded from the GGUF encoding first, as the reference does)."""
    hidden, gain = _c(hidden, np.float32).ravel(), _c(gain, np.float32).ravel()
    W = _c(lm_head, np.float32)
    V, H = W.shape
    if hidden.size != H or gain.size != H:
        raise OracleError("head lengths do not match")
    logits = np.empty(V, np.float32)
    tok = np.zeros(1, np.int32)
    _check(lib().oracle_next_token(_p(hidden, _f32p), H, _p(gain, _f32p), eps, _p(W, _f32p), V, _p(logits, _f32p),
                                   _p(tok, _i32p)), "next_token")
    return int(tok[0]), logits


# ---- block-scaled FP4 activation terms ------------------------------------------------

_E2M1 = np.array([0, 0.5, 1, 1.5, 2, 3, 4, 6], np.float64)


def e2m1_terms(x, terms: int):
    """x (length a multiple of 32) as `terms` E2M1 terms with E8M0 scales per 32
    elements (oracle_e2m1_terms): codes [terms][n/2] (low nibble first) and
    scales [terms][n/32]."""
    x = _c(x, np.float32).ravel()
    codes = np.empty((terms, x.size // 2), np.uint8)
    scales = np.empty((terms, x.size // 32), np.uint8)
    _check(lib().oracle_e2m1_terms(_p(x, _f32p), x.size, terms, _p(codes, _u8p), _p(scales, _u8p)), "e2m1_terms")
    return codes, scales


def e2m1_reconstruct(codes, scales):
    """sum_j q_j 2^(s_j - 127) in float64 from e2m1_terms' output."""
    codes, scales = np.asarray(codes, np.uint8), np.asarray(scales, np.uint8)
    nib = np.stack([codes & 15, codes >> 4], -1).reshape(codes.shape[0], -1)
    val = np.where(nib & 8, -1.0, 1.0) * _E2M1[nib & 7]
    scale = np.ldexp(1.0, scales.astype(np.int64) - 127).repeat(32, axis=1)
    return (val * scale).sum(0)


# ---- the attention half -------------------------------------------------------------

_ROPE_ERRORS = {-1: "rope head dimension must be positive and even",
                -2: "rope position offset must be non-negative",
                -3: "rope theta must be finite and positive",
                -4: "rope input length is not divisible by the head dimension"}


def _rope(x, head_dim, pos_offset, theta, yarn):
    x = _c(x, np.float32).ravel()
    out = np.empty_like(x)
    rc = lib().oracle_rope(_p(x, _f32p), x.size, head_dim, pos_offset, theta, 1 if yarn else 0, _p(out, _f32p))
    if rc != 0:
        raise OracleError(_ROPE_ERRORS.get(rc, f"rope rejected its arguments ({rc})"))
    return out


def rope(x, head_dim, pos_offset, theta):
    """RoPE (rope.go:10-13): rotate-half rotary embedding of [tokens, head_dim]."""
    return _rope(x, head_dim, pos_offset, theta, False)


def yarn_rope(x, head_dim, pos_offset, theta):
    """YaRNRoPE (rope.go:15-44): the gpt-oss YaRN frequencies and concentration."""
    return _rope(x, head_dim, pos_offset, theta, True)


class KVCache:
    """KVCache (attention.go:8-59): keys and values [capacity, kv_heads, head_dim];
    Append is transactional (a rejected append leaves the cache unchanged)."""

    def __init__(self, kv_heads: int, head_dim: int, capacity: int):
        if kv_heads <= 0 or head_dim <= 0 or capacity <= 0:
            raise OracleError("kv cache dimensions must be positive")
        self.kv_heads, self.head_dim, self.capacity, self.length = kv_heads, head_dim, capacity, 0
        self.keys = np.zeros(capacity * kv_heads * head_dim, np.float32)
        self.values = np.zeros_like(self.keys)

    def append(self, keys, values, seq: int):
        if seq <= 0:
            raise OracleError("kv append sequence length must be positive")
        if self.length + seq > self.capacity:
            raise OracleError("kv append exceeds capacity")
        keys, values = _c(keys, np.float32).ravel(), _c(values, np.float32).ravel()
        want = seq * self.kv_heads * self.head_dim
        if keys.size != want or values.size != want:
            raise OracleError("kv append lengths do not match")
        start = self.length * self.kv_heads * self.head_dim
        self.keys[start:start + want] = keys
        self.values[start:start + want] = values
        self.length += seq


_ATTN_ERRORS = {-1: "attention query heads must be a positive multiple of kv heads",
                -2: "attention sinks length does not match the query heads",
                -3: "attention sliding window must be non-negative",
                -4: "attention query pre-attention scalar must be finite and non-negative",
                -5: "attention logit softcap must be finite and non-negative",
                -6: "attention query length is not a non-empty multiple of the query width",
                -7: "attention query length exceeds cached length",
                -10: "prefill sequence length must be positive",
                -11: "kv append exceeds capacity"}


def causal_attention(query, q_heads: int, cache: KVCache, sinks=None, window: int = 0,
                     pre_scalar: float = 0.0, softcap: float = 0.0):
    """CausalAttentionWithConfig (attention.go:82-171) on the last query tokens."""
    if cache is None:
        raise OracleError("attention cache must not be nil")
    q = _c(query, np.float32).ravel()
    s = _c(sinks, np.float32).ravel() if sinks is not None else None
    out = np.empty_like(q)
    rc = lib().oracle_causal_attention(_p(q, _f32p), q.size, q_heads, _p(cache.keys, _f32p),
                                       _p(cache.values, _f32p), cache.length, cache.kv_heads, cache.head_dim,
                                       _p(s, _f32p), 0 if s is None else s.size, window, pre_scalar, softcap,
                                       _p(out, _f32p))
    if rc != 0:
        raise OracleError(_ATTN_ERRORS.get(rc, f"attention rejected its arguments ({rc})"))
    return out


def layer_window(index: int, sliding_window: int) -> int:
    """loadDecoderLayer's window rule (weights.go:118-122): even layers slide."""
    return sliding_window if index % 2 == 0 else 0


def attention_half(layer: dict, x, cache: KVCache, window: int):
    """The attention half of DecoderLayer.forward (layer.go:31-92) for the rows x
    [T, hidden]: returns input + o_proj(attention(YaRN(q), YaRN(k) appended, v))."""
    x = _c(x, np.float32).reshape(-1, layer["hidden"])
    keep = {k: _c(layer[k], np.float32) for k in ("norm1", "qkv_w", "qkv_b", "out_w", "out_b", "sinks")}
    L = OracleAttnLayer(layer["hidden"], layer["heads"], layer["kv_heads"], layer["head_dim"], layer["eps"],
                        layer["theta"], *[_p(keep[k], _f32p) for k in ("norm1", "qkv_w", "qkv_b", "out_w",
                                                                        "out_b", "sinks")])
    out = np.empty_like(x)
    n = ctypes.c_int(cache.length)
    rc = lib().oracle_attention_half(ctypes.byref(L), _p(x, _f32p), x.shape[0], _p(cache.keys, _f32p),
                                     _p(cache.values, _f32p), ctypes.byref(n), cache.capacity, window,
                                     _p(out, _f32p))
    if rc != 0:
        raise OracleError(_ATTN_ERRORS.get(rc, f"attention half rejected its arguments ({rc})"))
    cache.length = n.value
    return out

