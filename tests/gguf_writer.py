"""Writes small GGUF files for the tests (little-endian, v2 or v3).

The layout follows the GGUF format as the reference's own test fixture writer lays
it out (internal/gguf/gguf_test.go:237-277): magic, version, tensor count, metadata
count, metadata sorted by key, tensor infos with offsets rounded up to the
alignment, padding, then the tensor data at those offsets."""
import struct

import numpy as np

U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
GGUF_F32, GGUF_F16, GGUF_Q8_0, GGUF_BF16, GGUF_MXFP4 = 0, 1, 8, 30, 39


class Typed:
    """A metadata value with an explicit GGUF value type."""

    def __init__(self, vtype, value, elem=None):
        self.vtype, self.value, self.elem = vtype, value, elem


_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B", U64: "<Q",
           I64: "<q", F64: "<d"}


def _string(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(v) -> bytes:
    if not isinstance(v, Typed):
        if isinstance(v, str):
            v = Typed(STRING, v)
        elif isinstance(v, bool):
            v = Typed(BOOL, int(v))
        elif isinstance(v, int):
            v = Typed(U32, v)
        elif isinstance(v, float):
            v = Typed(F32, v)
        elif isinstance(v, list) and all(isinstance(x, str) for x in v):
            v = Typed(ARRAY, v, STRING)
        else:
            raise TypeError(v)
    out = struct.pack("<I", v.vtype)
    if v.vtype == STRING:
        return out + _string(v.value)
    if v.vtype == ARRAY:
        out += struct.pack("<IQ", v.elem, len(v.value))
        for x in v.value:
            out += _string(x) if v.elem == STRING else (struct.pack("<I", ARRAY) if v.elem == ARRAY else
                                                        struct.pack(_SCALAR[v.elem], x))
        return out
    if v.vtype not in _SCALAR:  # a type id the format does not define (for rejection tests)
        return out + b"\0" * 4
    return out + struct.pack(_SCALAR[v.vtype], v.value)


def gguf_bytes(metadata: dict, tensors: list, version: int = 3, alignment: int = 32,
               meta_order=None) -> bytes:
    """tensors: [(name, shape (fastest first), type, data bytes)]."""
    buf = bytearray(b"GGUF")
    buf += struct.pack("<IQQ", version, len(tensors), len(metadata))
    for key in (meta_order or sorted(metadata)):
        buf += _string(key) + _value(metadata[key])
    offset = 0
    for name, shape, ttype, data in tensors:
        offset = (offset + alignment - 1) // alignment * alignment
        buf += _string(name) + struct.pack("<I", len(shape))
        for d in shape:
            buf += struct.pack("<Q", d)
        buf += struct.pack("<IQ", ttype, offset)
        offset += len(data)
    while len(buf) % alignment:
        buf += b"\0"
    base = len(buf)
    for name, shape, ttype, data in tensors:
        while (len(buf) - base) % alignment:
            buf += b"\0"
        buf += data
    return bytes(buf)


def moe_metadata(H, I, E, k, layers, eps=1e-5, prefix="gptoss.", arch="gptoss"):
    m = {"general.architecture": arch, "tokenizer.ggml.tokens": ["a", "b", "c", "d"]}
    for key, v in {"embedding_length": H, "attention.head_count": 8, "attention.head_count_kv": 2,
                   "block_count": layers, "feed_forward_length": 2 * I, "expert_feed_forward_length": I,
                   "expert_count": E, "expert_used_count": k, "context_length": 4096}.items():
        m[prefix + key] = Typed(U32, v)
    m[prefix + "attention.layer_norm_rms_epsilon"] = Typed(F32, eps)
    return m


def layer_tensors(index: int, layer: dict, H: int, I: int, E: int, split: bool = False, norm_f16: bool = False,
                  norm_name: str = "ffn_norm.weight"):
    """One layer's MoE tensors in GGUF form from a workloads-style layer dict."""
    p = f"blk.{index}."
    norm = np.ascontiguousarray(layer["norm_gain"], np.float32)
    t = [(p + norm_name, [H], GGUF_F16 if norm_f16 else GGUF_F32,
          (norm.astype(np.float16) if norm_f16 else norm).tobytes()),
         (p + "ffn_gate_inp.weight", [H, E], GGUF_F32, np.ascontiguousarray(layer["router_w"], np.float32).tobytes()),
         (p + "ffn_gate_inp.bias", [E], GGUF_F32, np.ascontiguousarray(layer["router_b"], np.float32).tobytes())]
    gu = np.ascontiguousarray(layer["gate_up"], np.uint8).reshape(E, 2 * I, H // 32 * 17)
    gub = np.ascontiguousarray(layer["gate_up_b"], np.float32).reshape(E, 2 * I)
    if split:
        t += [(p + "ffn_gate_exps.weight", [H, I, E], GGUF_MXFP4, gu[:, 0::2].tobytes()),
              (p + "ffn_gate_exps.bias", [I, E], GGUF_F32, gub[:, 0::2].copy().tobytes()),
              (p + "ffn_up_exps.weight", [H, I, E], GGUF_MXFP4, gu[:, 1::2].tobytes()),
              (p + "ffn_up_exps.bias", [I, E], GGUF_F32, gub[:, 1::2].copy().tobytes())]
    else:
        t += [(p + "ffn_gate_up_exps.weight", [H, 2 * I, E], GGUF_MXFP4, gu.tobytes()),
              (p + "ffn_gate_up_exps.bias", [2 * I, E], GGUF_F32, gub.tobytes())]
    t += [(p + "ffn_down_exps.weight", [I, H, E], GGUF_MXFP4, np.ascontiguousarray(layer["down"], np.uint8).tobytes()),
          (p + "ffn_down_exps.bias", [H, E], GGUF_F32, np.ascontiguousarray(layer["down_b"], np.float32).tobytes())]
    return t
