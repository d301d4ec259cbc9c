"""GGUF reading (amoe_gguf_*), modelled on the reference's own reader tests
(internal/gguf/gguf_test.go:25-63, gptoss_test.go:122-157): v2 and v3 headers,
the tensor index, the GPT-OSS metadata dialects, and rejection of malformed
files.  The GPU test uploads layers from a GGUF file and checks that the block
computes exactly what it computes from the same tensors given as arrays."""
import numpy as np
import pytest

from airllm_b200 import moe
from airllm_b200 import workloads as W
from gguf_writer import (ARRAY, BOOL, F32, GGUF_F32, GGUF_MXFP4, GGUF_Q8_0, I32, STRING, U32, U64, Typed,
                         gguf_bytes, layer_tensors, moe_metadata)


def _write(tmp_path, data, name="m.gguf"):
    p = tmp_path / name
    p.write_bytes(data)
    return str(p)


def _fixture_tensors():
    rng = np.random.default_rng(5)
    return [("token_embd.weight", [8, 4], GGUF_F32, rng.standard_normal(32).astype(np.float32).tobytes()),
            ("blk.0.attn_norm.weight", [8], GGUF_F32, np.ones(8, np.float32).tobytes()),
            ("blk.0.attn_k.weight", [8, 8], GGUF_Q8_0, bytes(range(68))),
            ("blk.0.ffn_down_exps.weight", [64, 16, 2], GGUF_MXFP4, bytes((i * 7) & 255 for i in range(1088)))]


@pytest.mark.parametrize("version", [2, 3])
def test_open_v2_v3_and_index_one_tensor(tmp_path, version):
    tensors = _fixture_tensors()
    path = _write(tmp_path, gguf_bytes(moe_metadata(8, 16, 2, 1, 1), tensors, version=version))
    g = moe.GGUFFile(path)
    info = g.tensor("blk.0.attn_k.weight")
    assert info["type"] == GGUF_Q8_0 and info["shape"] == [8, 8] and info["bytes"] == 68
    raw = open(path, "rb").read()
    assert raw[info["offset"]:info["offset"] + info["bytes"]] == tensors[2][3]
    mx = g.tensor("blk.0.ffn_down_exps.weight")
    assert mx["bytes"] == 64 * 16 * 2 // 32 * 17 and raw[mx["offset"]:mx["offset"] + mx["bytes"]] == tensors[3][3]
    assert mx["offset"] % 32 == 0
    with pytest.raises(moe.AmoeError):
        g.tensor("absent")
    g.close()


@pytest.mark.parametrize("prefix,arch", [("gptoss.", "gptoss"), ("gpt-oss.", "gpt-oss")])
def test_gptoss_metadata_dialects(tmp_path, prefix, arch):
    md = moe_metadata(64, 32, 16, 4, 4, prefix=prefix, arch=arch)
    path = _write(tmp_path, gguf_bytes(md, []))
    cfg = moe.GGUFFile(path).moe_config()
    assert (cfg["hidden"], cfg["intermediate"], cfg["experts"], cfg["top_k"], cfg["layers"]) == (64, 32, 16, 4, 4)
    assert cfg["rms_eps"] == np.float32(1e-5)


def test_metadata_integer_widths_and_alignment(tmp_path):
    md = moe_metadata(64, 32, 16, 4, 2)
    md["gptoss.embedding_length"] = Typed(U64, 64)
    md["gptoss.expert_count"] = Typed(I32, 16)
    md["general.alignment"] = Typed(U32, 64)
    md["general.flag"] = Typed(BOOL, 1)
    tensors = _fixture_tensors()
    path = _write(tmp_path, gguf_bytes(md, tensors, alignment=64))
    g = moe.GGUFFile(path)
    assert g.moe_config()["experts"] == 16
    for name, *_ in tensors:
        assert g.tensor(name)["offset"] % 64 == 0


def _bad(tmp_path, data, needle):
    with pytest.raises(moe.AmoeError) as e:
        moe.GGUFFile(_write(tmp_path, data))
    assert needle in str(e.value), str(e.value)


def test_rejects_malformed_files(tmp_path):
    good = gguf_bytes(moe_metadata(8, 16, 2, 1, 1), _fixture_tensors())
    _bad(tmp_path, b"GGU", "magic")
    _bad(tmp_path, b"GGML" + good[4:], "invalid magic")
    for v in (1, 4):
        _bad(tmp_path, good[:4] + np.uint32(v).tobytes() + good[8:], "want 2 or 3")
    _bad(tmp_path, good[:40], "truncated")
    _bad(tmp_path, good[:-100], "exceeds file size")
    md = moe_metadata(8, 16, 2, 1, 1)
    order = sorted(md) + [sorted(md)[0]]
    dup = gguf_bytes(md, [], meta_order=order)
    dup = dup[:16] + np.uint64(len(order)).tobytes() + dup[24:]
    _bad(tmp_path, dup, "duplicate metadata key")
    t = _fixture_tensors()
    _bad(tmp_path, gguf_bytes(md, [t[0], t[0]]), "duplicate tensor")
    _bad(tmp_path, gguf_bytes(dict(md, nested=Typed(ARRAY, [], ARRAY)), []), "nested arrays")
    _bad(tmp_path, gguf_bytes(dict(md, flag=Typed(BOOL, 2)), []), "invalid boolean")
    _bad(tmp_path, gguf_bytes(dict(md, **{"general.alignment": Typed(U32, 0)}), []), "alignment")
    _bad(tmp_path, gguf_bytes(md, [("x", [48], GGUF_MXFP4, bytes(17))]), "divisible by 32")
    _bad(tmp_path, gguf_bytes(md, [("x", [4], 99, bytes(16))]), "unsupported tensor type")
    _bad(tmp_path, gguf_bytes(dict(md, odd=Typed(77, 0)), []), "unknown metadata value type")
    # element counts that fit int64 but whose encoded byte size does not
    # (reader.go:429-466): rejected, not wrapped to a small size
    for shape, ttype in [([1 << 62], 0), ([1 << 61, 2], 0), ([1 << 62], 1), ([1 << 62], 30),
                         ([(1 << 63) - (1 << 58)], GGUF_Q8_0)]:
        _bad(tmp_path, gguf_bytes(md, [("x", shape, ttype, b"")]), "encoded tensor size overflows int64")


def test_config_needs_gptoss_metadata(tmp_path):
    md = moe_metadata(64, 32, 16, 4, 2)
    for drop, needle in [("gptoss.expert_count", "missing metadata"),
                         ("gptoss.attention.layer_norm_rms_epsilon", "missing metadata")]:
        g = moe.GGUFFile(_write(tmp_path, gguf_bytes({k: v for k, v in md.items() if k != drop}, [])))
        with pytest.raises(moe.AmoeError) as e:
            g.moe_config()
        assert needle in str(e.value)
    g = moe.GGUFFile(_write(tmp_path, gguf_bytes(dict(md, **{"general.architecture": "llama"}), [])))
    with pytest.raises(moe.AmoeError) as e:
        g.moe_config()
    assert "unsupported architecture" in str(e.value)
    g = moe.GGUFFile(_write(tmp_path, gguf_bytes(dict(md, **{"gptoss.expert_count": Typed(STRING, "16")}), [])))
    with pytest.raises(moe.AmoeError):
        g.moe_config()
    g = moe.GGUFFile(_write(tmp_path, gguf_bytes(dict(md, **{"gptoss.attention.layer_norm_rms_epsilon":
                                                             Typed(F32, -1.0)}), [])))
    with pytest.raises(moe.AmoeError):
        g.moe_config()


@pytest.mark.gpu
def test_upload_from_gguf_matches_arrays(cuda_device, tmp_path):
    H, I, E, k = 128, 192, 8, 4
    shape = W.MoEShape(H, I, E, k)
    layers = [W.make_layer(shape, 70 + i) for i in range(2)]
    tensors = (layer_tensors(0, layers[0], H, I, E) +
               layer_tensors(1, layers[1], H, I, E, split=True, norm_f16=True, norm_name="post_attention_norm.weight"))
    g = moe.GGUFFile(_write(tmp_path, gguf_bytes(moe_metadata(H, I, E, k, 2), tensors)))
    cfg = g.moe_config()
    assert (cfg["hidden"], cfg["intermediate"], cfg["experts"], cfg["top_k"], cfg["layers"]) == (H, I, E, k, 2)
    x = W.make_tokens(shape, 40, 70)
    a = moe.MoEBlock(H, I, E, k, layers=2, max_tokens=40)
    b = moe.MoEBlock(H, I, E, k, layers=2, max_tokens=40)
    for i, L in enumerate(layers):
        ref = dict(L)
        if i == 1:  # the file holds this layer's norm gain as f16
            ref["norm_gain"] = np.asarray(L["norm_gain"], np.float32).astype(np.float16).astype(np.float32)
        a.upload_layer(i, ref)
        b.upload_layer_gguf(i, g)
    for i in range(2):
        assert np.array_equal(a.forward(x, layer=i)[0], b.forward(x, layer=i)[0])
    # a tensor with the wrong shape is refused with the reference's message
    bad = layer_tensors(0, layers[0], H, I, E)
    bad[1] = (bad[1][0], [E, H], GGUF_F32, bad[1][3])  # the router stored transposed
    gb = moe.GGUFFile(_write(tmp_path, gguf_bytes(moe_metadata(H, I, E, k, 2), bad), "bad.gguf"))
    with pytest.raises(moe.AmoeError) as e:
        b.upload_layer_gguf(0, gb)
    assert "want GGUF shape" in str(e.value)
    a.close()
    b.close()
