"""The attention-half oracle (oracle/attn_oracle.c) pinned to the reference's own
golden vectors and validation cases (tests/golden/reference_vectors.json,
transcribed from internal/backend/cpuref/attention_test.go, rope_test.go,
gptoss_test.go and gemma_test.go), cross-checked against an independent numpy restatement, and
checked for the causal-cache property a GPU decode path relies on: decoding
token by token gives the same rows as one prefill over the whole sequence."""
import json
import math
import os

import numpy as np
import pytest

import oracle

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_vectors.json")))
TOL = 2e-6  # assertClose, internal/backend/cpuref/primitives_test.go:76


def close(got, want, tol=TOL):
    np.testing.assert_allclose(np.asarray(got, np.float64), np.asarray(want, np.float64), rtol=0, atol=tol)


@pytest.mark.parametrize("name", ["rope_offset", "rope_zero"])
def test_rope_golden(name):
    g = GOLD[name]
    close(oracle.rope(g["input"], g["head_dim"], g["offset"], g["theta"]), g["want"])


def test_yarn_rope_gptoss_golden():
    g = GOLD["yarn_rope_gptoss"]
    close(oracle.yarn_rope(g["input"], g["head_dim"], g["offset"], g["theta"]), g["want"])


def _cache(g):
    c = oracle.KVCache(g["kv_heads"], g["head_dim"], g["capacity"])
    for a in g["appends"]:
        c.append(a["keys"], a["values"], a["seq"])
    return c


@pytest.mark.parametrize("name", ["attention_gqa", "attention_sink", "attention_window", "attention_scale_softcap"])
def test_attention_golden(name):
    g = GOLD[name]
    c = _cache(g)
    got = oracle.causal_attention(g["query"], g["q_heads"], c, sinks=g.get("sinks"), window=g.get("window", 0),
                                  pre_scalar=g.get("pre_scalar", 0.0), softcap=g.get("softcap", 0.0))
    close(got, g["want"])


def test_gqa_cache_holds_kv_heads_only():
    # attention_test.go:47-55: three tokens x two KV heads x two dims, not four query heads
    c = _cache(GOLD["attention_gqa"])
    assert c.keys.size == 12 and c.values.size == 12 and c.length == 3


def test_kv_append_is_transactional():
    # attention_test.go:58-78
    c = oracle.KVCache(1, 2, 1)
    with pytest.raises(oracle.OracleError):
        c.append([1, 2], [3], 1)
    assert c.length == 0
    c.append([1, 2], [3, 4], 1)
    with pytest.raises(oracle.OracleError):
        c.append([1, 2], [3, 4], 1)
    assert c.length == 1


def test_validation_like_reference():
    # rope_test.go:28-35
    with pytest.raises(oracle.OracleError, match="even"):
        oracle.rope([1, 2, 3], 3, 0, 10000)
    with pytest.raises(oracle.OracleError, match="non-negative"):
        oracle.rope([1, 2], 2, -1, 10000)
    # attention_test.go:80-98
    c = oracle.KVCache(2, 2, 1)
    c.append(np.zeros(4), np.zeros(4), 1)
    with pytest.raises(oracle.OracleError, match="multiple of kv heads"):
        oracle.causal_attention(np.zeros(6), 3, c)
    with pytest.raises(oracle.OracleError, match="exceeds cached length"):
        oracle.causal_attention(np.zeros(16), 4, c)
    with pytest.raises(oracle.OracleError, match="nil"):
        oracle.causal_attention(np.zeros(8), 4, None)
    with pytest.raises(oracle.OracleError, match="sinks"):
        oracle.causal_attention(np.zeros(8), 4, c, sinks=[0.0])


def test_layer_window_alternates():
    # weights.go:118-122: even layers use the model's window, odd layers attend to all
    assert [oracle.layer_window(i, 128) for i in range(4)] == [128, 0, 128, 0]


# ---- independent numpy restatement of the attention half --------------------------------

def _yarn_np(x, head_dim, offset, theta):
    half = head_dim // 2
    factor, orig, bf, bs = 32.0, 4096.0, 32.0, 1.0
    corr = lambda beta: head_dim * math.log(orig / (beta * 2 * math.pi)) / (2 * math.log(theta))
    low, high = max(0.0, math.floor(corr(bf))), min(half - 1.0, math.ceil(corr(bs)))
    i = np.arange(half, dtype=np.float64)
    base = theta ** (-2 * i / head_dim)
    ramp = np.clip((i - low) / (high - low) if high != low else np.zeros(half), 0, 1)
    freq = base * (ramp + (1 - ramp) / factor)
    conc = 1 + 0.1 * math.log(factor)
    x = np.asarray(x, np.float64).reshape(-1, head_dim)
    pos = offset + np.arange(x.shape[0], dtype=np.float64)[:, None]
    s, c = np.sin(pos * freq) * conc, np.cos(pos * freq) * conc
    a, b = x[:, :half], x[:, half:]
    return np.concatenate([a * c - b * s, b * c + a * s], axis=1).astype(np.float32)


def _attention_half_np(L, x, keys, values, window):
    """keys/values: lists of [kv_heads, head_dim] rows already in the cache (mutated)."""
    H, nh, nkv, d = L["hidden"], L["heads"], L["kv_heads"], L["head_dim"]
    out = np.empty_like(x)
    T, pos0 = x.shape[0], len(keys)
    qs = []
    for t in range(T):
        xn = oracle.rmsnorm(x[t], L["norm1"], L["eps"])
        qkv = (L["qkv_w"].astype(np.float64) @ xn.astype(np.float64)).astype(np.float32) + L["qkv_b"]
        qs.append(qkv[:nh * d].reshape(nh, d))
        keys.append(qkv[nh * d:(nh + nkv) * d].reshape(nkv, d))
        values.append(qkv[(nh + nkv) * d:].reshape(nkv, d))
    q = np.stack([_yarn_np(np.stack([qs[t][h] for t in range(T)]), d, pos0, L["theta"]) for h in range(nh)], 1)
    kr = np.stack([_yarn_np(np.stack([keys[pos0 + t][h] for t in range(T)]), d, pos0, L["theta"])
                   for h in range(nkv)], 1)
    for t in range(T):
        keys[pos0 + t] = kr[t]
    K, V = np.stack(keys).astype(np.float64), np.stack(values).astype(np.float64)
    for t in range(T):
        p = pos0 + t
        first = p - window + 1 if window > 0 and p >= window else 0
        att = np.empty(nh * d, np.float32)
        for h in range(nh):
            kv = h // (nh // nkv)
            sc = K[first:p + 1, kv] @ q[t, h].astype(np.float64) / math.sqrt(d)
            m = max(sc.max(), float(L["sinks"][h]))
            e = np.exp(sc - m)
            den = e.sum() + math.exp(float(L["sinks"][h]) - m)
            att[h * d:(h + 1) * d] = (e @ V[first:p + 1, kv] / den).astype(np.float32)
        proj = (L["out_w"].astype(np.float64) @ att.astype(np.float64)).astype(np.float32) + L["out_b"]
        out[t] = x[t] + proj
    return out


def _attn_layer(H=64, heads=4, kv_heads=2, head_dim=16, seed=0):
    r = np.random.default_rng(seed)
    qkvw = (heads + 2 * kv_heads) * head_dim
    return {"hidden": H, "heads": heads, "kv_heads": kv_heads, "head_dim": head_dim, "eps": 1e-5,
            "theta": 150000.0,
            "norm1": (1 + 0.1 * r.standard_normal(H)).astype(np.float32),
            "qkv_w": (0.1 * r.standard_normal((qkvw, H))).astype(np.float32),
            "qkv_b": (0.02 * r.standard_normal(qkvw)).astype(np.float32),
            "out_w": (0.1 * r.standard_normal((H, heads * head_dim))).astype(np.float32),
            "out_b": (0.02 * r.standard_normal(H)).astype(np.float32),
            "sinks": r.standard_normal(heads).astype(np.float32)}


@pytest.mark.parametrize("window", [0, 4])
def test_attention_half_matches_numpy_prefill_then_decode(window):
    L = _attn_layer(seed=window)
    r = np.random.default_rng(10 + window)
    x = r.standard_normal((9, L["hidden"])).astype(np.float32)
    cache = oracle.KVCache(L["kv_heads"], L["head_dim"], 16)
    keys, values = [], []
    got = [oracle.attention_half(L, x[:6], cache, window)]
    want = [_attention_half_np(L, x[:6], keys, values, window)]
    for t in range(6, 9):  # three decode steps
        got.append(oracle.attention_half(L, x[t:t + 1], cache, window))
        want.append(_attention_half_np(L, x[t:t + 1], keys, values, window))
    assert cache.length == 9
    close(np.concatenate(got), np.concatenate(want), tol=1e-5)


@pytest.mark.parametrize("window", [0, 3])
def test_decode_steps_equal_one_prefill(window):
    # a query attends to keys at or before its position only, and each position's
    # rotation depends on the position alone: token-by-token decoding reproduces the
    # rows of a single prefill exactly
    L = _attn_layer(seed=3)
    x = np.random.default_rng(4).standard_normal((7, L["hidden"])).astype(np.float32)
    full = oracle.attention_half(L, x, oracle.KVCache(L["kv_heads"], L["head_dim"], 8), window)
    c = oracle.KVCache(L["kv_heads"], L["head_dim"], 8)
    steps = np.concatenate([oracle.attention_half(L, x[t:t + 1], c, window) for t in range(7)])
    assert np.array_equal(full, steps)


def test_attention_half_rejects_a_full_cache():
    L = _attn_layer()
    c = oracle.KVCache(L["kv_heads"], L["head_dim"], 2)
    oracle.attention_half(L, np.zeros((2, L["hidden"]), np.float32), c, 0)
    with pytest.raises(oracle.OracleError, match="capacity"):
        oracle.attention_half(L, np.zeros((1, L["hidden"]), np.float32), c, 0)
    assert c.length == 2
