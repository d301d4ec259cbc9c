"""The CPU oracle pinned to the reference's own golden vectors (tests/golden/reference_vectors.json,
transcribed from the Go tests they cite) and to its structural invariants."""
import json
import math
import os

import numpy as np
import pytest

import oracle
from airllm_b200 import workloads as W

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_vectors.json")))
TOL = 2e-6  # assertClose, internal/backend/cpuref/primitives_test.go:76


def close(got, want):
    np.testing.assert_allclose(np.asarray(got, np.float64), np.asarray(want, np.float64), rtol=0, atol=TOL)


def test_linear_golden():
    g = GOLD["linear"]
    close(oracle.linear_bias(g["input"], g["weight"], None, g["in"], g["out"]), g["want"])


def test_linear_bias_golden():
    g = GOLD["linear_bias"]
    close(oracle.linear_bias(g["input"], g["weight"], g["bias"], g["in"], g["out"]), g["want"])


def test_rmsnorm_golden():
    g = GOLD["rmsnorm"]
    close(oracle.rmsnorm(g["input"], g["weight"], g["eps"]), g["want"])


def test_router_topk_selected_softmax_golden():
    g = GOLD["router_topk"]
    idx, w = oracle.router_topk(g["logits"], g["k"])
    assert idx.tolist() == g["want_idx"]
    close(w, g["want_w"])


def test_swiglu_golden_exercises_both_clamps():
    g = GOLD["swiglu"]
    close(oracle.swiglu(g["gate"], g["up"]), g["want"])


def test_mxfp4_encoded_sizes():
    g = GOLD["mxfp4_sizes"]
    for elements, nbytes in g["cases"]:
        assert oracle.mxfp4_encoded_size(elements) == nbytes
    for bad in g["rejects"]:
        with pytest.raises(oracle.OracleError):
            oracle.mxfp4_encoded_size(bad)


def test_mxfp4_all_nibbles_and_order():
    g = GOLD["mxfp4_all_nibbles"]
    block = bytearray(17)
    block[0] = g["scale_byte"]
    for i in range(16):
        block[1 + i] = i | (15 - i) << 4
    out = oracle.mxfp4_decode(bytes(block), 32)
    table = g["table"]
    for i in range(16):
        for pair, nib in enumerate((i, 15 - i)):  # low nibble -> element 2i, high -> 2i+1
            got, want = out[2 * i + pair], table[nib]
            assert got == want and math.copysign(1, got) == math.copysign(1, want)


def test_mxfp4_golden_scales_incl_denormal_and_nan():
    g = GOLD["mxfp4_scales"]
    table = GOLD["mxfp4_all_nibbles"]["table"]
    for e in g["exponents"]:
        block = bytearray(17)
        block[0] = e
        block[1] = g["byte1"]  # 0x73: nibbles 3 and 7 (values 1.5 and 6)
        out = oracle.mxfp4_decode(bytes(block), 32)
        for i, nib in enumerate(g["nibbles"]):
            if e == g["nan_exponent"]:
                assert np.isnan(out[i])
            else:
                with np.errstate(over="ignore"):  # 2^127 * 6 is +Inf in float32, as in Go
                    want = np.float32(math.ldexp(1.0, e - 127)) * np.float32(table[nib])
                    assert out[i] == want, (e, i, out[i], want)
                    # the reference test compares after float16 rounding (convert.go path)
                    assert np.float16(out[i]) == np.float16(want)


def test_validation_errors_like_reference():
    v = GOLD["validation"]
    with pytest.raises(oracle.OracleError):
        oracle.router_topk(v["topk_too_large"]["logits"], v["topk_too_large"]["k"])
    with pytest.raises(oracle.OracleError):
        r = v["rmsnorm_zero_eps"]
        oracle.rmsnorm(r["input"], r["weight"], r["eps"])
    with pytest.raises(oracle.OracleError):
        r = v["linear_bad_input"]
        oracle.linear_bias(r["input"], r["weight"], None, r["in"], r["out"])
    with pytest.raises(oracle.OracleError):
        oracle.swiglu(v["swiglu_mismatch"]["gate"], v["swiglu_mismatch"]["up"])


def test_topk_ties_resolve_to_lower_expert():
    idx, w = oracle.router_topk([0.5, 1.0, 1.0, 0.5, 1.0], 4)
    assert idx.tolist() == [1, 2, 4, 0]
    idx, w = oracle.router_topk([0.0, -0.0, 0.0, 0.0], 4)  # -0 == +0: stable
    assert idx.tolist() == [0, 1, 2, 3]
    close(w, [0.25] * 4)


def _moe_numpy(layer, x):
    """Independent numpy restatement (decode everything, float64 matmuls) used to
    cross-check the C oracle's indexing; float64 matmul sums in a different order,
    so agreement is to ~1e-5, not bitwise."""
    H, I, E, k = layer["hidden"], layer["intermediate"], layer["experts"], layer["top_k"]
    gu = oracle.mxfp4_decode(layer["gate_up"], E * 2 * I * H).reshape(E, 2 * I, H).astype(np.float64)
    dn = oracle.mxfp4_decode(layer["down"], E * H * I).reshape(E, H, I).astype(np.float64)
    out = np.empty_like(x)
    for t in range(x.shape[0]):
        xn = oracle.rmsnorm(x[t], layer["norm_gain"], layer["eps"])
        lg = (layer["router_w"].astype(np.float64) @ xn.astype(np.float64)).astype(np.float32) + layer["router_b"]
        idx, w = oracle.router_topk(lg, k)
        mix = np.zeros(H)
        for s, e in enumerate(idx):
            g = (gu[e] @ xn.astype(np.float64)).astype(np.float32) + layer["gate_up_b"][e]
            a = oracle.swiglu(g[0::2], g[1::2])
            y = (dn[e] @ a.astype(np.float64)).astype(np.float32) + layer["down_b"][e]
            mix += float(w[s]) * y.astype(np.float64)
        out[t] = x[t] + mix.astype(np.float32)
    return out


def test_oracle_block_matches_independent_numpy_restatement():
    layer = W.small_layer(hidden=64, intermediate=96, experts=6, top_k=3, seed=5)
    x = W.make_tokens(W.MoEShape(64, 96, 6, 3), 7, 5)
    out, idx, w, lg = oracle.moe_block(layer, x)
    np.testing.assert_allclose(out, _moe_numpy(layer, x), rtol=0, atol=1e-5)


def test_faithful_and_fused_decode_are_bit_identical():
    layer = W.small_layer(hidden=64, intermediate=64, experts=5, top_k=2, seed=3)
    x = W.make_tokens(W.MoEShape(64, 64, 5, 2), 6, 3)
    a = oracle.moe_block(layer, x, faithful=False, threads=1)
    b = oracle.moe_block(layer, x, faithful=True, threads=2)
    for u, v in zip(a, b):
        assert np.array_equal(u, v, equal_nan=True)


def test_token_subset_equals_full_run():
    layer = W.small_layer(seed=11)
    x = W.make_tokens(W.MoEShape(64, 128, 8, 4), 9, 11)
    full = oracle.moe_block(layer, x)[0]
    sub = oracle.moe_block(layer, x, tokens=[7, 2])[0]
    assert np.array_equal(sub[[2, 7]], full[[2, 7]])
    assert np.isnan(sub[0]).all()


def test_permutation_is_stable_sort_by_expert():
    rng = np.random.default_rng(0)
    T, k, E = 50, 4, 9
    idx = np.stack([rng.choice(E, size=k, replace=False) for _ in range(T)]).astype(np.int32)
    perm, counts, offsets, inv = oracle.permute(idx, E)
    flat = idx.ravel()
    assert np.array_equal(counts, np.bincount(flat, minlength=E))
    assert np.array_equal(offsets, np.concatenate([[0], np.cumsum(counts)]))
    keys = [(flat[p], p) for p in perm]
    assert keys == sorted(keys)  # (expert, t*k+s) ascending: stable by (e, t, s)
    assert np.array_equal(inv[perm], np.arange(T * k))


def test_route_matches_block_routing():
    layer = W.small_layer(seed=2)
    x = W.make_tokens(W.MoEShape(64, 128, 8, 4), 12, 2)
    lg, idx, w = oracle.route(layer, x)
    _, idx2, w2, lg2 = oracle.moe_block(layer, x)
    assert np.array_equal(idx, idx2) and np.array_equal(w, w2) and np.array_equal(lg, lg2)


@pytest.mark.parametrize("H,I,E,k,T,threads", [(64, 96, 6, 3, 7, 1), (192, 320, 16, 4, 77, 4),
                                                (2880, 2880, 32, 4, 9, 8), (64, 64, 128, 4, 40, 3)])
def test_expert_major_oracle_is_bit_identical_to_token_by_token(H, I, E, k, T, threads):
    """moe_block_grouped (every expert decoded once, its tokens' dot products side by
    side, each keeping the reference's sequential float64 order) returns exactly what
    the token-by-token oracle returns: outputs, routing and logits, bit for bit."""
    layer = W.small_layer(hidden=H, intermediate=I, experts=E, top_k=k, seed=H + E + T)
    x = W.make_tokens(W.MoEShape(H, I, E, k), T, T)
    a = oracle.moe_block(layer, x, threads=threads)
    b = oracle.moe_block_grouped(layer, x, threads=threads)
    for u, v in zip(a, b):
        assert np.array_equal(u, v, equal_nan=True)
    rows = [T - 1, 0, T // 2]
    a = oracle.moe_block(layer, x, tokens=rows)
    b = oracle.moe_block_grouped(layer, x, tokens=rows)
    for u, v in zip(a, b):
        assert np.array_equal(u, v, equal_nan=True)


def test_expert_major_oracle_keeps_nan_scales_and_denormals():
    layer = W.small_layer(hidden=128, intermediate=128, experts=8, top_k=4, seed=4, scale_lo=0, scale_hi=123)
    layer["down"].reshape(-1, 17)[5, 0] = 0xFF
    x = W.make_tokens(W.MoEShape(128, 128, 8, 4), 10, 4)
    a = oracle.moe_block(layer, x)
    b = oracle.moe_block_grouped(layer, x)
    for u, v in zip(a, b):
        assert np.array_equal(u, v, equal_nan=True)
