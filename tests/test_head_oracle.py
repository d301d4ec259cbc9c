"""The model head's oracle (Runtime.nextToken, internal/model/gptoss/runtime.go:234-250:
final RMSNorm, lm_head Linear without bias, first-max argmax), pinned by the
reference's own end-to-end golden case: the tiny synthetic GPT-OSS model of
internal/model/gptoss/runtime_test.go:123-189 generates tokens [1, 2] from the
prompt [0] (runtime_test.go:62-74).  The whole tiny model runs here through the
oracles: embeddings, two decoder layers (the attention half, then the MoE half
with the reference's routing and SwiGLU), and the head."""
import numpy as np
import pytest

import oracle

# runtime_test.go:136-151: embedding_length 2, 4 experts (all used), expert FFN 2,
# one attention head of dimension 2, rope base 10000, eps 1e-5, vocabulary of 4
H, E, K, I = 2, 4, 4, 2
EMBD = np.array([1, 0, 0, 1, -1, 0, 0, 0], np.float32).reshape(4, H)      # token_embd.weight [2, 4]
OUT_NORM = np.ones(H, np.float32)                                         # output_norm.weight
LM_HEAD = np.array([0, 0, 1, 0, 0, 1, 0, 0], np.float32).reshape(4, H)   # output.weight [2, 4]
DOWN_B = np.array([0.25, 0.25, 0.25, 0.25, 0, 0, 0, 0], np.float32).reshape(E, H)  # ffn_down_exps.bias
EOS = 2  # tokenizer.ggml.eos_token_id


def _attention_layer():
    # the fused dialect (runtime_test.go:176-182): zero qkv, output projection and sink
    return {"hidden": H, "heads": 1, "kv_heads": 1, "head_dim": 2, "eps": 1e-5, "theta": 10000.0,
            "norm1": np.ones(H, np.float32), "qkv_w": np.zeros((6, H), np.float32),
            "qkv_b": np.zeros(6, np.float32), "out_w": np.zeros((H, 2), np.float32),
            "out_b": np.zeros(H, np.float32), "sinks": np.zeros(1, np.float32)}


def _moe_half(x):
    """layer.go:94-123 with the fixture's zero router and expert weights
    (runtime_test.go:184-189): the routing is four tied logits, every expert's
    activation is SwiGLU(0, 0) and its output is its down bias."""
    out = np.empty_like(x)
    for t in range(x.shape[0]):
        xn = oracle.rmsnorm(x[t], np.ones(H, np.float32), 1e-5)
        logits = oracle.linear_bias(xn, np.zeros((E, H), np.float32), np.zeros(E, np.float32), H, E)
        idx, w = oracle.router_topk(logits, K)
        mix = np.zeros(H, np.float64)
        for s in range(K):
            act = oracle.swiglu(np.zeros(I, np.float32), np.zeros(I, np.float32))
            y = oracle.linear_bias(act, np.zeros((H, I), np.float32), DOWN_B[idx[s]], I, H)
            mix += float(w[s]) * y.astype(np.float64)
        out[t] = x[t] + mix.astype(np.float32)
    return out


def test_tiny_model_generates_the_reference_tokens():
    caches = [oracle.KVCache(1, 2, 8) for _ in range(2)]
    layer = _attention_layer()
    generated, token = [], 0
    for _ in range(5):  # Generate(ctx, [0], 5, ...) stops at the EOS token
        h = EMBD[token][None, :]
        for i in range(2):
            h = oracle.attention_half(layer, h, caches[i], oracle.layer_window(i, 128))
            h = _moe_half(h)
        token, _ = oracle.next_token(h[0], OUT_NORM, 1e-5, LM_HEAD)
        generated.append(token)
        if token == EOS:
            break
    assert generated == [1, 2]  # runtime_test.go:70-74


def test_argmax_takes_the_first_of_equal_maxima_and_skips_nan():
    W = np.zeros((5, 2), np.float32)
    W[1] = W[3] = [1, 0]  # logits 0, x, 0, x, 0: the first maximum wins
    assert oracle.next_token([1, 0], [1, 1], 1e-5, W)[0] == 1
    W = np.array([[1, 0], [np.nan, 0], [2, 0]], np.float32)  # a NaN never wins
    assert oracle.next_token([1, 0], [1, 1], 1e-5, W)[0] == 2
    W = np.array([[np.nan, 0], [5, 0], [6, 0]], np.float32)  # a NaN at index 0 is never replaced
    assert oracle.next_token([1, 0], [1, 1], 1e-5, W)[0] == 0


def test_rejects_mismatched_lengths():
    with pytest.raises(oracle.OracleError):
        oracle.next_token(np.zeros(3, np.float32), np.ones(2, np.float32), 1e-5, np.zeros((4, 2), np.float32))
