"""The model head on the GPU (amoe_head_*: final RMSNorm, lm_head, greedy token)
against the oracle (Runtime.nextToken, internal/model/gptoss/runtime.go:234-250),
through the C ABI: the reference's tiny-model golden tokens, GPT-OSS-shaped heads
in each GGUF encoding, first-of-equal-maxima and NaN rules, upload from a GGUF file
(with and without a separate output.weight), and the error statuses."""
import numpy as np
import pytest

import oracle
from airllm_b200 import moe
from gguf_writer import GGUF_F32, gguf_bytes, moe_metadata

pytestmark = pytest.mark.gpu


def bf16_bits(x):
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)  # round to nearest even


def bf16_value(bits):
    return (bits.astype(np.uint32) << 16).view(np.float32)


def check_tokens(tokens, logits, hidden, gain, W):
    """Each row's token and logits against the oracle; a different token only at a
    tie of the oracle's logits."""
    for t in range(hidden.shape[0]):
        ref_tok, ref_lg = oracle.next_token(hidden[t], gain, 1e-5, W)
        np.testing.assert_allclose(logits[t], ref_lg, rtol=2e-6, atol=1e-6)
        if tokens[t] != ref_tok:
            gap = abs(float(ref_lg[tokens[t]]) - float(ref_lg[ref_tok]))
            assert gap <= 1e-6 * max(1.0, abs(float(ref_lg[ref_tok]))), (t, tokens[t], ref_tok, gap)


def test_reference_tiny_model_tokens(cuda_device):
    # runtime_test.go:136-151: output_norm ones, output.weight rows [0,0],[1,0],[0,1],[0,0]; the
    # last layer's outputs for prompt token 0 and for token 1 (two layers each adding 0.125 per
    # dimension, see tests/test_head_oracle.py) give tokens 1, then 2 (runtime_test.go:70-74)
    W = np.array([[0, 0], [1, 0], [0, 1], [0, 0]], np.float32)
    head = moe.Head(2, 4)
    head.upload(np.ones(2, np.float32), W)
    tokens = head.next_token(np.array([[1.25, 0.25], [0.25, 1.25]], np.float32))
    head.close()
    assert tokens.tolist() == [1, 2]


@pytest.mark.parametrize("gtype,H,V,T", [(moe.GGUF_BF16, 2880, 50000, 1), (moe.GGUF_BF16, 2880, 50000, 3),
                                         (moe.GGUF_BF16, 2880, 20000, 16), (moe.GGUF_F16, 2880, 20000, 5),
                                         (GGUF_F32, 2880, 20000, 2), (moe.GGUF_BF16, 100, 3000, 4),
                                         (moe.GGUF_F16, 36, 777, 8), (GGUF_F32, 5, 64, 1)])
def test_head_matches_oracle(cuda_device, gtype, H, V, T):
    r = np.random.default_rng(H + V + T)
    W32 = (0.02 * r.standard_normal((V, H))).astype(np.float32)
    if gtype == moe.GGUF_BF16:
        stored = bf16_bits(W32)
        W = bf16_value(stored)
    elif gtype == moe.GGUF_F16:
        stored = W32.astype(np.float16)
        W = stored.astype(np.float32)
    else:
        stored = W = W32
    gain = (1 + 0.1 * r.standard_normal(H)).astype(np.float32)
    hidden = r.standard_normal((T, H)).astype(np.float32) * 3
    head = moe.Head(H, V)
    head.upload(gain, stored, gtype)
    tokens, logits = head.next_token(hidden, want_logits=True)
    again = head.next_token(hidden)
    head.close()
    assert np.array_equal(tokens, again)
    check_tokens(tokens, logits, hidden, gain, W)


def test_first_of_equal_maxima_and_nan_rules(cuda_device):
    H, V = 8, 300
    W = np.zeros((V, H), np.float32)
    W[[7, 40, 299], 0] = 2.0  # three equal maxima: the first wins
    head = moe.Head(H, V)
    head.upload(np.ones(H, np.float32), W)
    x = np.zeros((1, H), np.float32)
    x[0, 0] = 1.0
    assert head.next_token(x).tolist() == [7]
    W2 = W.copy()
    W2[7, 0] = np.nan  # a NaN never wins
    head.upload(np.ones(H, np.float32), W2)
    assert head.next_token(x).tolist() == [40]
    W3 = W.copy()
    W3[0, 0] = np.nan  # a NaN at index 0 is never replaced
    head.upload(np.ones(H, np.float32), W3)
    assert head.next_token(x).tolist() == [0]
    head.close()


@pytest.mark.parametrize("tied", [False, True])
def test_upload_from_gguf(cuda_device, tmp_path, tied):
    H, V = 64, 500
    r = np.random.default_rng(9)
    W = (0.05 * r.standard_normal((V, H))).astype(np.float32)
    bits = bf16_bits(W)
    norm = (1 + 0.1 * r.standard_normal(H)).astype(np.float32)
    name = "token_embd.weight" if tied else "output.weight"
    tensors = [("output_norm.weight", [H], GGUF_F32, norm.tobytes()), (name, [H, V], moe.GGUF_BF16, bits.tobytes())]
    path = tmp_path / "head.gguf"
    path.write_bytes(gguf_bytes(moe_metadata(H, 64, 4, 2, 1), tensors))
    g = moe.GGUFFile(str(path))
    head = moe.Head(H, V)
    head.upload_gguf(g)
    hidden = r.standard_normal((2, H)).astype(np.float32)
    tokens, logits = head.next_token(hidden, want_logits=True)
    head.close()
    g.close()
    check_tokens(tokens, logits, hidden, norm, bf16_value(bits))


def test_errors_are_status_codes(cuda_device):
    head = moe.Head(16, 32)
    with pytest.raises(moe.AmoeError) as e:
        head.next_token(np.zeros((1, 16), np.float32))
    assert e.value.code == moe.AMOE_ERR_STATE
    with pytest.raises(moe.AmoeError) as e:
        head.upload(np.ones(16, np.float32), np.zeros((32, 16), np.float32), 8)  # Q8_0 is not a head encoding
    assert e.value.code == moe.AMOE_ERR_INVALID
    head.upload(np.ones(16, np.float32), np.zeros((32, 16), np.float32))
    with pytest.raises(moe.AmoeError) as e:
        head.next_token(np.zeros((17, 16), np.float32))
    assert e.value.code == moe.AMOE_ERR_INVALID
    assert head.next_token(np.ones((2, 16), np.float32)).tolist() == [0, 0]  # all logits 0: the first
    head.close()
    with pytest.raises(moe.AmoeError):
        moe.Head(0, 10)
