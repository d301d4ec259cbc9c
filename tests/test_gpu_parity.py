"""CUDA path vs the oracle, through the C ABI (ctypes -> libamoe.so)."""
import numpy as np
import pytest

import oracle
from airllm_b200 import moe
from airllm_b200 import workloads as W
from parity_util import assert_block_parity, routing_mismatches

pytestmark = pytest.mark.gpu

PATHS = [moe.PATH_GEMV, moe.PATH_TENSOR]


def run_block(layer, x, path=moe.PATH_AUTO, max_tokens=None):
    blk = moe.MoEBlock.for_layer(layer, max_tokens=max_tokens or max(x.shape[0], 1), path=path)
    blk.upload_layer(0, layer)
    out, idx, w = blk.forward(x)
    routing = blk.last_routing(x.shape[0])
    blk.close()
    return out, idx, w, routing


def check_against_oracle(layer, x, path, tokens=None):
    out, idx, w, (logits, perm, counts, offsets) = run_block(layer, x, path)
    ref_lg, ref_idx, ref_w = oracle.route(layer, x)
    ties, bad = routing_mismatches(idx, ref_idx, ref_lg)
    assert not bad, f"routing differs beyond ties on rows {bad[:10]}"
    # logits: float64 sums in another order; near-zero logits can move by a few ulp
    # when one RMSNorm output rounds the other way, far inside the 1e-6 tie threshold
    np.testing.assert_allclose(logits, ref_lg, rtol=0, atol=1e-6)
    # the permutation is the stable (expert, token, slot) order of the GPU's own routing
    p_ref, c_ref, o_ref, _ = oracle.permute(idx, layer["experts"])
    assert np.array_equal(perm, p_ref) and np.array_equal(counts, c_ref) and np.array_equal(offsets, o_ref)
    if not ties:
        np.testing.assert_allclose(w, ref_w, rtol=2e-6, atol=0)
    rows = np.arange(x.shape[0]) if tokens is None else np.asarray(tokens)
    rows = np.setdiff1d(rows, ties)
    ref_out = oracle.moe_block(layer, x, tokens=rows)[0]
    return assert_block_parity(out, ref_out, rows)


def test_tiny_fixture_all_ties_and_bias_path(cuda_device):
    """MXFP4 analogue of the synthetic model of internal/model/gptoss/runtime_test.go:123-189:
    zero router (all logits tie -> experts 0..3 in index order, weights 1/4), zero expert
    weights, a down bias per expert; the block adds sum_k 1/4 * bias_k to the residual."""
    H, I, E, k = 64, 64, 4, 4
    layer = W.small_layer(hidden=H, intermediate=I, experts=E, top_k=k, seed=0)
    layer["router_w"][:] = 0
    layer["router_b"][:] = 0
    layer["gate_up"].reshape(-1, 17)[:, 1:] = 0  # every nibble is +0
    layer["down"].reshape(-1, 17)[:, 1:] = 0
    layer["gate_up_b"][:] = 0
    layer["down_b"][:] = np.array([[0.25], [0.25], [0.0], [0.0]], np.float32)
    x = W.make_tokens(W.MoEShape(H, I, E, k), 3, 0)
    for path in PATHS:
        out, idx, w, _ = run_block(layer, x, path)
        assert (idx == np.arange(4)).all()
        assert (w == np.float32(0.25)).all()
        np.testing.assert_array_equal(out, x + np.float32(0.125))


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("H,I,E,k,T", [
    (64, 128, 8, 4, 1), (64, 128, 8, 4, 3), (64, 128, 8, 4, 8), (64, 128, 8, 4, 9),
    (64, 128, 8, 4, 37), (128, 64, 5, 2, 17), (192, 320, 16, 4, 64), (64, 64, 128, 4, 40),
    (64, 64, 256, 8, 11), (128, 128, 3, 1, 5),
])
def test_small_layers_match_oracle(cuda_device, path, H, I, E, k, T):
    layer = W.small_layer(hidden=H, intermediate=I, experts=E, top_k=k, seed=H + I + E + T)
    x = W.make_tokens(W.MoEShape(H, I, E, k), T, T)
    check_against_oracle(layer, x, path)


@pytest.mark.parametrize("H,I,E,k,T", [
    (64, 128, 8, 4, 1), (192, 320, 16, 4, 2), (320, 192, 32, 4, 3), (128, 128, 128, 4, 4),
    (64, 64, 256, 8, 4), (128, 64, 5, 2, 4), (2880, 2880, 32, 4, 2),
])
def test_fused_decode_stage_matches_oracle(cuda_device, H, I, E, k, T):
    # T <= 4 on the GEMV path runs routing, gate_up, down and the combine as one
    # cooperative launch; the stage timer shows which kernel ran
    layer = W.small_layer(hidden=H, intermediate=I, experts=E, top_k=k, seed=7 * T + E)
    x = W.make_tokens(W.MoEShape(H, I, E, k), T, T + 1)
    blk = moe.MoEBlock.for_layer(layer, max_tokens=T, path=moe.PATH_GEMV)
    blk.upload_layer(0, layer)
    blk.set_profiling(True)
    outs = [blk.forward(x)[0] for _ in range(3)]  # epoch flags and arrival counters carry across launches
    st = blk.stats(reset=True)
    blk.close()
    assert st["stage_ms"]["decode_experts"] > 0 and st["stage_ms"]["gate_up"] == 0
    assert all(np.array_equal(o, outs[0]) for o in outs)
    ref_idx = oracle.route(layer, x)[1]
    ref = oracle.moe_block(layer, x)[0]
    assert_block_parity(outs[0], ref)
    assert ref_idx.shape == (T, k)


@pytest.mark.parametrize("path", PATHS)
def test_extreme_scales_incl_denormal(cuda_device, path):
    # E8M0 bytes 0..123: the subnormal 2^-127 scale and ~120 binades of small scales,
    # capped at the configs' 2^-4 so the outputs keep the magnitude the absolute bound assumes
    layer = W.small_layer(hidden=128, intermediate=128, experts=8, top_k=4, seed=4, scale_lo=0, scale_hi=123)
    x = W.make_tokens(W.MoEShape(128, 128, 8, 4), 6, 4)
    check_against_oracle(layer, x, path)


@pytest.mark.parametrize("E,k,T", [(4, 2, 300), (8, 4, 1), (32, 4, 600), (256, 4, 200)])
def test_tensor_path_ragged_token_blocks(cuda_device, E, k, T):
    # several 128-token blocks per expert, 1-token tiles, many empty experts
    layer = W.small_layer(hidden=192, intermediate=320, experts=E, top_k=k, seed=E + T)
    x = W.make_tokens(W.MoEShape(192, 320, E, k), T, E)
    check_against_oracle(layer, x, moe.PATH_TENSOR)


@pytest.mark.parametrize("path", PATHS)
def test_nan_scale_propagates_like_reference(cuda_device, path):
    layer = W.small_layer(hidden=64, intermediate=64, experts=4, top_k=4, seed=9)
    layer["down"].reshape(-1, 17)[5, 0] = 0xFF  # expert 0, one block of down row 2
    x = W.make_tokens(W.MoEShape(64, 64, 4, 4), 2, 9)
    out, idx, w, _ = run_block(layer, x, path)
    ref = oracle.moe_block(layer, x)[0]
    assert np.array_equal(np.isnan(out), np.isnan(ref)) and np.isnan(ref).any()


@pytest.mark.parametrize("path", PATHS)
def test_config0_decode_token(cuda_device, path):
    layer = W.config_layer(0)
    x = W.config_tokens(0)
    max_abs, rel = check_against_oracle(layer, x, path)
    print(f"config0 max-abs {max_abs:.3e} rel-L2 {rel:.3e}")


_REF = {}


def full_reference(config: int, T: int | None = None):
    """(layer, x, oracle out, idx, w, logits) of a benchmark configuration, every row:
    the expert-major oracle, bit-identical to the token-by-token one.  Cached per
    module: several tests compare with the same reference."""
    key = (config, T)
    if key not in _REF:
        layer = W.config_layer(config)
        x = W.config_tokens(config, T)
        _REF[key] = (layer, x) + oracle.moe_block_grouped(layer, x)
    return _REF[key]


def check_full(config: int, path: int, T: int | None = None, max_tokens: int | None = None):
    """Every output row, the top-k of every row and the permutation of one run
    against the oracle; returns (max-abs, rel-L2, rows compared, tie rows)."""
    layer, x, ref_out, ref_idx, ref_w, ref_lg = full_reference(config, T)
    out, idx, w, (logits, perm, counts, offsets) = run_block(layer, x, path, max_tokens)
    ties, bad = routing_mismatches(idx, ref_idx, ref_lg)
    assert not bad, f"routing differs beyond ties on rows {bad[:10]}"
    np.testing.assert_allclose(logits, ref_lg, rtol=0, atol=1e-6)
    p_ref, c_ref, o_ref, _ = oracle.permute(idx, layer["experts"])
    assert np.array_equal(perm, p_ref) and np.array_equal(counts, c_ref) and np.array_equal(offsets, o_ref)
    keep = np.setdiff1d(np.arange(x.shape[0]), ties)
    np.testing.assert_allclose(w[keep], ref_w[keep], rtol=2e-6, atol=0)
    max_abs, rel = assert_block_parity(out, ref_out, keep)
    return max_abs, rel, len(keep), ties, idx


@pytest.mark.parametrize("path", PATHS)
def test_config1_prefill_4096_every_row(cuda_device, path):
    """Config 1 (T=4096, Zipf-skewed routing): all 4096 output rows on both expert paths."""
    max_abs, rel, n, ties, _ = check_full(1, path)
    assert n + len(ties) == 4096
    print(f"config1 path {path}: rows {n} (ties {len(ties)}) max-abs {max_abs:.3e} rel-L2 {rel:.3e}")


@pytest.mark.parametrize("path", PATHS)
def test_config3_decode_batch_256_every_row(cuda_device, path):
    """Config 3 decode batch (T=256, E=128): all 256 rows on both expert paths."""
    max_abs, rel, n, ties, _ = check_full(3, path)
    assert n + len(ties) == 256
    print(f"config3 decode path {path}: rows {n} max-abs {max_abs:.3e} rel-L2 {rel:.3e}")


def test_config3_prefill_8192_every_row(cuda_device):
    """Config 3 prefill (T=8192, E=128, uniform logits) on one GPU: all 8192 rows."""
    max_abs, rel, n, ties, _ = check_full(3, moe.PATH_AUTO, T=8192)
    assert n + len(ties) == 8192
    print(f"config3 prefill: rows {n} max-abs {max_abs:.3e} rel-L2 {rel:.3e}")


def test_config4_adversarial_16384_every_row(cuda_device):
    """Config 4 (T=16384, router bias +4 on experts 0-7) on one GPU: all 16384 rows,
    among them every row routed to a hot expert."""
    max_abs, rel, n, ties, idx = check_full(4, moe.PATH_AUTO)
    assert n + len(ties) == 16384
    hot = np.nonzero((idx < W.HOT_EXPERTS).any(axis=1))[0]
    assert len(hot) > 8192  # the bias sends about half of the pairs to the hot experts
    print(f"config4: rows {n}, hot rows {len(hot)}, max-abs {max_abs:.3e} rel-L2 {rel:.3e}")


def test_device_forward_matches_host_forward_and_is_deterministic(cuda_device):
    import torch

    layer = W.small_layer(hidden=192, intermediate=128, experts=16, top_k=4, seed=21)
    x = W.make_tokens(W.MoEShape(192, 128, 16, 4), 33, 21)
    blk = moe.MoEBlock.for_layer(layer, max_tokens=64)
    blk.upload_layer(0, layer)
    out1, idx1, w1 = blk.forward(x)
    out2, _, _ = blk.forward(x)
    assert np.array_equal(out1, out2)
    xd = torch.from_numpy(x).cuda()
    od = torch.empty_like(xd)
    idd = torch.empty((33, 4), dtype=torch.int32, device="cuda")
    wd = torch.empty((33, 4), dtype=torch.float32, device="cuda")
    blk.forward_device(xd, od, topk_idx=idd, topk_w=wd)
    blk.synchronize()
    assert np.array_equal(od.cpu().numpy(), out1)
    assert np.array_equal(idd.cpu().numpy(), idx1) and np.array_equal(wd.cpu().numpy(), w1)
    blk.close()


def test_errors_are_status_codes(cuda_device):
    layer = W.small_layer()
    blk = moe.MoEBlock.for_layer(layer, max_tokens=8)
    x = W.make_tokens(W.MoEShape(64, 128, 8, 4), 9, 0)
    with pytest.raises(moe.AmoeError) as e:
        blk.forward(x[:2])  # layer 0 not uploaded yet
    assert e.value.code == moe.AMOE_ERR_STATE
    blk.upload_layer(0, layer)
    with pytest.raises(moe.AmoeError) as e:
        blk.forward(x)  # 9 > max_tokens
    assert e.value.code == moe.AMOE_ERR_INVALID
    with pytest.raises(moe.AmoeError) as e:
        blk.forward(x[:0])
    assert e.value.code == moe.AMOE_ERR_INVALID
    bad = dict(layer)
    bad["down"] = layer["down"][:-1]
    with pytest.raises(moe.AmoeError):
        blk.upload_layer(0, bad)
    with pytest.raises(moe.AmoeError) as e:
        blk.upload_layer(3, layer)
    assert e.value.code == moe.AMOE_ERR_INVALID
    out, _, _ = blk.forward(x[:2])  # still usable
    assert np.isfinite(out).all()
    blk.close()


@pytest.mark.parametrize("stream_slots", [0, 2])
def test_allocation_failures_return_nomem_and_keep_the_context_usable(cuda_device, monkeypatch, stream_slots):
    """Host-side fault injection (AMOE_FAIL_ALLOC_ABOVE: device and pinned-host
    allocations above the limit fail as out of memory): amoe_create and
    amoe_upload_layer report AMOE_ERR_NOMEM with a message, and a context whose
    upload failed still uploads and computes once memory is back."""
    layer = W.small_layer(hidden=128, intermediate=128, experts=8, top_k=4, seed=5)
    x = W.make_tokens(W.MoEShape(128, 128, 8, 4), 6, 5)
    monkeypatch.setenv("AMOE_FAIL_ALLOC_ABOVE", "4096")
    with pytest.raises(moe.AmoeError) as e:
        moe.MoEBlock.for_layer(layer, max_tokens=64, stream_slots=stream_slots)
    assert e.value.code == moe.AMOE_ERR_NOMEM and "out of memory" in str(e.value)
    monkeypatch.delenv("AMOE_FAIL_ALLOC_ABOVE")
    blk = moe.MoEBlock.for_layer(layer, max_tokens=64, stream_slots=stream_slots)
    monkeypatch.setenv("AMOE_FAIL_ALLOC_ABOVE", "65536")  # below one layer's device block
    with pytest.raises(moe.AmoeError) as e:
        blk.upload_layer(0, layer)
    assert e.value.code == moe.AMOE_ERR_NOMEM
    with pytest.raises(moe.AmoeError) as e:
        blk.forward(x)  # the layer is still absent
    assert e.value.code == moe.AMOE_ERR_STATE
    monkeypatch.delenv("AMOE_FAIL_ALLOC_ABOVE")
    blk.upload_layer(0, layer)
    out = blk.forward(x)[0]
    blk.close()
    assert_block_parity(out, oracle.moe_block(layer, x)[0])


@pytest.mark.parametrize("T,res_path", [(5, moe.PATH_TENSOR), (3, moe.PATH_AUTO)])
def test_streaming_slots_match_resident_layers(cuda_device, T, res_path):
    # streamed layers carry only the tensor-core planes: T <= 4 runs the fused decode
    # kernel, larger T the block-scaled GEMMs (the resident block is pinned to the same path)
    shape = W.MoEShape(128, 128, 8, 4)
    layers = [W.make_layer(shape, 50 + i) for i in range(3)]
    x = W.make_tokens(shape, T, 50)
    res = moe.MoEBlock(128, 128, 8, 4, layers=3, max_tokens=8, path=res_path)
    stm = moe.MoEBlock(128, 128, 8, 4, layers=3, max_tokens=8, stream_slots=2)
    assert stm.stats()["layer_bytes"] < res.stats()["layer_bytes"]
    for i, L in enumerate(layers):
        res.upload_layer(i, L)
        stm.upload_layer(i, L)
    h_res, h_stm = x, x
    for step in range(2):
        for i in range(3):
            h_res = res.forward(h_res, layer=i)[0]
            h_stm = stm.forward(h_stm, layer=i)[0]  # copies layer i+1 behind this forward
            assert np.array_equal(h_res, h_stm)
        stm.prefetch_layer(2)  # explicit request, then out-of-order use
        for i in (2, 0, 1):
            h_res = res.forward(h_res, layer=i)[0]
            h_stm = stm.forward(h_stm, layer=i)[0]
            assert np.array_equal(h_res, h_stm)
    res.close()
    stm.close()


@pytest.mark.parametrize("path,T,E", [(moe.PATH_AUTO, 3000, 8), (moe.PATH_GEMV, 2500, 16), (moe.PATH_TENSOR, 4100, 32)])
def test_pipelined_host_call_matches_one_device_pass(cuda_device, path, T, E):
    """amoe_forward splits calls of >= 2048 tokens into passes whose host copies
    overlap the neighbouring passes' compute; every pass keeps the call's expert
    path, so outputs, top-k and the reassembled routing equal one device pass."""
    import torch

    layer = W.small_layer(hidden=192, intermediate=128, experts=E, top_k=4, seed=T)
    x = W.make_tokens(W.MoEShape(192, 128, E, 4), T, T)
    blk = moe.MoEBlock.for_layer(layer, max_tokens=T, path=path)
    blk.upload_layer(0, layer)
    out, idx, w = blk.forward(x)  # host buffers: pipelined passes
    routing = blk.last_routing(T)
    xd = torch.from_numpy(x).cuda()
    od = torch.empty_like(xd)
    idd = torch.empty((T, 4), dtype=torch.int32, device="cuda")
    wd = torch.empty((T, 4), dtype=torch.float32, device="cuda")
    blk.forward_device(xd, od, topk_idx=idd, topk_w=wd)  # one pass
    blk.synchronize()
    routing1 = blk.last_routing(T)
    blk.close()
    assert np.array_equal(out, od.cpu().numpy())
    assert np.array_equal(idx, idd.cpu().numpy()) and np.array_equal(w, wd.cpu().numpy())
    for a, b in zip(routing, routing1):
        assert np.array_equal(a, b)


@pytest.mark.parametrize("T", [1, 3, 6, 40])
def test_expert_streaming_matches_resident_layers(cuda_device, T):
    """stream_experts: each call routes first and copies only its routed experts from
    pinned host memory; the output equals resident layers on the same kernels."""
    shape = W.MoEShape(128, 192, 16, 4)
    layers = [W.make_layer(shape, 60 + i) for i in range(3)]
    x = W.make_tokens(shape, T, 60 + T)
    res = moe.MoEBlock(128, 192, 16, 4, layers=3, max_tokens=40, path=moe.PATH_TENSOR)
    stm = moe.MoEBlock(128, 192, 16, 4, layers=3, max_tokens=40, stream_slots=2, stream_experts=1)
    for i, L in enumerate(layers):
        res.upload_layer(i, L)
        stm.upload_layer(i, L)
    h_res, h_stm = x, x
    for i in (0, 1, 2, 1, 0):
        o_res, idx_res, w_res = res.forward(h_res, layer=i)
        o_stm, idx_stm, w_stm = stm.forward(h_stm, layer=i)
        assert np.array_equal(o_res, o_stm) and np.array_equal(idx_res, idx_stm) and np.array_equal(w_res, w_stm)
        h_res, h_stm = o_res, o_stm
    stm.prefetch_layer(2)  # nothing to prefetch before routing: a no-op
    res.close()
    stm.close()


@pytest.mark.parametrize("stream_experts", [0, 1])
def test_streamed_stack_matches_oracle_layer_by_layer(cuda_device, stream_experts):
    """A streamed stack of four config-0-statistics layers (the 20B shape, weights in
    pinned host memory, two device slots or routed-expert copies) decoding three
    steps of two tokens; every layer's output is checked against the oracle run on
    the same input (Generate's layer loop, runtime.go:146-199)."""
    L = 4
    layers = [W.stream_layer(i) for i in range(L)]
    blk = moe.MoEBlock.for_layer(layers[0], layers=L, max_tokens=2, stream_slots=2, stream_experts=stream_experts)
    for i, layer in enumerate(layers):
        blk.upload_layer(i, layer)
    h = W.make_tokens(W.GPTOSS_20B, 2, 2)
    worst = (0.0, 0.0)
    for step in range(3):
        for i in range(L):
            out, idx, _ = blk.forward(h, layer=i)
            ref, ref_idx, _, ref_lg = oracle.moe_block(layers[i], h)
            ties, bad = routing_mismatches(idx, ref_idx, ref_lg)
            assert not bad and not ties, (step, i)
            max_abs, rel = assert_block_parity(out, ref)
            worst = (max(worst[0], max_abs), max(worst[1], rel))
            h = out
    blk.close()
    print(f"streamed stack (stream_experts={stream_experts}): max-abs {worst[0]:.3e} rel-L2 {worst[1]:.3e}")
