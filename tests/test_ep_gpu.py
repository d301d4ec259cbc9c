"""Expert parallelism on 2, 4 and 8 GPUs, through the C ABI, against the oracle
and against the single-GPU path.  Each rank routes its own tokens and owns E/N
experts; rows and outputs move by stores into the peers' memory.  The per-row
arithmetic is identical to one GPU, so outputs must match it bit for bit --
including ranks with different token counts, a rank with a single token, and
repeated steps (the exchange's buffers and epoch flags are reused) -- and every
output row must meet the oracle parity bar.  The GPT-OSS-120B-shaped prefill
(8192 tokens, 128 experts) runs at 2, 4 and 8 GPUs and the adversarial 16384-token
configuration at 8.  A rank that never calls forward makes the others fail with a
timeout status (bounded device waits, no GPU fault).  Skips on boxes with too few
GPUs.  NVLS stays off (the exchange uses plain peer stores; NCCL only trades the
IPC handles at create)."""
import os

import numpy as np
import pytest

import oracle
from airllm_b200 import moe
from airllm_b200 import workloads as W
from parity_util import assert_block_parity, routing_mismatches

pytestmark = pytest.mark.gpu


def _steps(world, T):
    """Per step, the token rows each rank forwards (ragged, one single-token rank)."""
    rng = np.random.default_rng(world * 1000 + T)
    steps = [np.array_split(np.arange(T), world)]
    cuts = np.sort(rng.choice(np.arange(1, T), size=world - 1, replace=False))
    steps.append(np.split(np.arange(T), cuts))
    one = [np.arange(0, 1)] + [np.arange(1 + r, T, world) for r in range(world - 1)]
    steps.append(one)
    steps.append(steps[0])
    return steps


def _workload(spec):
    """(layer, x) of a spec: ("config", index, T) regenerates a benchmark
    configuration from its seed (cheaper than sending 1.7 GB to every process);
    ("arrays", layer, x) passes them as they are."""
    if spec[0] == "config":
        return W.config_layer(spec[1]), W.config_tokens(spec[1], spec[2])
    return spec[1], spec[2]


def _rank(rank, world, uid, spec, path, steps, q):
    try:
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        import torch

        torch.cuda.set_device(rank)
        layer, x = _workload(spec)
        max_t = max(len(s[r]) for s in steps for r in range(world))
        blk = moe.MoEBlock.for_layer(layer, max_tokens=max_t, device=rank, ep_size=world, ep_rank=rank,
                                     nccl_id=uid, path=path)
        blk.upload_layer(0, layer)
        del layer
        res = [blk.forward(x[s[rank]]) for s in steps]
        blk.close()
        q.put((rank, [r[0] for r in res], [r[1] for r in res], None))
    except Exception as exc:
        q.put((rank, None, None, repr(exc)))


_ORACLE = {}


def _oracle(spec):
    key = (spec[0], spec[1], spec[2]) if spec[0] == "config" else None
    if key is not None and key in _ORACLE:
        return _ORACLE[key]
    layer, x = _workload(spec)
    ref = (layer, x) + oracle.moe_block_grouped(layer, x)
    if key is not None:
        _ORACLE.clear()  # one large reference at a time
        _ORACLE[key] = ref
    return ref


def _run(world, path, spec, steps=None):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    layer, x, ref_out, ref_idx, _, ref_lg = _oracle(spec)
    T = x.shape[0]
    one = moe.MoEBlock.for_layer(layer, max_tokens=T, device=0, path=path)
    one.upload_layer(0, layer)
    one_out = one.forward(x)[0]
    one.close()
    steps = steps or _steps(world, T)
    uid = moe.ep_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, uid, spec, path, steps, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in procs:
        rank, outs, idxs, err = q.get(timeout=600)
        assert err is None, f"rank {rank}: {err}"
        results[rank] = (outs, idxs)
    for p in procs:
        p.join(timeout=60)
    worst = (0.0, 0.0)
    for i, s in enumerate(steps):
        rows = np.concatenate([s[r] for r in range(world)])  # a step need not cover every row
        out = np.zeros_like(x)
        idx = ref_idx.copy()
        for r in range(world):
            assert np.array_equal(results[r][0][i], one_out[s[r]]), (r, i)
            out[s[r]] = results[r][0][i]
            idx[s[r]] = results[r][1][i]
        ties, bad = routing_mismatches(idx[rows], ref_idx[rows], ref_lg[rows])
        assert not bad, f"step {i}: routing differs beyond ties on rows {rows[bad][:10]}"
        max_abs, rel = assert_block_parity(out, ref_out, np.setdiff1d(rows, rows[ties]))
        worst = (max(worst[0], max_abs), max(worst[1], rel))
    return worst


def _small(H, I, E, T, seed=41):
    return ("arrays", W.make_layer(W.MoEShape(H, I, E, 4), seed), W.make_tokens(W.MoEShape(H, I, E, 4), T, seed))


@pytest.mark.parametrize("path,T,E", [(moe.PATH_GEMV, 24, 16), (moe.PATH_GEMV, 5, 8), (moe.PATH_TENSOR, 256, 16),
                                      (moe.PATH_AUTO, 1024, 8)])
def test_expert_parallel_two_gpus_matches_single_gpu(cuda_device, path, T, E):
    _run(2, path, _small(192, 256, E, T))


@pytest.mark.parametrize("path,T,E", [(moe.PATH_GEMV, 40, 128), (moe.PATH_TENSOR, 600, 32)])
def test_expert_parallel_four_gpus_matches_single_gpu(cuda_device, path, T, E):
    _run(4, path, _small(192, 256, E, T))


@pytest.mark.parametrize("path,T,E", [(moe.PATH_GEMV, 64, 64), (moe.PATH_AUTO, 2048, 32)])
def test_expert_parallel_eight_gpus_matches_single_gpu(cuda_device, path, T, E):
    _run(8, path, _small(192, 256, E, T))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_expert_parallel_gptoss120b_prefill_8192(cuda_device, world):
    """Config 3 prefill: 8192 tokens, 128 experts sharded 128/N; an even and a
    ragged split of the tokens over the ranks; every output row against the oracle."""
    steps = _steps(world, 8192)[:2]
    max_abs, rel = _run(world, moe.PATH_AUTO, ("config", 3, 8192), steps)
    print(f"config3 prefill ep{world}: max-abs {max_abs:.3e} rel-L2 {rel:.3e}")


@pytest.mark.parametrize("world", [2, 8])
def test_expert_parallel_gptoss120b_decode_256(cuda_device, world):
    """Config 3 decode batch: 256 tokens over N ranks (the GEMV exchange path)."""
    max_abs, rel = _run(world, moe.PATH_AUTO, ("config", 3, 256), _steps(world, 256)[:3])
    print(f"config3 decode ep{world}: max-abs {max_abs:.3e} rel-L2 {rel:.3e}")


def test_expert_parallel_adversarial_16384_eight_gpus(cuda_device):
    """Config 4: 16384 tokens, the 8 hot experts (router bias +4) all on rank 0."""
    steps = [np.array_split(np.arange(16384), 8)]
    max_abs, rel = _run(8, moe.PATH_AUTO, ("config", 4, 16384), steps)
    print(f"config4 ep8: max-abs {max_abs:.3e} rel-L2 {rel:.3e}")


def _absent_rank(rank, uid, layer, x, q, done):
    try:
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        os.environ["AMOE_EP_WAIT_MS"] = "1500"
        import torch

        torch.cuda.set_device(rank)
        blk = moe.MoEBlock.for_layer(layer, max_tokens=8, device=rank, ep_size=2, ep_rank=rank, nccl_id=uid,
                                     path=moe.PATH_GEMV)
        blk.upload_layer(0, layer)
        codes = []
        if rank == 0:  # rank 1 never calls forward: the count exchange runs out
            for _ in range(2):
                try:
                    blk.forward(x)
                    codes.append(0)
                except moe.AmoeError as e:
                    codes.append(e.code)
            done.set()
        else:
            done.wait(120)  # leaves only after rank 0 has stopped writing to its window
        blk.close()
        q.put((rank, codes, None))
    except Exception as exc:
        q.put((rank, None, repr(exc)))


def test_missing_rank_times_out_with_status(cuda_device):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    layer = W.make_layer(W.MoEShape(64, 64, 8, 4), 3)
    x = W.make_tokens(W.MoEShape(64, 64, 8, 4), 4, 3)
    uid = moe.ep_unique_id()
    ctx = mp.get_context("spawn")
    q, done = ctx.Queue(), ctx.Event()
    procs = [ctx.Process(target=_absent_rank, args=(r, uid, layer, x, q, done)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    for _ in procs:
        rank, codes, err = q.get(timeout=300)
        assert err is None, f"rank {rank}: {err}"
        results[rank] = codes
    for p in procs:
        p.join(timeout=60)
    # first forward: the bounded wait gives up; second: the group is marked out of step
    assert results[0] == [moe.AMOE_ERR_TIMEOUT, moe.AMOE_ERR_STATE]
