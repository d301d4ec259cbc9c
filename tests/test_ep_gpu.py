"""Expert parallelism on 2 (and 4) GPUs against the single-GPU path, through the
C ABI.  Each rank routes its own tokens and owns E/N experts; rows and outputs
move by stores into the peers' memory.  The per-row arithmetic is identical to
one GPU, so outputs must match bit for bit -- including ranks with different
token counts, a rank with a single token, and repeated steps (the exchange's
buffers and epoch flags are reused).  A rank that never calls forward makes the
others fail with a timeout status (bounded device waits, no GPU fault).  Skips
on boxes with too few GPUs.  NVLS stays off (the exchange uses plain peer
stores; NCCL only trades the IPC handles at create)."""
import os

import numpy as np
import pytest

from airllm_b200 import moe
from airllm_b200 import workloads as W

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


def _rank(rank, world, uid, layer, x, path, steps, q):
    try:
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        import torch

        torch.cuda.set_device(rank)
        max_t = max(len(s[r]) for s in steps for r in range(world))
        blk = moe.MoEBlock.for_layer(layer, max_tokens=max_t, device=rank, ep_size=world, ep_rank=rank,
                                     nccl_id=uid, path=path)
        blk.upload_layer(0, layer)
        outs = [blk.forward(x[s[rank]])[0] for s in steps]
        blk.close()
        q.put((rank, outs, None))
    except Exception as exc:
        q.put((rank, None, repr(exc)))


def _run(world, path, T, E, H=192, I=256, seed=41):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    layer = W.make_layer(W.MoEShape(H, I, E, 4), seed)
    x = W.make_tokens(W.MoEShape(H, I, E, 4), T, seed)
    ref = moe.MoEBlock.for_layer(layer, max_tokens=T, device=0, path=path)
    ref.upload_layer(0, layer)
    ref_out = ref.forward(x)[0]
    ref.close()
    steps = _steps(world, T)
    uid = moe.ep_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, uid, layer, x, path, steps, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in procs:
        rank, outs, err = q.get(timeout=300)
        assert err is None, f"rank {rank}: {err}"
        results[rank] = outs
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        for i, s in enumerate(steps):
            assert np.array_equal(results[r][i], ref_out[s[r]]), (r, i)


@pytest.mark.parametrize("path,T,E", [(moe.PATH_GEMV, 24, 16), (moe.PATH_GEMV, 5, 8), (moe.PATH_TENSOR, 256, 16),
                                      (moe.PATH_AUTO, 1024, 8)])
def test_expert_parallel_two_gpus_matches_single_gpu(cuda_device, path, T, E):
    _run(2, path, T, E)


@pytest.mark.parametrize("path,T,E", [(moe.PATH_GEMV, 40, 128), (moe.PATH_TENSOR, 600, 32)])
def test_expert_parallel_four_gpus_matches_single_gpu(cuda_device, path, T, E):
    _run(4, path, T, E)


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
