"""Expert parallelism on 2 GPUs (NCCL) against the single-GPU path, through the
C ABI.  Each rank routes half of the tokens and owns half of the experts; the
per-row arithmetic is identical, so outputs must match bit for bit.  Skips on
boxes with fewer than two GPUs."""
import numpy as np
import pytest

from airllm_b200 import moe
from airllm_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _rank(rank, world, uid, layer, x, path, q):
    try:
        import torch

        torch.cuda.set_device(rank)
        T = x.shape[0] // world
        blk = moe.MoEBlock.for_layer(layer, max_tokens=T, device=rank, ep_size=world, ep_rank=rank,
                                     nccl_id=uid, path=path)
        blk.upload_layer(0, layer)
        outs = [blk.forward(x[rank * T:(rank + 1) * T])[0] for _ in range(2)]  # twice: reused buffers
        blk.close()
        q.put((rank, outs[0], outs[1], None))
    except Exception as exc:
        q.put((rank, None, None, repr(exc)))


@pytest.mark.parametrize("path,T,E", [(moe.PATH_GEMV, 24, 16), (moe.PATH_TENSOR, 256, 16),
                                      (moe.PATH_AUTO, 1024, 8)])
def test_expert_parallel_two_gpus_matches_single_gpu(cuda_device, path, T, E):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    layer = W.make_layer(W.MoEShape(192, 256, E, 4), 41)
    x = W.make_tokens(W.MoEShape(192, 256, E, 4), T, 41)
    ref = moe.MoEBlock.for_layer(layer, max_tokens=T, device=0, path=path)
    ref.upload_layer(0, layer)
    ref_out = ref.forward(x)[0]
    ref.close()
    uid = moe.ep_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, uid, layer, x, path, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    for _ in procs:
        rank, o1, o2, err = q.get(timeout=300)
        assert err is None, f"rank {rank}: {err}"
        results[rank] = (o1, o2)
    for p in procs:
        p.join(timeout=60)
    half = T // 2
    for r in range(2):
        o1, o2 = results[r]
        assert np.array_equal(o1, ref_out[r * half:(r + 1) * half])
        assert np.array_equal(o2, o1)
