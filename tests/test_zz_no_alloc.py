"""amoe_route_noalloc against the routing of the regular entry point.

amoe_route_noalloc serves callers that cannot allocate device memory -- a host
runtime that plans every device region up front, or a process whose GPU memory
another allocator already holds.  It keeps its scratch in a fixed device array
inside the library instead of calling cudaMalloc.  It must route exactly like
amoe_forward: same experts, weights and logits, call after call (the array
keeps the previous call's contents, so two calls in a row with different sizes
are checked).  This file is named to run last.
"""
import numpy as np
import pytest

from airllm_b200 import moe
from airllm_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _noalloc(lib, torch, layer, dev, x):
    T, E, k, H = x.shape[0], layer["experts"], layer["top_k"], layer["hidden"]
    xd = torch.from_numpy(x).cuda()
    lg = torch.empty((T, E), dtype=torch.float32, device="cuda")
    ti = torch.empty((T, k), dtype=torch.int32, device="cuda")
    tw = torch.empty((T, k), dtype=torch.float32, device="cuda")
    rc = lib.amoe_route_noalloc(0, H, E, k, layer["eps"], xd.data_ptr(), T, dev["gain"].data_ptr(),
                                dev["w"].data_ptr(), dev["b"].data_ptr(), lg.data_ptr(), ti.data_ptr(),
                                tw.data_ptr(), None)
    assert rc == moe.AMOE_OK, lib.amoe_last_error(None).decode()
    torch.cuda.synchronize()
    return lg.cpu().numpy(), ti.cpu().numpy(), tw.cpu().numpy()


@pytest.mark.parametrize("config,sizes", [(0, (5, 37)), (3, (64, 1))])
def test_noalloc_routing_matches_forward_on_consecutive_calls(cuda_device, config, sizes):
    import torch

    lib = moe.load_library()
    layer = W.config_layer(config)
    shape = W.CONFIG_SHAPE[config]
    dev = {"gain": torch.from_numpy(layer["norm_gain"]).cuda(), "w": torch.from_numpy(layer["router_w"]).cuda(),
           "b": torch.from_numpy(layer["router_b"]).cuda()}
    blk = moe.MoEBlock.for_layer(layer, max_tokens=64)
    blk.upload_layer(0, layer)
    for i, T in enumerate(sizes):  # two calls in a row, different sizes
        x = W.make_tokens(shape, T, 500 + i)
        _, idx, w = blk.forward(x)
        ref_logits = blk.last_routing(T)[0]
        lg, ti, tw = _noalloc(lib, torch, layer, dev, x)
        assert np.array_equal(ti, idx)
        np.testing.assert_allclose(tw, w, rtol=2e-6, atol=0)
        np.testing.assert_allclose(lg, ref_logits, rtol=0, atol=1e-6)
    blk.close()


def test_noalloc_rejects_sizes_beyond_its_fixed_scratch(cuda_device):
    lib = moe.load_library()
    bad = lib.amoe_route_noalloc(0, 2880, 32, 4, 1e-5, 1, 65, 1, 1, 1, 1, 1, 1, None)
    assert bad == moe.AMOE_ERR_INVALID
    assert "64" in lib.amoe_last_error(None).decode()
    assert lib.amoe_route_noalloc(0, 8192, 32, 4, 1e-5, 1, 1, 1, 1, 1, 1, 1, 1, None) == moe.AMOE_ERR_INVALID
    assert lib.amoe_route_noalloc(0, 2880, 256, 4, 1e-5, 1, 1, 1, 1, 1, 1, 1, 1, None) == moe.AMOE_ERR_INVALID
