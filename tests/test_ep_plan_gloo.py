"""Expert-parallel exchange on CPU: two gloo ranks run the same exchange the
library performs with NCCL -- count exchange, amoe_ep_plan (the library's host
planning step), row dispatch, expert-major reorder by the plan's segments,
return of the outputs, combine -- with the oracle computing each rank's
experts.  The result must equal the single-process oracle bit for bit."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from airllm_b200 import moe
from airllm_b200 import workloads as W

SHAPE = W.MoEShape(64, 64, 8, 3)
TOKENS_PER_RANK = 21


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _exchange(world, rank, send, send_off, send_rows, recv_off, recv_rows, width, dtype):
    """Variable all-to-all of row blocks over gloo point-to-point."""
    out = np.zeros((int(recv_off[-1] + recv_rows[-1]), width), dtype)
    reqs, bufs = [], []
    for q in range(world):
        if q == rank:
            out[recv_off[q]:recv_off[q] + recv_rows[q]] = send[send_off[q]:send_off[q] + send_rows[q]]
            continue
        if send_rows[q]:
            reqs.append(dist.isend(torch.from_numpy(np.ascontiguousarray(
                send[send_off[q]:send_off[q] + send_rows[q]])), q))
        if recv_rows[q]:
            b = torch.empty((int(recv_rows[q]), width), dtype=torch.from_numpy(np.zeros(1, dtype)).dtype)
            bufs.append((q, b))
            reqs.append(dist.irecv(b, q))
    for r in reqs:
        r.wait()
    for q, b in bufs:
        out[recv_off[q]:recv_off[q] + recv_rows[q]] = b.numpy()
    return out


def _rank(rank, world, port, failures):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        layer = W.make_layer(SHAPE, 31)
        E, k, H = SHAPE.experts, SHAPE.top_k, SHAPE.hidden
        El = E // world
        x_all = W.make_tokens(SHAPE, world * TOKENS_PER_RANK, 31)
        x = x_all[rank * TOKENS_PER_RANK:(rank + 1) * TOKENS_PER_RANK]
        # local routing and expert-sorted rows
        _, idx, w = oracle.route(layer, x)
        perm, counts, offsets, inv = oracle.permute(idx, E)
        xn = oracle.normalize_rows(layer, x)
        rows = xn[perm // k]
        # 1. counts to every rank
        gathered = [torch.zeros(E, dtype=torch.int32) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(counts))
        recv_counts = np.stack([g.numpy()[rank * El:(rank + 1) * El] for g in gathered])
        # 2. the library's plan
        plan = moe.ep_plan(world, El, rank, offsets, recv_counts)
        assert plan["send_off"].tolist() == [int(offsets[q * El]) for q in range(world)]
        # 3. dispatch, reorder expert-major, run this rank's experts
        recv = _exchange(world, rank, rows, plan["send_off"], plan["send_rows"], plan["recv_off"],
                         plan["recv_rows"], H, np.float32)
        R = recv.shape[0]
        ex = np.zeros_like(recv)
        ret = np.zeros(R, np.int64)
        for src, dst, n in plan["segments"]:
            ex[dst:dst + n] = recv[src:src + n]
            ret[dst:dst + n] = np.arange(src, src + n)
        y_send = np.zeros((R, H), np.float32)
        for e in range(El):
            a, b = plan["offsets_loc"][e], plan["offsets_loc"][e + 1]
            if b > a:
                y_send[ret[a:b]] = oracle.expert_rows(layer, rank * El + e, ex[a:b], threads=1)
        # 4. outputs back, combine in slot order (layer.go:109-121)
        y_back = _exchange(world, rank, y_send, plan["recv_off"], plan["recv_rows"], plan["send_off"],
                           plan["send_rows"], H, np.float32)
        out = np.empty_like(x)
        for t in range(x.shape[0]):
            mix = np.zeros(H)
            for s in range(k):
                mix += np.float64(w[t, s]) * y_back[inv[t * k + s]].astype(np.float64)
            out[t] = x[t] + mix.astype(np.float32)
        ref = oracle.moe_block(layer, x, threads=1)[0]
        assert np.array_equal(out, ref), float(np.abs(out - ref).max())
        dist.destroy_process_group()
    except Exception as exc:  # reported to the parent
        failures.put(f"rank {rank}: {exc!r}")
        raise


def test_expert_parallel_exchange_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    failures = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, failures)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("gloo rank did not finish")
    errs = []
    while not failures.empty():
        errs.append(failures.get())
    assert not errs and all(p.exitcode == 0 for p in procs), errs


def test_plan_rejects_inconsistent_counts():
    with pytest.raises(moe.AmoeError):
        # expert offsets must not decrease
        moe.ep_plan(2, 4, 0, np.array([0, 1, 2, 3, 5, 5, 5, 5, 2], np.int32), np.zeros((2, 4), np.int32))
    with pytest.raises(moe.AmoeError):
        moe.ep_plan(2, 4, 0, np.arange(9, dtype=np.int32), -np.ones((2, 4), np.int32))
    plan = moe.ep_plan(2, 4, 1, np.arange(9, dtype=np.int32), np.array([[1, 0, 2, 0], [0, 3, 0, 1]], np.int32))
    assert plan["recv_rows"].tolist() == [3, 4] and plan["offsets_loc"].tolist() == [0, 1, 4, 6, 7]
    assert plan["segments"].tolist() == [[0, 0, 1], [1, 1, 0], [1, 4, 2], [3, 6, 0],
                                         [3, 1, 0], [3, 1, 3], [6, 6, 0], [6, 6, 1]]
