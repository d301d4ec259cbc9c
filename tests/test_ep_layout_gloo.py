"""Expert-parallel exchange layout on CPU.

Two gloo ranks run the exchange the library performs over NVLink peer memory:
all-gather of the per-expert counts, amoe_ep_layout (the arithmetic the count
kernel runs on the device), placement of every routed row at its row of the
owner's expert-major receive buffer, this rank's experts computed by the oracle,
and the return of each output to its source's sorted position from
(seg_start, src_pos).  The combined result must equal the single-process oracle
bit for bit, and every receive and return slot must be written exactly once."""
import datetime
import os
import socket

import numpy as np
import pytest
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


def layout_np(N, El, me, table):
    """Plain restatement of the layout formulas (per element, no prefix arrays)."""
    E = N * El
    col = table.sum(axis=0)
    send_base = np.array([col[(e // El) * El:e].sum() + table[:me, e].sum() for e in range(E)], np.int64)
    offsets_loc = np.array([col[me * El:me * El + el].sum() for el in range(El + 1)], np.int64)
    seg_start = np.array([[offsets_loc[el] + table[:s, me * El + el].sum() for s in range(N)]
                          for el in range(El)], np.int64)
    src_pos = np.array([[table[s, :me * El + el].sum() for s in range(N)] for el in range(El)], np.int64)
    return send_base, offsets_loc, seg_start, src_pos


@pytest.mark.parametrize("N,El", [(1, 4), (2, 3), (4, 8), (8, 16), (8, 1)])
def test_layout_matches_restatement(N, El):
    rng = np.random.default_rng(N * 100 + El)
    table = rng.integers(0, 9, size=(N, N * El)).astype(np.int32)
    table[:, rng.integers(0, N * El)] = 0  # an expert nobody routes to
    for me in range(N):
        got = moe.ep_layout(N, El, me, table)
        want = layout_np(N, El, me, table)
        for k, w in zip(("send_base", "offsets_loc", "seg_start", "src_pos"), want):
            assert np.array_equal(got[k], w), (me, k)


def test_layout_rejects_bad_arguments():
    with pytest.raises(moe.AmoeError):
        moe.ep_layout(2, 2, 0, -np.ones((2, 4), np.int32))
    with pytest.raises(moe.AmoeError):
        moe.ep_layout(9, 1, 0, np.zeros((9, 9), np.int32))
    with pytest.raises(moe.AmoeError):
        moe.ep_layout(2, 2, 2, np.zeros((2, 4), np.int32))


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
        _, idx, w = oracle.route(layer, x)
        perm, counts, offsets, inv = oracle.permute(idx, E)
        xn = oracle.normalize_rows(layer, x)
        # 1. count table, then the layout every rank derives from it
        tables = [None] * world
        dist.all_gather_object(tables, counts.astype(np.int32))
        table = np.stack(tables)
        lay = moe.ep_layout(world, El, rank, table)
        # 2. dispatch: sorted pair q -> row send_base[e] + (q - offsets[e]) of e's owner
        sends = {q: ([], []) for q in range(world)}
        experts = idx.ravel()[perm]
        for q in range(len(perm)):
            e = int(experts[q])
            sends[e // El][0].append(int(lay["send_base"][e] + q - offsets[e]))
            sends[e // El][1].append(xn[perm[q] // k])
        boxes = [None] * world
        dist.all_gather_object(boxes, sends)
        R = int(lay["offsets_loc"][El])
        recv = np.zeros((R, H), np.float32)
        hits = np.zeros(R, np.int64)
        for src in range(world):
            rows, data = boxes[src][rank]
            for r, v in zip(rows, data):
                recv[r] = v
                hits[r] += 1
        assert (hits == 1).all()
        # 3. this rank's experts, outputs addressed to (source, sorted position)
        y = np.zeros((R, H), np.float32)
        for el in range(El):
            a, b = lay["offsets_loc"][el], lay["offsets_loc"][el + 1]
            if b > a:
                y[a:b] = oracle.expert_rows(layer, rank * El + el, recv[a:b], threads=1)
        back = {q: ([], []) for q in range(world)}
        for p in range(R):
            el = int(np.searchsorted(lay["offsets_loc"], p, side="right") - 1)
            ss = lay["seg_start"][el]
            s = int(np.searchsorted(ss, p, side="right") - 1)
            back[s][0].append(int(lay["src_pos"][el, s] + p - ss[s]))
            back[s][1].append(y[p])
        boxes = [None] * world
        dist.all_gather_object(boxes, back)
        y_back = np.zeros((len(perm), H), np.float32)
        hits = np.zeros(len(perm), np.int64)
        for src in range(world):
            rows, data = boxes[src][rank]
            for r, v in zip(rows, data):
                y_back[r] = v
                hits[r] += 1
        assert (hits == 1).all()
        # 4. combine in slot order (layer.go:109-121)
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
