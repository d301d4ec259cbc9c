"""The fused decode kernel's work table (amoe_decode_schedule, host arithmetic).

The kernel runs, per CTA, the units this table lists for the number of active
experts, and every cross-CTA hand-off counts arrivals: a box range covered twice
or not at all would corrupt a result or leave a waiter to time out.  These tests
check, for every number of active experts, that the gate_up pieces of every tile
cover its K boxes exactly once in piece order, that every down unit (one per
output tile and K half) appears exactly once, that gate_up pieces come before
down units within every CTA, that the box loads are even to within one down
unit, and that rows fit their fixed size."""
import numpy as np
import pytest

from airllm_b200 import moe

MAX_PIECES = 4


def kpad128(x):
    return (x + 127) // 128 * 128


def decode(w0, w1):
    """(phase, slot, tile, piece, pieces, first K box, end K box, split index)"""
    w0, w1 = w0 & 0xffffffff, w1 & 0xffffffff
    return (w0 >> 31, (w0 >> 20) & 1023, (w0 >> 8) & 4095, (w0 >> 4) & 15, w0 & 15,
            w1 >> 24, (w1 >> 16) & 255, w1 & 0xffff)


@pytest.mark.parametrize("H,I,E,k,G", [
    (2880, 2880, 32, 4, 148),    # GPT-OSS-20B shape on a B200
    (2880, 2880, 128, 4, 148),   # GPT-OSS-120B shape
    (64, 128, 8, 4, 148),        # one K box per down tile: no K halves
    (192, 320, 16, 4, 7),        # more units than CTAs at every n
    (320, 192, 32, 4, 148),
    (64, 64, 256, 8, 148),       # 32 possible active experts
    (2880, 2880, 32, 4, 60),     # long gate_up ranges per CTA
])
def test_every_box_once_gate_up_first_and_balanced(H, I, E, k, G):
    rows = moe.decode_schedule(H, I, E, k, G)
    S = min(E, 4 * k)
    nkb1, nkb2 = kpad128(H) // 128, kpad128(I) // 128
    nmt1, nmt2 = 2 * I // 128, (H + 127) // 128
    nkp, half2 = (2 if nkb2 >= 2 else 1), (nkb2 + 1) // 2
    assert rows.shape == (G, moe.DECODE_SCHED_WORDS)
    for n in range(1, S + 1):
        pieces = {}   # (slot, tile) -> [(piece, pieces, kb0, kb1, split, cta)]
        downs = {}
        loads = np.zeros(G, np.int64)
        for b in range(G):
            row = rows[b]
            assert row[0] == S + 1
            u0, u1 = int(row[n - 1]), int(row[n])
            assert S + 1 <= u0 <= u1 <= moe.DECODE_SCHED_WORDS and (u1 - u0) % 2 == 0
            assert (u1 - u0) // 2 <= 64  # units per CTA the kernel stages
            phases = []
            for w in range(u0, u1, 2):
                ph, sl, mt, pc, npc, kb0, kb1, split = decode(int(row[w]), int(row[w + 1]))
                assert 0 <= sl < n and kb0 < kb1
                phases.append(ph)
                loads[b] += kb1 - kb0
                if ph == 0:
                    assert mt < nmt1 and kb1 <= nkb1 and 1 <= npc <= MAX_PIECES
                    pieces.setdefault((sl, mt), []).append((pc, npc, kb0, kb1, split, b))
                else:
                    assert mt < nmt2 and npc == nkp and pc < nkp and split == 0
                    assert (kb0, kb1) == ((half2 if pc else 0), (nkb2 if nkp == 1 or pc else half2))
                    assert (sl, mt, pc) not in downs, (n, sl, mt, pc, "listed twice")
                    downs[(sl, mt, pc)] = b
            assert phases == sorted(phases), (n, b, "a down unit before a gate_up piece")
        assert set(downs) == {(sl, m, kp) for sl in range(n) for m in range(nmt2) for kp in range(nkp)}
        assert set(pieces) == {(sl, m) for sl in range(n) for m in range(nmt1)}, (n, "gate_up tiles missing")
        splits = set()
        for key, pl in pieces.items():
            pl.sort()
            npc = pl[0][1]
            assert [p[0] for p in pl] == list(range(npc)) and all(p[1] == npc for p in pl), (n, key, pl)
            assert pl[0][2] == 0 and pl[-1][3] == nkb1 and all(pl[i][3] == pl[i + 1][2] for i in range(npc - 1))
            assert len({p[5] for p in pl}) == npc, (n, key, "two pieces of one tile on one CTA")
            if npc > 1:
                assert len({p[4] for p in pl}) == 1 and pl[0][4] < G and pl[0][4] not in splits
                splits.add(pl[0][4])
        assert loads.max() - loads.min() <= max(nkb1, half2), (n, loads.min(), loads.max())


def test_rows_are_deterministic():
    a = moe.decode_schedule(2880, 2880, 32, 4, 148)
    b = moe.decode_schedule(2880, 2880, 32, 4, 148)
    assert np.array_equal(a, b)


@pytest.mark.parametrize("args", [
    (2880, 2880, 32, 0, 148), (2880, 2880, 32, 33, 148), (100, 2880, 32, 4, 148),
    (2880, 8192, 32, 4, 148), (2880, 2880, 300, 4, 148), (2880, 2880, 32, 4, 0),
])
def test_shapes_the_kernel_does_not_run_are_refused(args):
    with pytest.raises(moe.AmoeError) as e:
        moe.decode_schedule(*args)
    assert e.value.code == moe.AMOE_ERR_INVALID
