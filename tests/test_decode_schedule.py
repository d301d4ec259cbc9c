"""The fused decode kernel's work table (amoe_decode_schedule, host arithmetic).

The kernel runs, per CTA, the units this table lists for the number of active
experts, and every cross-CTA hand-off counts arrivals: a unit listed twice or
not at all would corrupt a result or leave a waiter to time out.  These tests
check, for every number of active experts, that each unit appears exactly once,
that gate_up units come before down units within every CTA, that the box loads
are balanced to within one unit, and that rows fit their fixed size."""
import numpy as np
import pytest

from airllm_b200 import moe


def kpad128(x):
    return (x + 127) // 128 * 128


def decode(code):
    return (code >> 30) & 1, (code >> 20) & 1023, (code >> 8) & 4095, code & 1


def expected_units(H, I, n):
    nkb1, nkb2 = kpad128(H) // 128, kpad128(I) // 128
    nmt1, nmt2 = 2 * I // 128, (H + 127) // 128
    nkp, half2 = (2 if nkb2 >= 2 else 1), (nkb2 + 1) // 2
    units = {}
    for sl in range(n):
        for m in range(nmt1):
            units[(0, sl, m, 0)] = nkb1
        for m in range(nmt2):
            for kp in range(nkp):
                units[(1, sl, m, kp)] = nkb2 if nkp == 1 else (nkb2 - half2 if kp else half2)
    return units


@pytest.mark.parametrize("H,I,E,k,G", [
    (2880, 2880, 32, 4, 148),    # GPT-OSS-20B shape on a B200
    (2880, 2880, 128, 4, 148),   # GPT-OSS-120B shape
    (64, 128, 8, 4, 148),        # one K box per down tile: no K halves
    (192, 320, 16, 4, 7),        # more units than CTAs at every n
    (320, 192, 32, 4, 148),
    (64, 64, 256, 8, 148),       # 32 possible active experts
])
def test_every_unit_once_gate_up_first_and_balanced(H, I, E, k, G):
    rows = moe.decode_schedule(H, I, E, k, G)
    S = min(E, 4 * k)
    assert rows.shape == (G, moe.DECODE_SCHED_WORDS)
    for n in range(1, S + 1):
        want = expected_units(H, I, n)
        seen = {}
        loads = np.zeros(G, np.int64)
        for b in range(G):
            row = rows[b]
            assert row[0] == S + 1
            u0, u1 = int(row[n - 1]), int(row[n])
            assert S + 1 <= u0 <= u1 <= moe.DECODE_SCHED_WORDS
            assert u1 - u0 <= 64  # units per CTA the kernel stages
            phases = []
            for code in row[u0:u1]:
                u = decode(int(code))
                assert u in want, (n, b, u)
                assert u not in seen, (n, u, "listed twice")
                seen[u] = b
                loads[b] += want[u]
                phases.append(u[0])
            assert phases == sorted(phases), (n, b, "a down unit before a gate_up unit")
        assert set(seen) == set(want), (n, "units missing")
        assert loads.max() - loads.min() <= max(want.values()), (n, loads.min(), loads.max())


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
