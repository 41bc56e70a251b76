"""Expert residency state (free-first slots, LFU victim, pins, over-capacity
refusal): the native manager (``vb_res_*``) against the oracle restatement
and both against the reference's own model of its demand state machine.

Host logic only: these tests call the library's host functions and launch
nothing on a GPU.
"""
import json
import os
import random

import pytest

from oracle.residency import ResidencyOracle

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "residency_refreal.json")


def _native(*a, **k):
    from vates_b200.residency import NativeResidency
    return NativeResidency(*a, **k)


def _golden_cases():
    with open(GOLDEN) as f:
        return json.load(f)["cases"]


@pytest.mark.parametrize("which", ["oracle", "native"])
def test_matches_reference_refreal_sequences(which):
    """test_demand_dual_native.py:826-840 (seed 12345, cap 4, 200 requests) and
    four more seeded sequences: every slot and every resident set."""
    for case in _golden_cases():
        cap, E = case["cap"], case["num_experts"]
        m = (ResidencyOracle if which == "oracle" else _native)(
            1, cap, E, lfu=case["lfu"], decay_interval=case["decay"])
        for step, (flat, want, res) in enumerate(zip(case["requests"], case["local"],
                                                    case["resident"])):
            local, place, stats, over = m.demand(0, flat)
            assert not over
            assert local == want, f"seed {case['seed']} step {step}"
            if which == "oracle":
                got_res = sorted(m.L[0].e2r.items())
            else:
                got_res = sorted(m.resident(0))
            assert got_res == [tuple(p) for p in res], f"seed {case['seed']} step {step}"
            assert stats[2] == len(place)


def _random_ops(seed, cap, E, steps, pin_rate=0.05, max_req=None):
    rng = random.Random(seed)
    ops = []
    for _ in range(steps):
        layer = rng.randrange(2)
        if rng.random() < pin_rate:
            ops.append(("pin", layer, [rng.randrange(E) for _ in range(rng.randint(1, 2))]))
        else:
            n = rng.randint(1, max_req or cap + 2)
            # skewed ids so that LFU counts differ
            ops.append(("demand", layer, [min(E - 1, int(rng.expovariate(0.15))) for _ in range(n)]))
    return ops


@pytest.mark.parametrize("cap,E,lfu,decay,seed", [(4, 16, True, 0, 1), (8, 40, True, 0, 2),
                                                  (8, 40, False, 0, 3), (6, 24, True, 7, 4),
                                                  (12, 64, True, 3, 5), (3, 10, True, 1, 6)])
def test_native_matches_oracle_with_pins_and_overcapacity(cap, E, lfu, decay, seed):
    """Random demands on two layers with duplicates, occasional pins and
    requests larger than the pool: outputs, tables, counts and order agree."""
    orc = ResidencyOracle(2, cap, E, lfu=lfu, decay_interval=decay)
    nat = _native(2, cap, E, lfu=lfu, decay_interval=decay)
    n_over = n_pin_err = 0
    for step, (kind, layer, ids) in enumerate(_random_ops(seed, cap, E, 600)):
        if kind == "pin":
            try:
                want = orc.pin(layer, ids)
            except ValueError:
                with pytest.raises(ValueError):
                    nat.pin(layer, ids)
                n_pin_err += 1
                continue
            assert nat.pin(layer, ids) == want, f"step {step}"
        else:
            want = orc.demand(layer, ids)
            got = nat.demand(layer, ids)
            assert got[0] == want[0] and got[1] == want[1], f"step {step}"
            assert tuple(got[2]) == tuple(want[2]) and got[3] == want[3], f"step {step}"
            n_over += int(want[3])
        for l in range(2):
            c = orc.L[l]
            assert nat.table(l) == c.table, f"step {step}"
            assert nat.resident(l) == [(e, c.e2r[e]) for e in c.order], f"step {step}"
            assert nat.counts(l) == {e: f for e, f in c.freq.items() if f}, f"step {step}"
    assert n_over > 0  # the sequences do reach the refusal path
    del n_pin_err


def test_known_answers_from_reference_pool_tests():
    """Scenarios of test_resident_pool.py and test_demand_dual_native.py,
    restated on the native state (no data movement)."""
    # miss then hit: same slots (test_resident_pool.py:112-121)
    r = _native(1, 4, 16)
    a = r.demand(0, [2, 5])
    b = r.demand(0, [2, 5])
    assert a[0] == b[0] and a[2] == (0, 2, 2) and b[2] == (2, 0, 0)
    # LFU keeps the frequent expert over the oldest (242-254)
    r = _native(1, 2, 8)
    for ids in ([0], [1], [0], [0], [1], [2]):
        r.demand(0, ids)
    assert r.demand(0, [0])[2] == (1, 0, 0)
    # pinned expert survives eviction (219-229)
    r = _native(1, 2, 8)
    r.pin(0, [0])
    r.demand(0, [1])
    r.demand(0, [2])
    assert r.demand(0, [0])[2] == (1, 0, 0)
    # decay off: counts keep growing (256-265); interval 4 halves 4 -> 2 (267-275)
    r = _native(1, 4, 8)
    for _ in range(20):
        r.demand(0, [0])
    assert r.counts(0) == {0: 20}
    r = _native(1, 4, 8, decay_interval=4)
    for _ in range(4):
        r.demand(0, [0])
    assert r.counts(0) == {0: 2}
    # all-hit demands count too (277-286)
    r = _native(1, 4, 8)
    r.demand(0, [2, 5])
    for _ in range(3):
        r.demand(0, [2, 5])
    assert r.counts(0) == {2: 4, 5: 4}
    # counting off (288-295)
    r = _native(1, 4, 8, lfu=False)
    r.demand(0, [2, 5])
    r.demand(0, [2, 5])
    assert r.counts(0) == {}
    # per-layer isolation (136-140)
    r = _native(2, 2, 8)
    r.demand(0, [0, 1])
    r.demand(1, [0, 1])
    assert len(r.resident(0)) == 2 and len(r.resident(1)) == 2
    # within capacity nothing is evicted (194-204)
    r = _native(1, 16, 32)
    for e in range(16):
        r.demand(0, [e])
    assert all(r.demand(0, [e])[2] == (1, 0, 0) for e in range(16))
    # all-miss request places every id in its own slot
    # (test_demand_dual_native.py:45-62: stats [0, 3, 3])
    r = _native(1, 4, 16)
    local, place, stats, over = r.demand(0, [5, 6, 7])
    assert stats == (0, 3, 3) and sorted(local) == [0, 1, 2] and not over
    assert place == [(5, 0), (6, 1), (7, 2)]
    # over capacity leaves the state untouched (233-248: stats [0, 5, 0])
    r = _native(1, 4, 16)
    local, place, stats, over = r.demand(0, [1, 2, 3, 4, 5])
    assert over and stats == (0, 5, 0) and local == [0] * 5 and place == []
    assert r.resident(0) == [] and r.table(0) == [-1] * 16


def test_pin_refusal_and_protection():
    r = _native(1, 3, 10)
    r.pin(0, [1, 2])
    with pytest.raises(ValueError):
        r.pin(0, [3, 4])            # 4 pinned > 3 slots: nothing changes
    assert sorted(e for e, _ in r.resident(0)) == [1, 2]
    # a request needing 2 experts plus 2 pins it does not use: refused
    assert r.demand(0, [5, 6])[3]
    # the pins are never victims
    r.demand(0, [5])
    r.demand(0, [6])
    assert {1, 2} <= {e for e, _ in r.resident(0)}


def test_invalid_arguments_raise():
    from vates_b200._lib import VbError
    r = _native(1, 4, 8)
    with pytest.raises(VbError):
        r.demand(0, [8])            # expert id out of range
    with pytest.raises(VbError):
        r.demand(1, [0])            # layer out of range
    with pytest.raises(VbError):
        _native(0, 4, 8)
