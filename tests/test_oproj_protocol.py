"""Slot-reuse protocol of the fused o_proj + all-reduce (csrc/oproj_allreduce.cu), checked on
CPU over random schedules.  This models the protocol, not the kernel.

Each rank runs calls e = 1, 2, ... one after another (stream order).  A call covers M_e rows,
split into work units (units of one call run concurrently, in any order; a unit may be empty,
unit 0 never is; the same unit index covers different rows in different calls).  Per unit:
  push     write this rank's rows of the unit into every rank's slot[e % 2][this rank]
  publish  set every rank's ready flag [unit][this rank] = e
  wait     until this rank's flags [unit][r] show e for every r: e, or e + 1 when rank r is
           one call ahead (low-latency words instead: the slot words themselves hold e)
  read     slot[e % 2][r][rows] for every r, an interval from begin to end
A call ends when its units are read; nothing else orders the ranks.  The checker asserts that
every read sees epoch-e data, that no push overwrites rows while they are being read, and that
no schedule deadlocks.
"""
import random

import pytest


class Violation(AssertionError):
    pass


def simulate(ranks, calls, seed, low_latency=False, parities=2, exact_flags=False, max_rows=12):
    """low_latency: False, True, or "mixed" (each call picks; low-latency calls use their own
    slot buffer, as small batches do)."""
    rng = random.Random(seed)
    plans, modes = [], []  # per call: list of units (each a list of rows), low-latency or not
    for _ in range(calls):
        m = rng.randint(1, max_rows)
        nu = rng.randint(1, 4)
        per = -(-m // nu)
        units = [list(range(min(m, i * per), min(m, (i + 1) * per))) for i in range(nu)]
        plans.append(units)
        modes.append(rng.random() < 0.5 if low_latency == "mixed" else bool(low_latency))
    slot, flag, reading = {}, {}, {}
    cur = [0] * ranks  # index of the running call
    prog = [[0 if rows else 4 for rows in plans[0]] for _ in range(ranks)]
    done = [False] * ranks

    def shows(v, e):
        return v == e or (not exact_flags and v == e + 1)

    while not all(done):
        actions = []
        for r in range(ranks):
            if done[r]:
                continue
            e = cur[r] + 1
            ll = modes[cur[r]]
            par = (ll, e % parities)
            for u, rows in enumerate(plans[cur[r]]):
                st = prog[r][u]
                if st == 0:
                    actions.append((r, u, "push"))
                elif st == 1:
                    actions.append((r, u, "publish"))
                elif st == 2:
                    if ll:
                        ok = all(slot.get((r, par, s, row)) == e for s in range(ranks) for row in rows)
                    else:
                        ok = all(shows(flag.get((r, u, s), 0), e) for s in range(ranks))
                    if ok:
                        actions.append((r, u, "begin"))
                elif st == 3:
                    actions.append((r, u, "end"))
            if all(p == 4 for p in prog[r]):
                actions.append((r, None, "next"))
        if not actions:
            raise Violation("deadlock")
        r, u, a = rng.choice(actions)
        e = cur[r] + 1
        ll = modes[cur[r]]
        par = (ll, e % parities)
        rows = plans[cur[r]][u] if u is not None else []
        if a == "push":
            for q in range(ranks):
                for row in rows:
                    key = (q, par, r, row)
                    if key in reading:
                        raise Violation(f"rank {r} call {e} overwrites rank {q}'s row {row} "
                                        f"while it reads call {reading[key]}")
                    slot[key] = e
            prog[r][u] = 2 if ll else 1
        elif a == "publish":
            for q in range(ranks):
                flag[(q, u, r)] = e
            prog[r][u] = 2
        elif a in ("begin", "end"):
            for s in range(ranks):
                for row in rows:
                    key = (r, par, s, row)
                    if slot.get(key) != e:
                        raise Violation(f"rank {r} call {e} reads epoch {slot.get(key)} data from rank {s}")
                    if a == "begin":
                        reading[key] = e
                    else:
                        del reading[key]
            prog[r][u] = 3 if a == "begin" else 4
        else:
            if cur[r] + 1 == calls:
                done[r] = True
            else:
                cur[r] += 1
                prog[r] = [0 if rows_ else 4 for rows_ in plans[cur[r]]]
    return True


@pytest.mark.parametrize("low_latency", [False, True, "mixed"])
@pytest.mark.parametrize("ranks", [2, 3, 4])
def test_protocol_holds_on_random_schedules(ranks, low_latency):
    for seed in range(150):
        assert simulate(ranks, calls=10, seed=seed, low_latency=low_latency)


def test_checker_catches_a_single_slot_buffer():
    """A planted mistake: one slot buffer instead of two alternating by parity."""
    caught = 0
    for seed in range(150):
        try:
            simulate(2, calls=10, seed=seed, parities=1)
        except Violation:
            caught += 1
    assert caught > 0


def test_checker_catches_exact_flag_match_as_a_deadlock():
    """A planted mistake: ready flags that must equal e exactly.  A peer one call ahead has
    already overwritten the flag with e + 1, so some schedules stall."""
    caught = 0
    for seed in range(300):
        try:
            simulate(2, calls=10, seed=seed, exact_flags=True)
        except Violation:
            caught += 1
    assert caught > 0
