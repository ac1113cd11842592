"""CPU model of the barrier protocol of the backward kernel (packed_encoders_b200/csrc/attn_bwd.cuh):
the producer, MMA and compute roles of one CTA as coroutines over mbarrier phase counts, run in
random interleavings. Each role yields ('wait', barrier, k): phase k must have completed, with the
parity semantics of mbarrier.try_wait.parity (a waiter that falls two phases behind is reported as
parity aliasing). Commits and TMA completions are modelled as immediate arrivals. The model checks
that every role finishes and that no TMEM region or shared-memory tile is overwritten before its
reader is done. The roles follow the kernel's loops statement by statement; a change to the
kernel's barrier protocol must be mirrored here.
"""

import random

import pytest

class Bars:
    def __init__(s, counts):
        s.count = dict(counts); s.arr = {b: 0 for b in counts}; s.done = {b: 0 for b in counts}
    def arrive(s, b):
        s.arr[b] += 1
        if s.arr[b] == s.count[b]:
            s.arr[b] = 0; s.done[b] += 1

def run(units, order="new", seed=0, verbose=False):
    rnd = random.Random(seed)
    B = Bars({"kv_full": 1, "kv_empty": 1, "qd_full0": 1, "qd_full1": 1, "qd_empty0": 1, "qd_empty1": 1,
              "row_empty0": 1, "row_empty1": 1, "s_full": 1, "p_ready": 1, "dq_full": 1, "dq_free": 1,
              "dkv_full": 1, "dkv_free": 1})
    slot = {0: None, 1: None}
    errors = []
    grads_done = set()

    def producer():
        i = nu = 0
        for steps in units:
            if nu > 0: yield ("wait", "kv_empty", nu - 1)
            B.arrive("kv_full"); nu += 1
            for s in range(steps):
                st = i % 2
                if i >= 2: yield ("wait", f"qd_empty{st}", i // 2 - 1)
                if i >= 2: yield ("wait", f"row_empty{st}", i // 2 - 1)
                slot[st] = (i, s, steps); B.arrive(f"qd_full{st}"); i += 1
        st = i % 2
        if i >= 2:
            yield ("wait", f"qd_empty{st}", i // 2 - 1); yield ("wait", f"row_empty{st}", i // 2 - 1)
        slot[st] = (i, -1, -1); B.arrive(f"qd_full{st}")
        for j in range(max(0, i - 2), i): yield ("wait", f"qd_empty{j % 2}", j // 2)
        if nu > 0: yield ("wait", "kv_empty", nu - 1)

    def mma():
        st_ = {"nu": 0, "ug": 0}
        def grads(j, jst, jstep, jsteps):
            if jstep == 0 and st_["ug"] > 0: yield ("wait", "dkv_free", st_["ug"] - 1)
            if jstep == 0 and B.done["dkv_free"] < st_["ug"]: errors.append(f"dK/dV overwrite before readout j={j}")
            B.arrive(f"qd_empty{jst}")
            if j > 0: yield ("wait", "dq_free", j - 1)
            if B.done["dq_free"] < j: errors.append(f"dQ overwrite j={j}")
            grads_done.add(j)
            B.arrive("dq_full")
            if jstep == jsteps - 1:
                B.arrive("dkv_full"); B.arrive("kv_empty"); st_["ug"] += 1
        pend = None
        i = 0
        while True:
            st = i % 2
            yield ("wait", f"qd_full{st}", i // 2)
            idx, step, steps = slot[st]
            if idx != i: errors.append(f"mma read slot {idx} for {i}")
            if steps < 0: break
            if pend is not None: yield ("wait", "p_ready", pend[0])
            if order == "old_buggy" and step == 0 and pend is not None:
                yield from grads(*pend); pend = None
            if step == 0:
                if pend is not None: errors.append("pending at unit start")
                yield ("wait", "kv_full", st_["nu"]); st_["nu"] += 1
            if B.done["p_ready"] < i: errors.append(f"S/dP overwrite i={i}")
            B.arrive("s_full")
            if pend is not None: yield from grads(*pend)
            if order == "new" and step == steps - 1:
                yield ("wait", "p_ready", i); yield from grads(i, st, step, steps); pend = None
            else:
                pend = (i, st, step, steps)
            i += 1
        if pend is not None:
            yield ("wait", "p_ready", pend[0]); yield from grads(*pend)

    def compute():
        st_ = {"ug": 0}
        def finish(j, last):
            yield ("wait", "dq_full", j); B.arrive("dq_free")
            if last:
                yield ("wait", "dkv_full", st_["ug"]); B.arrive("dkv_free"); st_["ug"] += 1
        pend = None
        i = 0
        while True:
            st = i % 2
            yield ("wait", f"qd_full{st}", i // 2)
            idx, step, steps = slot[st]
            if idx != i: errors.append(f"compute read slot {idx} for {i}")
            if steps < 0: break
            B.arrive(f"row_empty{st}")
            yield ("wait", "s_full", i)
            if i >= 2 and (i - 2) not in grads_done: errors.append(f"P/dS buffer overwrite i={i}")
            B.arrive("p_ready")
            if pend is not None: yield from finish(*pend)
            pend = (i, step == steps - 1)
            i += 1
        if pend is not None: yield from finish(*pend)

    roles = {"producer": producer(), "mma": mma(), "compute": compute()}
    waiting = {r: None for r in roles}
    alive = set(roles)
    def ready(w):
        _, b, k = w
        c = B.done[b]
        if c >= k + 2: errors.append(f"parity alias on {b}: waiting phase {k}, completed {c}")
        return (c & 1) != (k & 1) and c >= k + 1
    steps_taken = 0
    while alive:
        runnable = [r for r in alive if waiting[r] is None or ready(waiting[r])]
        if not runnable:
            return False, {r: waiting[r] for r in alive}, errors
        r = rnd.choice(runnable)
        waiting[r] = None
        try:
            waiting[r] = next(roles[r])
        except StopIteration:
            alive.discard(r)
        steps_taken += 1
    return True, None, errors


def _mixes(n, seed0=0):
    for seed in range(seed0, seed0 + n):
        rnd = random.Random(seed)
        yield seed, [rnd.choice([1, 1, 2, 3, 5, 8]) for _ in range(rnd.randint(0, 6))]


def test_backward_protocol_finishes_without_hazards():
    """The kernel's order: a unit's last sub-block issues its gradients at once."""
    for seed, units in _mixes(1500):
        ok, stuck, errors = run(units, "new", seed)
        assert ok and not errors, f"units {units}: stuck {stuck}, errors {errors[:3]}"


def test_deferring_a_units_last_gradients_deadlocks():
    """The order of the development build that deadlocked at full size: the producer waits for K and
    V to be released before it loads the next unit's first Q / dO, and the MMA warp waits for that
    Q / dO before it issues the gradients that release K and V."""
    stuck_runs = sum(not run(units, "old_buggy", seed)[0] for seed, units in _mixes(300))
    assert stuck_runs > 0
    assert run([3], "old_buggy", 0)[0]  # one unit per CTA (every earlier test case) never shows it
