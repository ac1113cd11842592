"""CPU model of the barrier protocol of the forward kernel (packed_encoders_b200/csrc/attn_fwd.cu,
attn_fwd_kernel): the TMA producer, the MMA issuer and the softmax warps of one CTA as coroutines
over mbarrier phase counts, run in random interleavings, for every layout the library launches
(key-ring and V-ring depths, Q buffers, S buffers with P.V one or two tiles behind QK, Q in TMEM).

Each role yields ('wait', barrier, k): phase k must have completed, with the parity semantics of
mbarrier.try_wait.parity (a waiter two phases behind is reported as parity aliasing). Commits and
TMA completions are modelled as immediate arrivals: the tensor pipe and the copy engine wait on
nothing but work already issued, so they always finish. The model checks that every role finishes
and that no buffer is overwritten before its reader is done: an S buffer before the P.V that reads
its P was issued (issue order is execution order on the tensor pipe), the O accumulator before the
previous unit's epilogue read it. The roles follow the kernel's loops; a change to the kernel's
barrier protocol must be mirrored here.
"""

import random

import pytest


class Bars:
    def __init__(self):
        self.count, self.arr, self.done = {}, {}, {}

    def add(self, name, count=1):
        self.count[name], self.arr[name], self.done[name] = count, 0, 0

    def arrive(self, name):
        self.arr[name] += 1
        if self.arr[name] == self.count[name]:
            self.arr[name] = 0
            self.done[name] += 1


def run(units, *, ST, VST, QB, NS, qtm, seed=0, rescale_p=0.1, mutation=None):
    """units: key-tile counts of the CTA's units (all > 0, as the producer skips empty units).
    mutation: a deliberate protocol change used to check that the model catches it."""
    rnd = random.Random(seed)
    lag = 2 if NS >= 3 else 1
    B = Bars()
    for j in range(ST):
        B.add(f"k_full{j}"); B.add(f"k_empty{j}")
    for j in range(VST):
        B.add(f"v_full{j}"); B.add(f"v_empty{j}")
    for j in range(QB):
        B.add(f"q_full{j}"); B.add(f"q_empty{j}"); B.add(f"row_empty{j}")
    for j in range(NS):
        B.add(f"s_full{j}"); B.add(f"p_full{j}")
    B.add("o_full")
    slot = {}
    errors = []
    pv_issued = set()
    epilogues_done = set()
    unit_of_tile = {}

    def producer():
        i = lu = 0
        v_pending = None

        def issue_v(j):
            st = j % VST
            if j >= VST:
                yield ("wait", f"v_empty{st}", j // VST - 1)
            B.arrive(f"v_full{st}")

        for n_kv in units:
            qb = lu % QB
            if lu >= QB:
                yield ("wait", f"q_empty{qb}", lu // QB - 1)
            if lu >= QB:
                yield ("wait", f"row_empty{qb}", lu // QB - 1)
            slot[qb] = (lu, n_kv)
            B.arrive(f"q_full{qb}")
            for t in range(n_kv):
                st = i % ST
                if i >= ST:
                    yield ("wait", f"k_empty{st}", i // ST - 1)
                unit_of_tile[i] = lu
                B.arrive(f"k_full{st}")
                if v_pending is not None:
                    yield from issue_v(v_pending)
                v_pending = i
                i += 1
            lu += 1
        if v_pending is not None:
            yield from issue_v(v_pending)
        qb = lu % QB
        if lu >= QB:
            yield ("wait", f"q_empty{qb}", lu // QB - 1)
            yield ("wait", f"row_empty{qb}", lu // QB - 1)
        slot[qb] = (lu, -1)
        B.arrive(f"q_full{qb}")
        for j in range(max(0, i - ST), i):
            yield ("wait", f"k_empty{j % ST}", j // ST)

    def mma():
        i = 0
        pend = []  # (tile, first, last)

        def issue_pv(j, first, last):
            yield ("wait", f"p_full{j % NS}", j // NS)
            yield ("wait", f"v_full{j % VST}", j // VST)
            if first and unit_of_tile[j] > 0 and unit_of_tile[j] - 1 not in epilogues_done:
                errors.append(f"O overwritten before unit {unit_of_tile[j] - 1}'s epilogue")
            pv_issued.add(j)
            if last:
                B.arrive("o_full")
            B.arrive(f"v_empty{j % VST}")

        lu = 0
        while True:
            qb = lu % QB
            while pend:
                yield from issue_pv(*pend.pop(0))
            yield ("wait", f"q_full{qb}", lu // QB)
            u, n_kv = slot[qb]
            if u != lu:
                errors.append(f"mma read slot of unit {u} for {lu}")
            if n_kv < 0:
                break
            if qtm:
                B.arrive(f"q_empty{qb}")
            for t in range(n_kv):
                if NS == 1 and mutation != "ns1_no_flush":
                    while pend:
                        yield from issue_pv(*pend.pop(0))
                yield ("wait", f"k_full{i % ST}", i // ST)
                if i >= NS and i - NS not in pv_issued:
                    errors.append(f"S buffer of tile {i} overwritten before the P.V of tile {i - NS}")
                B.arrive(f"s_full{i % NS}")
                B.arrive(f"k_empty{i % ST}")
                if not qtm and t == n_kv - 1:
                    B.arrive(f"q_empty{qb}")
                pend.append((i, t == 0, t == n_kv - 1))
                if len(pend) > lag:
                    yield from issue_pv(*pend.pop(0))
                i += 1
            lu += 1
        while pend:
            yield from issue_pv(*pend.pop(0))

    def softmax():
        i = 0

        def read_header(u):
            qb = u % QB
            yield ("wait", f"q_full{qb}", u // QB)
            uu, n_kv = slot[qb]
            if uu != u:
                errors.append(f"softmax read slot of unit {uu} for {u}")
            if n_kv >= 0:
                B.arrive(f"row_empty{qb}")
            return n_kv

        n_kv = yield from read_header(0)
        lu = 0
        while n_kv >= 0:
            for t in range(n_kv):
                yield ("wait", f"s_full{i % NS}", i // NS)
                if t > 0 and rnd.random() < rescale_p:  # O rescale: the previous P.V must have landed
                    yield ("wait", f"v_empty{(i - 1) % VST}", (i - 1) // VST)
                B.arrive(f"p_full{i % NS}")
                i += 1
            next_n = yield from read_header(lu + 1)
            yield ("wait", "o_full", lu)
            epilogues_done.add(lu)
            n_kv = next_n
            lu += 1

    roles = {"producer": producer(), "mma": mma(), "softmax": softmax()}
    waiting = {r: None for r in roles}
    alive = set(roles)

    def ready(w):
        _, b, k = w
        c = B.done[b]
        if c >= k + 2:
            errors.append(f"parity alias on {b}: waiting phase {k}, completed {c}")
        return (c & 1) != (k & 1) and c >= k + 1

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
    return True, None, errors


# The layouts launch_attention uses: (ST, VST, QB, NS, Q in TMEM).
LAYOUTS = {
    "d64-global": (4, 3, 2, 2, True),
    "d64-windowed": (4, 3, 2, 3, False),
    "d64-short-batches": (4, 3, 2, 3, False),
    "d128": (2, 2, 2, 2, False),
    "d256": (3, 2, 1, 2, True),
}


@pytest.mark.parametrize("layout", sorted(LAYOUTS))
def test_forward_protocol_finishes_without_hazards(layout):
    ST, VST, QB, NS, qtm = LAYOUTS[layout]
    for seed in range(600):
        rnd = random.Random(seed)
        units = [rnd.choice([1, 1, 2, 3, 4, 9]) for _ in range(rnd.randint(0, 7))]
        ok, stuck, errors = run(units, ST=ST, VST=VST, QB=QB, NS=NS, qtm=qtm, seed=seed)
        assert ok and not errors, f"{layout} units {units}: stuck {stuck}, errors {errors[:3]}"


def test_model_catches_an_s_buffer_overwrite():
    """With one S buffer the kernel issues the pending P.V before the next QK; a protocol without
    that flush overwrites S before its P was read, and the model reports it."""
    ok, _, errors = run([3, 2], ST=4, VST=3, QB=2, NS=1, qtm=False, seed=1)
    assert ok and not errors
    ok, _, errors = run([3, 2], ST=4, VST=3, QB=2, NS=1, qtm=False, seed=1, mutation="ns1_no_flush")
    assert any("overwritten before the P.V" in e for e in errors)
