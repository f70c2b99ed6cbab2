"""CPU model of the persistent prefill attention kernel's barrier protocol.

``flash_prefill_kernel`` (awesome_acceleration_b200/csrc/prefill_attn_tc.cu)
runs five roles per CTA over a sequence of work items (each a pair of query
tiles A/B with nt_a <= nt_b key tiles; nt_b = 0 when the pair has no tile B):

* the TMA producer: per item, Q (after ``q_free`` of the previous item) then
  the K/V units K_0, K_1, V_0, K_2, V_1, ..., V_{nkv-1} into a 3-slot ring
  (``full`` / two-arrival ``empty``);
* one MMA issuer per tile: per item ``q_full``, then the same units in order,
  issuing S for K units (after ``s_free``) and P.V for V units (after
  ``p_full``, the item's first one also after ``o_free``), releasing every
  unit on ``empty`` (a plain arrival for units past the tile's diagonal) and
  ``q_free`` after its last S (or at once if the tile is absent);
* one softmax group per tile: ``s_full`` -> ``s_free`` -> (``pv_done`` of the
  previous step) -> ``p_full`` per key tile, then ``pv_done`` -> ``o_free``.

Every barrier's phase runs on across items.  The model executes the roles as
generators under random interleavings and asserts what the hardware needs:
no deadlock, no waiter polling a parity two phases behind (it would wait
forever), and no role arriving twice within one phase of a multi-arrival
barrier.  Barrier arrivals are immediate in the model; in the kernel an MMA
commit lands later, which only delays completions the model already orders.
"""
from __future__ import annotations

import random

import pytest

SLOTS = 3


def _units(nkv):
    out = [("K", 0)]
    for j in range(nkv - 1):
        out += [("K", j + 1), ("V", j)]
    out.append(("V", nkv - 1))
    return out


def _run(items, seed, skip_unused_release=False):
    """Run the five roles over `items` under a random interleaving; raise
    AssertionError on a protocol violation.  skip_unused_release plants a
    bug: the issuers do not release ring units past their tile's diagonal."""
    rng = random.Random(seed)
    done: dict = {}
    pend: dict = {}

    def arrive(b, count=1, who=None):
        s = pend.setdefault(b, [])
        assert who is None or who not in s, f"{who} arrived twice in one phase of {b}"
        s.append(who)
        if len(s) == count:
            pend[b] = []
            done[b] = done.get(b, 0) + 1

    def producer():
        U = nq = 0
        for nt_a, nt_b in items:
            nkv = max(nt_a, nt_b)
            if nq:
                yield ("q_free",), nq
            arrive(("q_full",))
            nq += 1
            for _ in range(2 * nkv):
                if U >= SLOTS:
                    yield ("empty", U % SLOTS), U // SLOTS
                arrive(("full", U % SLOTS))
                U += 1

    def issuer(t):
        V = nq = nsf = npf = nof = seen = 0
        for nt_a, nt_b in items:
            nkv, nt = max(nt_a, nt_b), (nt_b if t else nt_a)
            yield ("q_full",), nq + 1
            nq += 1
            if nt == 0:
                arrive(("q_free",), 2, ("issuer", t))
            for kind, j in _units(nkv):
                u = V
                V += 1
                yield ("full", u % SLOTS), u // SLOTS + 1
                if j >= nt:
                    if not skip_unused_release:
                        arrive(("empty", u % SLOTS), 2, ("issuer", t))
                    continue
                if kind == "K":
                    if j > 0 or seen:
                        yield ("s_free", t), nsf + 1
                        nsf += 1
                    arrive(("s_full", t))
                    if j == nt - 1:
                        arrive(("q_free",), 2, ("issuer", t))
                else:
                    if j == 0 and seen:
                        yield ("o_free", t), nof + 1
                        nof += 1
                    yield ("p_full", t), npf + 1
                    npf += 1
                    arrive(("pv_done", t))
                arrive(("empty", u % SLOTS), 2, ("issuer", t))
            seen += nt > 0

    def softmax(t):
        nsf = npd = 0
        for nt_a, nt_b in items:
            nt = nt_b if t else nt_a
            if nt == 0:
                continue
            for i in range(nt):
                yield ("s_full", t), nsf + 1
                nsf += 1
                arrive(("s_free", t))
                if i:
                    yield ("pv_done", t), npd + 1
                    npd += 1
                arrive(("p_full", t))
            yield ("pv_done", t), npd + 1
            npd += 1
            arrive(("o_free", t))

    roles = [producer(), issuer(0), issuer(1), softmax(0), softmax(1)]
    waits = [next(r, None) for r in roles]
    while any(w is not None for w in waits):
        ready = []
        for k, w in enumerate(waits):
            if w is None:
                continue
            bar, need = w
            assert done.get(bar, 0) <= need, f"role {k} polls {bar} two phases behind"
            if done.get(bar, 0) >= need:
                ready.append(k)
        assert ready, f"deadlock on items {items}: {waits}"
        k = rng.choice(ready)
        waits[k] = next(roles[k], None)


def _random_items(rng):
    items = []
    for _ in range(rng.randint(1, 7)):
        a = rng.randint(1, 6)
        items.append((a, 0 if rng.random() < 0.3 else rng.randint(a, a + 2)))
    return items


@pytest.mark.parametrize("seed", range(4))
def test_prefill_barrier_protocol(seed):
    rng = random.Random(seed)
    for trial in range(150):
        _run(_random_items(rng), seed * 1000 + trial)


def test_model_catches_a_planted_bug():
    """Not vacuous: issuers that skip releasing the ring units past their
    tile's diagonal (here tile A, with fewer key tiles than B) stall the
    producer, and the model reports the deadlock."""
    with pytest.raises(AssertionError, match="deadlock"):
        _run([(1, 3), (2, 4), (1, 2)], 0, skip_unused_release=True)
