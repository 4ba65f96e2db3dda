"""The persistent kernel's weight ring, modelled on the host.

The producer fills ring slot g mod NS with stage g after stage g - NS was
released; consumers wait on the slot's "full" mbarrier with the parity of the
use they expect, (g / NS) & 1.  A parity wait cannot tell phases two apart, so
a consumer must never wait for a use of a slot while the use before it is
still in flight.  The layer phases consume every stage with all 8 warps in
lockstep; the narrow kernels' LM head hands stage k to one warp, k mod nw,
with nw the largest divisor of NS not above 8, so every slot is used by one
warp only.  This model runs random completion orders and interleavings for
every ring depth the engine can choose and checks that no wait is satisfied
by the wrong phase -- and that the mapping k mod 8 does break for a ring of 4
(the model catches it).

The producer runs at most LA stages ahead in the layer phases (LA <= NS) and NS
in the LM head.  Before it fills slot g mod NS it must see both stage g - LA and
stage g - NS released: after the LM head, whose warps release out of order, the
look-ahead bound alone would let it overwrite a slot that a slower warp still
reads (the model catches that too)."""
from __future__ import annotations

import random

import pytest

KCW = 8


def lm_warps(ns: int) -> int:
    nw = KCW
    while ns % nw:
        nw -= 1
    return nw


def simulate(ns: int, n_pre: int, n_lm: int, mapping, seed: int, la: int | None = None, n_post: int = 0,
             slot_wait: bool = True, self_refill: bool = False) -> str:
    """Return "ok", "alias" (a wait passed on the wrong phase), "overwrite" (a slot
    refilled before its previous stage was released) or "deadlock".  Stages
    [0, n_pre) and [n_pre + n_lm, total) are layer stages (all warps, look-ahead
    la); the n_lm in between are LM stages (one warp each, look-ahead ns)."""
    rng = random.Random(seed)
    la = ns if la is None else la
    total = n_pre + n_lm + n_post
    rel = set()  # released stages
    completed = [0] * ns  # full-barrier phases completed per slot
    released = [0] * ns   # empty-barrier phases completed per slot
    landed = set()        # stages whose copy landed
    issued = 0  # stages issued so far
    in_flight = []        # issued, not landed
    # consumer state: per warp, its stages in order and the index of the next one
    stages_of = {w: [] for w in range(KCW)}
    def is_lm(g):
        return n_pre <= g < n_pre + n_lm

    for g in range(total):
        if not is_lm(g):
            for w in range(KCW):
                stages_of[w].append(g)
        else:
            w = mapping(g - n_pre, ns)
            if w is not None:
                stages_of[w].append(g)
    pos = {w: 0 for w in range(KCW)}
    arrivals = {}  # stage -> warps that finished it (general phases need all 8)
    done_pre_all = False
    gate = False  # the producer skipped LM stages and has not yet seen the LM head finish
    steps = 0
    while True:
        steps += 1
        if steps > 200000:
            return "deadlock"
        moves = []
        # producer: issue the next stage when the look-ahead bound (and the slot's own
        # previous use, if slot_wait) was released -- parity waits on the empty barriers.
        # self_refill: LM stages from ns on are issued by the warp that read the slot
        # before; the producer only counts them and, before its next issue, waits until
        # every LM stage was released (a flag the consumers set after the LM head)
        if issued < total:
            if self_refill and is_lm(issued) and issued - n_pre >= ns:
                moves.append(("skip", None))
            elif not (gate and not all(x in rel for x in range(n_pre, n_pre + n_lm))):
                ahead = ns if is_lm(issued) else la
                waits = [issued - ahead] if issued >= ahead else []
                if slot_wait and issued >= ns:
                    waits.append(issued - ns)
                ok = True
                for j in waits:
                    slot, use = j % ns, j // ns
                    if (released[slot] & 1) != (use & 1):  # try_wait.parity passes
                        if released[slot] != use + 1:
                            return "alias"
                    else:
                        ok = False
                if ok:
                    moves.append(("issue", None))
        if in_flight:
            moves.append(("land", None))
        for w in range(KCW):
            if pos[w] < len(stages_of[w]):
                g = stages_of[w][pos[w]]
                if g >= n_pre and not done_pre_all:
                    continue  # the LM phase starts after a CTA barrier
                if g >= n_pre + n_lm and not all(x in rel for x in range(n_pre, n_pre + n_lm)):
                    continue  # and ends with one
                slot, use = g % ns, g // ns
                if (completed[slot] & 1) != (use & 1):  # try_wait.parity(use & 1) passes
                    moves.append(("consume", w))
        if not moves:
            if all(pos[w] >= len(stages_of[w]) for w in range(KCW)) and issued == total:
                return "ok"
            return "deadlock"
        kind, w = rng.choice(moves)
        if kind == "skip":
            issued += 1
            gate = True
        elif kind == "issue":
            if issued >= ns and (issued - ns) not in rel:
                return "overwrite"
            in_flight.append(issued)
            issued += 1
            gate = False
        elif kind == "land":
            g = in_flight.pop(rng.randrange(len(in_flight)))  # copies may complete out of order
            landed.add(g)
            # a slot's phase completes when its pending copy lands (uses complete in order per slot)
            slot = g % ns
            while (completed[slot] * ns + slot) in landed:
                completed[slot] += 1
        else:
            g = stages_of[w][pos[w]]
            slot, use = g % ns, g // ns
            if completed[slot] != use + 1:
                return "alias"
            pos[w] += 1
            if not is_lm(g):
                arrivals.setdefault(g, set()).add(w)
                if len(arrivals[g]) == KCW:
                    released[slot] += 1
                    rel.add(g)
            else:
                if self_refill and is_lm(g + ns):
                    in_flight.append(g + ns)  # the warp refills its slot before releasing it
                released[slot] += 1  # one warp arrives with the count of 8
                rel.add(g)
            if not done_pre_all and all(pos[x] >= sum(1 for s in stages_of[x] if s < n_pre) for x in range(KCW)):
                done_pre_all = True


@pytest.mark.parametrize("ns", list(range(2, 25)))
def test_lm_stage_per_warp_mapping_never_aliases(ns):
    nw = lm_warps(ns)
    for seed in range(20):
        r = simulate(ns, n_pre=3 * ns + 1, n_lm=22, mapping=lambda k, n: k % nw, seed=seed)
        assert r == "ok", (ns, seed, r)


def test_model_catches_the_eight_warp_mapping_on_a_ring_of_four():
    results = {simulate(4, n_pre=9, n_lm=22, mapping=lambda k, n: k % KCW, seed=s) for s in range(50)}
    assert "alias" in results


@pytest.mark.parametrize("self_refill", [False, True])
@pytest.mark.parametrize("ns,la", [(7, 4), (14, 8), (8, 8), (6, 4), (24, 4)])
def test_producer_waits_for_the_slot_and_the_look_ahead(ns, la, self_refill):
    """Also with the LM head's warps refilling their own slots from stage NS on."""
    nw = lm_warps(ns)
    for seed in range(30):
        r = simulate(ns, n_pre=2 * ns + 3, n_lm=22, mapping=lambda k, n: k % nw, seed=seed, la=la,
                     n_post=2 * ns, self_refill=self_refill)
        assert r == "ok", (ns, la, seed, r)


def test_model_catches_a_producer_that_tracks_self_refilled_stages_by_parity():
    """The first self-refill design: the producer waited on the empty barrier for each
    self-refilled stage's predecessor; the warps can advance a slot two phases past it."""
    nw = lm_warps(7)

    def run(seed):
        return simulate_parity_tracking_producer(7, 17, 22, nw, seed)
    assert "alias" in {run(s) for s in range(300)}


def simulate_parity_tracking_producer(ns, n_pre, n_lm, nw, seed):
    """Self-refilling warps, and a producer that waits (by parity) for the release of
    stage g - ns before counting each self-refilled stage g."""
    rng = random.Random(seed)
    released = [0] * ns
    consumed = {w: 0 for w in range(nw)}  # LM stages consumed per warp
    lm_stages = {w: [k for k in range(n_lm) if k % nw == w] for w in range(nw)}
    g = ns  # next self-refilled LM stage the producer counts
    for _ in range(10000):
        moves = [w for w in range(nw) if consumed[w] < len(lm_stages[w])]
        if g < n_lm:
            moves.append(-1)
        if not moves:
            return "ok"
        m = rng.choice(moves)
        if m == -1:
            j = n_pre + g - ns
            slot, use = j % ns, j // ns
            if (released[slot] & 1) != (use & 1):
                if released[slot] != use + 1:
                    return "alias"
                g += 1
        else:
            k = lm_stages[m][consumed[m]]
            released[(n_pre + k) % ns] += 1  # consumed, refilled, released
            consumed[m] += 1
    return "ok"


def test_model_catches_a_producer_that_only_waits_for_the_look_ahead():
    nw = lm_warps(7)
    results = {simulate(7, n_pre=17, n_lm=22, mapping=lambda k, n: k % nw, seed=s, la=4, n_post=14,
                        slot_wait=False) for s in range(200)}
    assert "overwrite" in results
