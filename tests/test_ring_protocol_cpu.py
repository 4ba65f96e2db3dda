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
(the model catches it)."""
from __future__ import annotations

import random

import pytest

KCW = 8


def lm_warps(ns: int) -> int:
    nw = KCW
    while ns % nw:
        nw -= 1
    return nw


def simulate(ns: int, n_pre: int, n_lm: int, mapping, seed: int) -> str:
    """Return "ok", "alias" (a wait passed on the wrong phase) or "deadlock"."""
    rng = random.Random(seed)
    total = n_pre + n_lm
    completed = [0] * ns  # full-barrier phases completed per slot
    released = [0] * ns   # empty-barrier phases completed per slot
    landed = set()        # stages whose copy landed
    issued = 0  # stages issued so far
    in_flight = []        # issued, not landed
    # consumer state: per warp, its stages in order and the index of the next one
    stages_of = {w: [] for w in range(KCW)}
    for g in range(total):
        if g < n_pre:
            for w in range(KCW):
                stages_of[w].append(g)
        else:
            w = mapping(g - n_pre, ns)
            if w is not None:
                stages_of[w].append(g)
    pos = {w: 0 for w in range(KCW)}
    arrivals = {}  # stage -> warps that finished it (general phases need all 8)
    done_pre_all = False
    steps = 0
    while True:
        steps += 1
        if steps > 200000:
            return "deadlock"
        moves = []
        # producer: issue the next stage when stage issued - ns was released
        if issued < total and (issued < ns or released[issued % ns] >= issued // ns):
            moves.append(("issue", None))
        if in_flight:
            moves.append(("land", None))
        for w in range(KCW):
            if pos[w] < len(stages_of[w]):
                g = stages_of[w][pos[w]]
                if g >= n_pre and not done_pre_all:
                    continue  # the LM phase starts after a CTA barrier
                slot, use = g % ns, g // ns
                if (completed[slot] & 1) != (use & 1):  # try_wait.parity(use & 1) passes
                    moves.append(("consume", w))
        if not moves:
            if all(pos[w] >= len(stages_of[w]) for w in range(KCW)) and issued == total:
                return "ok"
            return "deadlock"
        kind, w = rng.choice(moves)
        if kind == "issue":
            in_flight.append(issued)
            issued += 1
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
            if g < n_pre:
                arrivals.setdefault(g, set()).add(w)
                if len(arrivals[g]) == KCW:
                    released[slot] += 1
            else:
                released[slot] += 1  # one warp arrives with the count of 8
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
