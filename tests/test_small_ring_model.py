"""CPU model of the small-width expert kernel's ring protocol
(k_experts_small in firewing_b200/csrc/fw_experts.cu).

One CTA: a producer issues the CTA's stages in steps of 8 (one lane per
stage, each lane waiting on its own ring slot's "empty" barrier); copies
land in any order; 7 consumer warps take the units round-robin and wait on
"full" barriers indexed by stage mod NF by mbarrier parity; a down unit
also waits until every up unit of its slot is consumed.  Random
interleavings (up units published per warp and slot, as the kernel batches
them) check the claims the kernel's comments make:
  - whenever a parity wait passes, the stage it names has landed (no phase
    aliasing), with NF = 128 >= R + 64;
  - a barrier is re-armed only after its previous use completed, and ring
    slots are consumed in issue order;
  - the protocol never deadlocks while R exceeds a unit's stage count.
Indexing the full barriers by ring slot (NF = R) aliases.
"""
import numpy as np
import pytest

WARPS, LANES = 7, 8


class Aliased(AssertionError):
    pass


def build_passes(rng, max_nch_up=8):
    """Passes (phase, slot, n_units, nch) in the kernel's order: every up
    pass, then every down pass (one pass per slot at small widths)."""
    slots = int(rng.integers(1, 4))
    nch_up = int(rng.integers(1, max_nch_up + 1))
    nch_dn = int(rng.integers(1, 3))
    up = [(0, s, int(rng.integers(1, 8)), nch_up) for s in range(slots)]
    dn = [(1, s, int(rng.integers(1, 12)), nch_dn) for s in range(slots)]
    return up + dn


def simulate(passes, R, NF, seed):
    rng = np.random.default_rng(seed)
    units = []  # (phase, slot, first stage, nch)
    g = 0
    for phase, slot, n, nch in passes:
        for _ in range(n):
            units.append((phase, slot, g, nch))
            g += nch
    total = g
    steps = []  # producer steps: consecutive stages of one pass, at most 8
    g = 0
    for phase, slot, n, nch in passes:
        stages = n * nch
        for o in range(0, stages, LANES):
            steps.append(list(range(g + o, g + min(o + LANES, stages))))
        g += stages
    assert max(u[3] for u in units) < R, "the kernel requires R > a unit's stages"

    full = np.zeros(NF, dtype=np.int64)   # completed phases per full barrier
    empty = np.zeros(R, dtype=np.int64)   # completed phases per empty barrier
    issued = np.zeros(total, dtype=bool)
    landed = np.zeros(total, dtype=bool)
    consumed = np.zeros(total, dtype=bool)
    in_flight = []
    step = 0
    up_left = {}
    for phase, slot, _, _ in units:
        if phase == 0:
            up_left[slot] = up_left.get(slot, 0) + 1
    mine = [[u for u in range(len(units)) if u % WARPS == w] for w in range(WARPS)]
    pos = [0] * WARPS     # unit index into mine[w]
    chunk = [0] * WARPS   # stage within the unit
    pend = [None] * WARPS  # [slot, n]: up units done but not yet published

    def flush(w):
        if pend[w] is not None:
            up_left[pend[w][0]] -= pend[w][1]
            pend[w] = None

    def try_wait(count, parity):  # mbarrier.try_wait.parity
        return (count & 1) != parity

    while not consumed.all():
        actions = []
        if step < len(steps):
            for gs in steps[step]:
                if not issued[gs] and (gs < R or try_wait(empty[gs % R], ((gs // R) - 1) & 1)):
                    actions.append(("issue", gs))
        for gs in in_flight:
            actions.append(("land", gs))
        for w in range(WARPS):
            if pos[w] >= len(mine[w]):
                continue
            phase, slot, first, nch = units[mine[w][pos[w]]]
            if phase == 1 and chunk[w] == 0 and up_left[slot] > 0:
                continue  # the down unit's wait on up_done
            gs = first + chunk[w]
            if try_wait(full[gs % NF], (gs // NF) & 1):
                actions.append(("consume", w))
        if not actions:
            raise AssertionError(f"deadlock: step {step}/{len(steps)}, consumed {consumed.sum()}/{total}")
        kind, arg = actions[int(rng.integers(len(actions)))]
        if kind == "issue":
            gs = arg
            if gs >= R:
                # the slot's previous use (gs - R) was consumed, its next is not
                assert empty[gs % R] == gs // R, (gs, empty[gs % R])
            # arrive.expect_tx re-arms the full barrier: its previous use landed
            assert full[gs % NF] == gs // NF, ("re-armed before the previous use landed", gs)
            issued[gs] = True
            in_flight.append(gs)
            if all(issued[s] for s in steps[step]):
                step += 1
        elif kind == "land":
            gs = arg
            in_flight.remove(gs)
            assert full[gs % NF] == gs // NF
            full[gs % NF] += 1
            landed[gs] = True
        else:
            w = arg
            u = mine[w][pos[w]]
            phase, slot, first, nch = units[u]
            gs = first + chunk[w]
            if not landed[gs]:
                raise Aliased(f"warp {w} passed the wait for stage {gs} before it landed")
            assert empty[gs % R] == gs // R, "ring slots are consumed in issue order"
            empty[gs % R] += 1
            consumed[gs] = True
            chunk[w] += 1
            if chunk[w] == nch:
                chunk[w] = 0
                pos[w] += 1
                if phase == 0:
                    # published when the warp moves to another slot or leaves
                    # the up phase (before any down wait)
                    if pend[w] is not None and pend[w][0] != slot:
                        flush(w)
                    if pend[w] is None:
                        pend[w] = [slot, 0]
                    pend[w][1] += 1
                    nxt = units[mine[w][pos[w]]] if pos[w] < len(mine[w]) else None
                    if nxt is None or nxt[0] == 1:
                        flush(w)
    return total


@pytest.mark.parametrize("R", [12, 16, 21, 25, 32])
def test_full_barriers_by_stage_mod_128_never_alias(R):
    rng = np.random.default_rng(R)
    for trial in range(40):
        passes = build_passes(rng, max_nch_up=min(8, R - 1))
        simulate(passes, R, 128, seed=1000 * R + trial)


def test_slot_indexed_full_barriers_alias():
    # Full barriers indexed by ring slot alias: a warp that reaches stage g
    # before the slot's previous use (g - R, another warp's) has landed
    # passes the parity test on the old phase.
    rng = np.random.default_rng(7)
    hits = 0
    for trial in range(60):
        passes = [(0, 0, 14, 4), (0, 1, 14, 4), (1, 0, 20, 1), (1, 1, 20, 1)]
        try:
            simulate(passes, 16, 16, seed=trial + int(rng.integers(1 << 20)))
        except Aliased:
            hits += 1
    assert hits > 0
