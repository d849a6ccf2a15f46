"""A CPU model of the barrier protocol of the decode-regime projection kernel
(`umma_proj_kernel`, data-synth-tpu_b200/csrc/umma_proj.cuh): the weight ring filled by one
producer and drained by two decode groups that take alternate stages, and the TMEM A
buffers written by those groups and read by the MMA issuer.

mbarrier semantics as the PTX ISA states them: a phase completes when its pending arrivals
and its transaction count both reach zero; `try_wait.parity P` succeeds when the current
phase's parity differs from P. A waiter that means phase k therefore passes wrongly if the
barrier is still in phase k - 1 (the parities differ), and never passes if it is in phase
k + 2. The model flags both, flags an arrival on a phase that already has all its arrivals,
and flags a deadlock. Copies land in a random order (bulk copies complete out of order); MMA
commits complete in issue order (tcgen05.commit tracks all earlier MMAs of its thread).

The kernel's form is checked for ring sizes 2..9 with its three A buffers and with many: a
full barrier per (slot, decode group), `wfull[2 s + sc % 2]`, waited at phase
`wfull_phase(sc)`. The form with one full barrier per slot is planted here, in the model:
it is caught at ring size 3 with three A buffers, and at 5, 7 and 9 once the A buffers are
many. (With three, a group's A-buffer wait at stage sc - 2 needs the MMA of sc - 5 and so
the other group's decode of it: from five slots up that orders the slot's previous copy
before the group's next use, which is why only the three-slot rings could alias.) A second
model runs the kernel's full form: a decode warp per actor, per-half A-buffer barriers with
the kernel's arrival counts, and one, two or four MMA issuers with their own commits."""

import random

import pytest


class Alias(AssertionError):
    pass


class Bar:
    def __init__(self, name, count):
        self.name, self.count, self.pending, self.tx, self.phase = name, count, count, 0, 0

    def _complete(self):
        if self.pending == 0 and self.tx == 0:
            self.phase += 1
            self.pending = self.count

    def arrive(self):
        if self.pending == 0:
            raise Alias(f"{self.name}: arrival on phase {self.phase}, which has all its arrivals")
        self.pending -= 1
        self._complete()

    def expect_tx(self, n):
        self.tx += n
        self.arrive()

    def complete_tx(self, n):
        self.tx -= n
        assert self.tx >= 0
        self._complete()

    def passes(self, want):
        """try_wait.parity(want & 1) by a waiter that means phase `want`."""
        ok = (self.phase & 1) != (want & 1)
        if ok and self.phase <= want:
            raise Alias(f"{self.name}: a wait for phase {want} passed in phase {self.phase}")
        if not ok and self.phase >= want + 2:
            raise Alias(f"{self.name}: a wait for phase {want} would never pass (phase {self.phase})")
        return ok


def wfull_phase(sw, sc):
    """The kernel's wfull_phase<SW>: earlier stages of the same slot and decode group."""
    return sc // sw if sw % 2 == 0 else (sc // sw) >> 1


def run_model(sw, ab, stages, seed, per_group_full=True):
    rng = random.Random(seed)
    nfull = 2 * sw if per_group_full else sw
    wfull = [Bar(f"wfull[{i}]", 1) for i in range(nfull)]
    wempty = [Bar(f"wempty[{s}]", 1) for s in range(sw)]  # one arrival per decode group (its warps as one)
    afull = [Bar(f"afull[{b}]", 1) for b in range(ab)]
    aempty = [Bar(f"aempty[{b}]", 1) for b in range(ab)]
    copies, commits = [], []  # copies land in any order, commits in issue order

    def full_of(sc):
        s = sc % sw
        if per_group_full:
            return wfull[2 * s + (sc & 1)], wfull_phase(sw, sc)
        return wfull[s], sc // sw

    def producer():
        for sc in range(stages):
            s = sc % sw
            if sc >= sw:
                yield lambda b=wempty[s], k=sc // sw - 1: b.passes(k)
            bar, _ = full_of(sc)
            bar.expect_tx(2)
            copies.extend([bar, bar])  # two weight tiles, one unit each

    def decoder(g):
        for sc in range(g, stages, 2):
            s, b = sc % sw, sc % ab
            bar, k = full_of(sc)
            yield lambda bar=bar, k=k: bar.passes(k)
            wempty[s].arrive()  # codes in registers: the slot is free
            if sc >= ab:
                yield lambda bb=aempty[b], k=sc // ab - 1: bb.passes(k)
            afull[b].arrive()  # decoded into A buffer b

    def issuer():
        for sc in range(stages):
            b = sc % ab
            yield lambda bb=afull[b], k=sc // ab: bb.passes(k)
            commits.append(aempty[b])

    actors = [producer(), decoder(0), decoder(1), issuer()]
    conds = [next(a, None) for a in actors]
    while True:
        runnable = [i for i, c in enumerate(conds) if c is not None and c()]
        choices = runnable + (["copy"] if copies else []) + (["commit"] if commits else [])
        if not choices:
            if any(c is not None for c in conds):
                raise Alias("deadlock: every actor waits and nothing is in flight")
            return
        pick = rng.choice(choices)
        if pick == "copy":
            copies.pop(rng.randrange(len(copies))).complete_tx(1)
        elif pick == "commit":
            commits.pop(0).arrive()
        else:
            conds[pick] = next(actors[pick], None)


@pytest.mark.parametrize("sw", range(2, 10))
@pytest.mark.parametrize("ab", [3, 16])
def test_per_group_full_barriers_never_alias(sw, ab):
    for seed in range(40):
        run_model(sw, ab=ab, stages=64, seed=seed)


def _caught(sw, ab, seeds=200):
    n = 0
    for seed in range(seeds):
        try:
            run_model(sw, ab=ab, stages=64, seed=seed, per_group_full=False)
        except Alias:
            n += 1
    return n


@pytest.mark.parametrize("sw,ab", [(3, 3), (5, 12), (7, 16), (9, 16)])
def test_one_full_barrier_per_slot_aliases_at_odd_ring_sizes(sw, ab):
    assert _caught(sw, ab) > 0


@pytest.mark.parametrize("sw,ab", [(5, 3), (7, 3), (6, 3), (6, 16)])
def test_one_full_barrier_per_slot_holds_where_the_uses_are_ordered(sw, ab):
    # three A buffers order the stages from five slots up; an even ring gives every use of a
    # slot to one group
    assert _caught(sw, ab, seeds=60) == 0


def run_kernel_model(sw, ab, ni, stages, seed, warps_per_half=2, plant=None):
    """The kernel's full form: every decode warp its own actor (group g = sc % 2, half h of the
    block), per-half A-buffer barriers afull / aempty[2 b + h] with the kernel's counts (the
    half's warps; the commits of the ni / 2 issuers whose K atoms lie in that half, or 1),
    and ni MMA issuers, each with its own in-order commits."""
    rng = random.Random(seed)
    wfull = [Bar(f"wfull[{i}]", 1) for i in range(2 * sw)]
    wempty = [Bar(f"wempty[{s}]", 2 * warps_per_half) for s in range(sw)]
    afull_count = 2 * warps_per_half if plant == "afull_whole_group" else warps_per_half
    aempty_count = ni if plant == "aempty_all_issuers" else (ni // 2 if ni >= 2 else 1)
    afull = [Bar(f"afull[{i}]", afull_count) for i in range(2 * ab)]
    aempty = [Bar(f"aempty[{i}]", aempty_count) for i in range(2 * ab)]
    atoms = 16 // ni // 4  # 64-value K atoms per issuer
    copies, commits = [], [[] for _ in range(ni)]

    def producer():
        for sc in range(stages):
            s = sc % sw
            if sc >= sw:
                yield lambda b=wempty[s], k=sc // sw - 1: b.passes(k)
            bar = wfull[2 * s + (sc & 1)]
            bar.expect_tx(2)
            copies.extend([bar, bar])

    def decode_warp(g, h):
        for sc in range(g, stages, 2):
            s, b = sc % sw, sc % ab
            yield lambda bar=wfull[2 * s + g], k=wfull_phase(sw, sc): bar.passes(k)
            wempty[s].arrive()
            if sc >= ab:
                yield lambda bb=aempty[2 * b + h], k=sc // ab - 1: bb.passes(k)
            afull[2 * b + h].arrive()

    def issuer(mi):
        h0, h1 = (mi * atoms) // 2, (mi * atoms + atoms - 1) // 2
        for sc in range(stages):
            b = sc % ab
            yield lambda bb=afull[2 * b + h0], k=sc // ab: bb.passes(k)
            if h1 != h0:
                yield lambda bb=afull[2 * b + h1], k=sc // ab: bb.passes(k)
            commits[mi].append(aempty[2 * b + h0])
            if h1 != h0:
                commits[mi].append(aempty[2 * b + h1])

    actors = [producer()]
    actors += [decode_warp(g, h) for g in range(2) for h in range(2) for _ in range(warps_per_half)]
    actors += [issuer(mi) for mi in range(ni)]
    conds = [next(a, None) for a in actors]
    while True:
        runnable = [i for i, c in enumerate(conds) if c is not None and c()]
        choices = runnable + (["copy"] if copies else []) + [("commit", m) for m in range(ni) if commits[m]]
        if not choices:
            if any(c is not None for c in conds):
                raise Alias("deadlock: every actor waits and nothing is in flight")
            return
        pick = rng.choice(choices)
        if pick == "copy":
            copies.pop(rng.randrange(len(copies))).complete_tx(1)
        elif isinstance(pick, tuple):
            commits[pick[1]].pop(0).arrive()
        else:
            conds[pick] = next(actors[pick], None)


@pytest.mark.parametrize("ni", [1, 2, 4])
@pytest.mark.parametrize("sw", [3, 4, 5, 6, 7, 8])
def test_kernel_form_with_per_half_a_buffers_and_several_issuers(sw, ni):
    # ni = 4: the narrow gate/up pass; 2: the narrow down pass; 1: the wide form
    for seed in range(12):
        run_kernel_model(sw, ab=3, ni=ni, stages=36, seed=seed)


@pytest.mark.parametrize("plant,ni", [("afull_whole_group", 4), ("aempty_all_issuers", 4),
                                      ("aempty_all_issuers", 2)])
def test_kernel_model_catches_wrong_per_half_counts(plant, ni):
    # the counts of one barrier per whole A buffer, planted on the per-half barriers
    with pytest.raises(Alias):
        run_kernel_model(6, ab=3, ni=ni, stages=36, seed=0, plant=plant)


@pytest.mark.parametrize("sw", range(2, 10))
def test_wfull_phase_counts_the_groups_earlier_uses(sw):
    seen = {}
    for sc in range(400):
        key = (sc % sw, sc & 1)
        assert wfull_phase(sw, sc) == seen.get(key, -1) + 1
        seen[key] = wfull_phase(sw, sc)
