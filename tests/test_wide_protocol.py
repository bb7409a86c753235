"""A model of the wide-layout GEMV's barrier protocol (se12_b200/csrc/se12_gemv.cu,
gemv_kernel<..., LAYOUT = kLayoutWide>), checked on the CPU under random interleavings.

In the wide layout one CTA has a producer warp, 4 groups of 4 consumer warps
that take the pipeline stages in turn (group c the stages i with i % 4 == c),
and a reducer warp. The waits are mbarrier parity waits, and a parity wait is
exact only while the barrier is at most one phase away from the phase
waited for. A group never waits on the stage that used its slot before (that
stage belongs to another group), so before waiting for stage i it waits for
stage i - S to be consumed (the slot's empty barrier), which makes both waits
exact. The model follows the kernel's steps:

* producer: escape records one group ahead, then per stage: wait for the
  slot's empty barrier (stage i - S consumed), arm the full barrier, start
  the copy (it lands at a random later time);
* consumer warp: deposit its partials of every row before its tile (all
  warps, every row, in order: the reducer's buffer is free once row r - 2 is
  summed), settle the record groups in order, wait for stage i - S consumed,
  wait for stage i landed, release the stage and the records;
* reducer: per row, wait for all 16 deposits, sum, free the buffer.

The barriers keep arrival counts and phases and answer parity waits as the
hardware does. The test fails if a parity wait passes before its phase
completed, a barrier gets more arrivals than its count in a phase, a slot
holds another stage than the one its consumer waited for, a buffer entry is
overwritten before it was summed, or the agents deadlock. The same model
without the wait for stage i - S must fail (copies that land late), which
shows the check can see the hazard.
"""

import random

import pytest

GROUPS, STAGE_WARPS, CONSUMERS, REC_SLOTS, REC_STAGES = 4, 4, 16, 4, 4


class ProtocolError(Exception):
    pass


class Barrier:
    def __init__(self, name, count):
        self.name, self.count, self.pending, self.phase, self.tx = name, count, count, 0, 0

    def arrive(self):
        self.pending -= 1
        if self.pending < 0:
            raise ProtocolError(f"{self.name}: an arrival too many in phase {self.phase}")
        self._complete()

    def arrive_expect_tx(self):
        self.tx += 1
        self.arrive()

    def complete_tx(self):
        self.tx -= 1
        self._complete()

    def _complete(self):
        if self.pending == 0 and self.tx == 0:
            self.phase += 1
            self.pending = self.count

    def parity_passes(self, phase):
        return (self.phase & 1) != (phase & 1)


def simulate(tile_cols, rows, stages, seed, land_probability, wait_previous_stage=True):
    rng = random.Random(seed)
    tiles = rows * tile_cols
    nstages = (tiles + 3) // 4
    ngroups = (nstages + REC_STAGES - 1) // REC_STAGES
    full = [Barrier(f"full[{s}]", 1) for s in range(stages)]
    empty = [Barrier(f"empty[{s}]", STAGE_WARPS) for s in range(stages)]
    rec_full = [Barrier(f"rec_full[{r}]", 1) for r in range(REC_SLOTS)]
    rec_empty = [Barrier(f"rec_empty[{r}]", CONSUMERS) for r in range(REC_SLOTS)]
    deposited = [Barrier(f"deposited[{p}]", CONSUMERS) for p in range(2)]
    redfree = [Barrier(f"redfree[{p}]", 1) for p in range(2)]
    slot_stage, slot_group = [None] * stages, [None] * REC_SLOTS
    buffers = [dict(), dict()]
    summed = [0]
    copies = []

    def wait(barrier, phase, who):
        yield lambda: barrier.parity_passes(phase)
        if barrier.phase - 1 < phase:
            raise ProtocolError(f"{who}: wait on {barrier.name} for phase {phase} passed with {barrier.phase} complete")

    def producer():
        issued_group = 0
        for i in range(nstages):
            while issued_group <= i // REC_STAGES + 1:
                r = issued_group
                if r * REC_STAGES < nstages:
                    if r >= REC_SLOTS:
                        yield from wait(rec_empty[r % REC_SLOTS], r // REC_SLOTS - 1, "producer")
                    rec_full[r % REC_SLOTS].arrive_expect_tx()
                    copies.append(("records", r, r % REC_SLOTS))
                issued_group += 1
                yield None
            s = i % stages
            if i >= stages:
                yield from wait(empty[s], i // stages - 1, "producer")
            full[s].arrive_expect_tx()
            copies.append(("stage", i, s))
            yield None

    def deposit(warp, row):
        pb = row & 1
        yield from wait(redfree[pb], (row >> 1) - 1, f"warp {warp}")
        previous = buffers[pb].get(warp)
        if previous is not None and summed[0] <= previous:
            raise ProtocolError(f"warp {warp} overwrote row {previous} before it was summed")
        buffers[pb][warp] = row
        deposited[pb].arrive()
        yield None

    def consumer(warp):
        group, tile_in_stage = warp // 4, warp % 4
        next_row, settled = 0, 0
        for i in range(group, nstages, GROUPS):
            first = 4 * i
            have = tile_in_stage < min(4, tiles - first)
            row = (first + tile_in_stage) // tile_cols
            while have and next_row < row:
                yield from deposit(warp, next_row)
                next_row += 1
            record_group = i // REC_STAGES
            while settled <= record_group:
                yield from wait(rec_full[settled % REC_SLOTS], settled // REC_SLOTS, f"warp {warp}")
                if settled < record_group:
                    rec_empty[settled % REC_SLOTS].arrive()
                settled += 1
            if slot_group[record_group % REC_SLOTS] != record_group:
                raise ProtocolError(f"warp {warp}: record slot holds another group")
            s = i % stages
            if wait_previous_stage and i >= stages:
                yield from wait(empty[s], i // stages - 1, f"warp {warp}")
            yield from wait(full[s], i // stages, f"warp {warp}")
            if slot_stage[s] != i:
                raise ProtocolError(f"warp {warp}: slot {s} holds stage {slot_stage[s]}, waited for {i}")
            yield None
            empty[s].arrive()
            rec_empty[record_group % REC_SLOTS].arrive()
            yield None
        while next_row < rows:
            yield from deposit(warp, next_row)
            next_row += 1
        while settled < ngroups:
            yield from wait(rec_full[settled % REC_SLOTS], settled // REC_SLOTS, f"warp {warp}")
            rec_empty[settled % REC_SLOTS].arrive()
            settled += 1

    def reducer():
        for row in range(rows):
            pb = row & 1
            yield from wait(deposited[pb], row >> 1, "reducer")
            if {w for w, r in buffers[pb].items() if r == row} != set(range(CONSUMERS)):
                raise ProtocolError(f"reducer: row {row} misses deposits")
            summed[0] = row + 1
            redfree[pb].arrive()
            yield None

    agents = {"producer": producer(), "reducer": reducer()}
    agents.update({f"warp {w}": consumer(w) for w in range(CONSUMERS)})
    blocked = dict.fromkeys(agents)

    def land():
        kind, index, slot = copies.pop(rng.randrange(len(copies)))
        if kind == "stage":
            slot_stage[slot] = index
            full[slot].complete_tx()
        else:
            slot_group[slot] = index
            rec_full[slot].complete_tx()

    while agents:
        if copies and rng.random() < land_probability:
            land()
            continue
        ready = [k for k in agents if blocked[k] is None or blocked[k]()]
        if not ready:
            if not copies:
                raise ProtocolError("deadlock")
            land()
            continue
        k = rng.choice(ready)
        try:
            blocked[k] = next(agents[k])
        except StopIteration:
            del agents[k], blocked[k]


# (tile columns per row, rows in the CTA, pipeline stages): 1-tile rows,
# rows shorter and longer than a round of 16 tiles, depths 6..8
CASES = [(9, 12, 8), (1, 40, 8), (36, 3, 7), (2, 20, 6), (5, 9, 8), (18, 6, 7)]


@pytest.mark.parametrize("tile_cols,rows,stages", CASES)
@pytest.mark.parametrize("land_probability", [0.3, 0.01])
def test_wide_layout_waits_are_exact(tile_cols, rows, stages, land_probability):
    for seed in range(6):
        simulate(tile_cols, rows, stages, seed, land_probability)


def test_parity_wait_alone_can_pass_on_an_older_phase():
    failures = 0
    for tile_cols, rows, stages in CASES:
        for seed in range(6):
            try:
                simulate(tile_cols, rows, stages, seed, 0.01, wait_previous_stage=False)
            except ProtocolError:
                failures += 1
    assert failures > 0
