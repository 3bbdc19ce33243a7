"""CPU simulation of the pair kernel's barrier protocol.

The GEMM kernel (blackwell_gemm_b200/csrc/gemm_kernel.cuh, gemm_bf16_pair_kernel)
coordinates its warps only through mbarriers waited on by phase parity.  This
test replays that protocol step for step on the CPU, under random schedules,
and checks what the data path relies on:

* a ring slot of either CTA is written by TMA only after the tensor pipe has
  read the slot's previous contents;
* the tensor pipe reads every (unit, K block) stage in production order, with
  the data of both CTAs present;
* an accumulator buffer is read by the epilogue only once it holds the whole
  tile, and the MMA writes a buffer only after every epilogue warp of the pair
  released it;
* no schedule deadlocks.

Modelled as in the kernel (line numbers of gemm_kernel.cuh):
  full[s]      in the leader, 2 arrivals (one arrive.expect_tx per CTA) plus
               the transaction bytes of both CTAs' TMA loads (503, 565-572)
  empty[s]     one per CTA, 1 arrival: tcgen05.commit in the leader; the
               leader's producer forwards each completion to the peer's
               empty[s] once it has passed its own wait on that slot (504,
               553-560, 628)
  acc_full[b]  one per CTA, 1 arrival: tcgen05.commit to both CTAs (507, 633-634)
  acc_empty[b] in the leader, 2 x epilogue-warps arrivals (508, 726/802/879)
  waits        empty with parity phase ^ 1, full with parity phase,
               acc_empty with acc_phase ^ 1, acc_full with acc_phase,
               buf = it % bufs, acc_phase = (it / bufs) & 1 (553, 597-606, 661-668)
tcgen05.mma and tcgen05.commit are asynchronous and complete in issue order
(one in-order tensor-pipe queue); TMA loads complete in any order.
Planted mistakes (a wrong parity, a slot handed on a lap early, an
accumulator released before it is read) must make the simulation fail: that
shows the checks can see a broken protocol.
"""
from __future__ import annotations

import random

import pytest


class Barrier:
    """mbarrier: a phase completes when its arrivals and transaction bytes are
    all in; try_wait(parity) is true once the phase of that parity completed
    (i.e. the current phase's parity differs)."""

    def __init__(self, count: int):
        self.count = count
        self.pending = count
        self.tx = 0
        self.phase = 0

    def _maybe_complete(self):
        if self.pending == 0 and self.tx == 0:
            self.phase += 1
            self.pending = self.count

    def arrive(self, expect_tx: int = 0):
        assert self.pending > 0, "arrival beyond the barrier's count"
        self.tx += expect_tx
        self.pending -= 1
        self._maybe_complete()

    def complete_tx(self, nbytes: int):
        self.tx -= nbytes
        self._maybe_complete()

    def try_wait(self, parity: int) -> bool:
        return (self.phase & 1) != parity


class Sim:
    def __init__(self, units, k_blocks, stages, bufs, epi_warps, rng, plant=None):
        self.units, self.kb, self.S, self.bufs, self.E = units, k_blocks, stages, bufs, epi_warps
        self.rng, self.plant = rng, plant
        self.full = [Barrier(2) for _ in range(stages)]                  # leader's
        self.empty = [[Barrier(1) for _ in range(stages)] for _ in range(2)]
        self.acc_full = [[Barrier(1) for _ in range(bufs)] for _ in range(2)]
        self.acc_empty = [Barrier(2 * epi_warps) for _ in range(bufs)]   # leader's
        # slot contents per CTA: (unit, kb) or None; consumed flags
        self.slot = [[None] * stages for _ in range(2)]
        self.consumed = [[True] * stages for _ in range(2)]
        # accumulator per buffer: (unit, K blocks accumulated); readers
        self.acc = [[None, 0] for _ in range(bufs)]
        self.acc_readers = [0] * bufs
        self.tma_queue = []      # pending loads: (cta, stage, unit, kb)
        self.pipe = []           # in-order tensor pipe ops
        self.next_read = 0       # expected global stage sequence number
        self.epi_done = []

    # ---------------------------------------------------------------- roles
    def producer(self, r):
        stage, phase, filled = 0, 0, 0
        for u in range(self.units):
            for kb in range(self.kb):
                want = phase ^ 1
                if self.plant == "producer_parity" and r == 1:
                    want = phase
                yield lambda s=stage, w=want: self.empty[r][s].try_wait(w)
                first_lap = self.S - 1 if self.plant == "early_forward" else self.S
                if r == 0 and filled >= first_lap:
                    self.empty[1][stage].arrive()          # forward to the peer
                filled += 1
                self.full[stage].arrive(expect_tx=1)       # this CTA's bytes (1 unit)
                self.tma_queue.append((r, stage, u, kb))
                stage += 1
                if stage == self.S:
                    stage, phase = 0, phase ^ 1

    def mma(self):
        stage, phase = 0, 0
        seq = 0
        for it in range(self.units):
            buf, acc_phase = it % self.bufs, (it // self.bufs) & 1
            want = acc_phase ^ 1
            if self.plant == "acc_parity":
                want = acc_phase
            yield lambda b=buf, w=want: self.acc_empty[b].try_wait(w)
            for kb in range(self.kb):
                yield lambda s=stage, p=phase: self.full[s].try_wait(p)
                self.pipe.append(("mma", stage, it, kb, buf, seq))
                seq += 1
                self.pipe.append(("commit", self.empty[0][stage]))
                stage += 1
                if stage == self.S:
                    stage, phase = 0, phase ^ 1
            self.pipe.append(("commit", self.acc_full[0][buf]))
            self.pipe.append(("commit", self.acc_full[1][buf]))

    def epilogue(self, r, w):
        for it in range(self.units):
            buf, acc_phase = it % self.bufs, (it // self.bufs) & 1
            yield lambda b=buf, p=acc_phase: self.acc_full[r][b].try_wait(p)
            if self.plant == "early_release":
                self.acc_empty[buf].arrive()               # released before the drain
                yield None
            unit, n = self.acc[buf]
            assert unit == it and n == self.kb, \
                f"epilogue read buffer {buf} holding {self.acc[buf]}, expected unit {it} complete"
            self.acc_readers[buf] += 1
            yield None                                     # drain takes a step
            self.acc_readers[buf] -= 1
            if self.plant != "early_release":
                self.acc_empty[buf].arrive()
        self.epi_done.append((r, w))

    # ------------------------------------------------------ asynchronous units
    def tma_step(self):
        i = self.rng.randrange(len(self.tma_queue))
        r, s, u, kb = self.tma_queue.pop(i)
        assert self.consumed[r][s], f"TMA overwrote CTA {r} slot {s} before the MMA read it"
        self.slot[r][s] = (u, kb)
        self.consumed[r][s] = False
        self.full[s].complete_tx(1)

    def pipe_step(self):
        op = self.pipe.pop(0)
        if op[0] == "commit":
            op[1].arrive()
            return
        _, s, it, kb, buf, seq = op
        assert seq == self.next_read
        self.next_read += 1
        for r in range(2):
            assert self.slot[r][s] == (it, kb) and not self.consumed[r][s], \
                f"MMA read CTA {r} slot {s} = {self.slot[r][s]}, expected {(it, kb)}"
            self.consumed[r][s] = True
        assert self.acc_readers[buf] == 0, "MMA wrote an accumulator the epilogue is reading"
        if kb == 0:
            self.acc[buf] = [it, 1]
        else:
            assert self.acc[buf][0] == it
            self.acc[buf][1] += 1

    # ------------------------------------------------------------ scheduler
    def run(self):
        actors = [self.producer(0), self.producer(1), self.mma()]
        actors += [self.epilogue(r, w) for r in range(2) for w in range(self.E)]
        waits = [None] * len(actors)
        live = list(range(len(actors)))
        steps = 0
        # Random speed per role and per asynchronous unit: some schedules starve
        # one of them for long stretches, which opens the windows a race needs.
        speeds = [0.02, 0.2, 1.0, 1.0, 5.0]
        w_actor = [self.rng.choice(speeds) for _ in actors]
        w_tma, w_pipe = self.rng.choice(speeds), self.rng.choice(speeds)
        while live or self.tma_queue or self.pipe:
            steps += 1
            assert steps < 10_000_000
            ready = [i for i in live if waits[i] is None or waits[i]()]
            choices = [("actor", i) for i in ready]
            weights = [w_actor[i] for i in ready]
            if self.tma_queue:
                choices.append(("tma", None))
                weights.append(w_tma)
            if self.pipe:
                choices.append(("pipe", None))
                weights.append(w_pipe)
            if not choices:
                raise RuntimeError("deadlock: every role waits and nothing is in flight")
            kind, i = self.rng.choices(choices, weights)[0]
            if kind == "tma":
                self.tma_step()
            elif kind == "pipe":
                self.pipe_step()
            else:
                try:
                    waits[i] = next(actors[i])
                except StopIteration:
                    live.remove(i)
        assert len(self.epi_done) == 2 * self.E
        assert self.next_read == self.units * self.kb


@pytest.mark.parametrize("bufs,epi_warps", [(2, 4), (1, 8)])   # 256-wide / 512-wide tiles
@pytest.mark.parametrize("stages", [2, 4, 6])
def test_protocol_holds_under_random_schedules(bufs, epi_warps, stages):
    for seed in range(100):
        rng = random.Random(seed * 1000 + stages * 10 + bufs)
        units = rng.randint(1, 6)
        k_blocks = rng.randint(1, 9)
        Sim(units, k_blocks, stages, bufs, epi_warps, rng).run()


@pytest.mark.parametrize("plant,failure", [
    ("producer_parity", RuntimeError),   # peer producer waits on the wrong parity: deadlock
    ("acc_parity", RuntimeError),        # MMA waits on the wrong accumulator parity: deadlock
    ("early_forward", AssertionError),   # slot handed to the peer a lap early: overwrite
    ("early_release", AssertionError),   # accumulator released before the drain: race
])
def test_planted_protocol_mistake_is_caught(plant, failure):
    """Every seed may fail either way (a skewed phase can also end in a
    deadlock); the expected kind of failure must show up in some of them."""
    kinds = []
    for seed in range(200):
        rng = random.Random(seed)
        try:
            Sim(4, 7, 3, 2, 4, rng, plant=plant).run()
        except (AssertionError, RuntimeError) as e:
            kinds.append(type(e))
    assert failure in kinds, f"planted mistake {plant} went unnoticed ({len(kinds)} other failures)"
