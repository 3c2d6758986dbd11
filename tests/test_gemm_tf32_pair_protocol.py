"""The barrier protocol of the CTA-pair 3xTF32 GEMM (gemm_tf32.cu,
gemm_tf32_kernel<true>), modelled on the CPU: in each CTA of the pair a TMA
producer, the split warps and the epilogue; in the leader the MMA thread,
whose MMAs read both CTAs' stages and write both CTAs' accumulators, and
whose commits arrive on a barrier in both CTAs (multicast). Barriers follow
the hardware's phase and parity semantics (try_wait.parity(p) succeeds once
the phase of parity p has completed); stages and accumulators are walked as
the kernel walks them (stage and phase, acc and acc_phase). Under random
schedules no role may wait forever, every MMA must read the stage's hi and
lo halves of its own k-block, and every epilogue must read a whole tile."""
import random

import pytest

STAGES = 3


class Bar:
    def __init__(self, n):
        self.n, self.pend, self.phase = n, n, 0

    def arrive(self):
        self.pend -= 1
        if self.pend == 0:
            self.phase += 1
            self.pend = self.n

    def done(self, parity):
        return (self.phase & 1) != parity


def simulate(tiles, kblocks, seed):
    rng = random.Random(seed)
    cta = (0, 1)
    bars = {}
    for c in cta:
        for s in range(STAGES):
            bars[("full", c, s)] = Bar(1)
            bars[("empty", c, s)] = Bar(1)
        for a in range(2):
            bars[("tfull", c, a)] = Bar(1)
    for s in range(STAGES):
        bars[("split", 0, s)] = Bar(2)  # one arrival a CTA, on the leader's barrier
    for a in range(2):
        bars[("tempty", 0, a)] = Bar(2)  # every epilogue of the pair (one group a CTA here)
    hi = {(c, s): None for c in cta for s in range(STAGES)}
    lo = dict(hi)
    acc = {(c, a): None for c in cta for a in range(2)}
    fifo, tma = [], []

    def tensor(op):
        if op[0] == "mma":
            t, kb, s, a = op[1:]
            for c in cta:
                assert hi[(c, s)] == (t, kb) and lo[(c, s)] == (t, kb), ("MMA operands", t, kb, c)
                if kb == 0:
                    acc[(c, a)] = [t, 1]
                else:
                    assert acc[(c, a)] == [t, kb], ("accumulates", t, kb)
                    acc[(c, a)][1] += 1
        else:
            for c in cta:  # tcgen05.commit ... multicast::cluster to both CTAs
                bars[(op[1], c, op[2])].arrive()

    def producer(c):
        stage = phase = 0
        for t in range(tiles):
            for kb in range(kblocks):
                yield (("empty", c, stage), phase ^ 1)
                tma.append((c, stage, (t, kb)))
                stage += 1
                if stage == STAGES:
                    stage, phase = 0, phase ^ 1

    def split(c):
        stage = phase = 0
        for t in range(tiles):
            for kb in range(kblocks):
                yield (("full", c, stage), phase)
                assert hi[(c, stage)] == (t, kb), ("split reads", c, t, kb)
                lo[(c, stage)] = (t, kb)
                bars[("split", 0, stage)].arrive()
                stage += 1
                if stage == STAGES:
                    stage, phase = 0, phase ^ 1

    def mma():
        stage = phase = a = a_phase = 0
        for t in range(tiles):
            yield (("tempty", 0, a), a_phase ^ 1)
            for kb in range(kblocks):
                yield (("split", 0, stage), phase)
                fifo.append(("mma", t, kb, stage, a))
                fifo.append(("commit", "empty", stage))
                stage += 1
                if stage == STAGES:
                    stage, phase = 0, phase ^ 1
            fifo.append(("commit", "tfull", a))
            a += 1
            if a == 2:
                a, a_phase = 0, a_phase ^ 1

    def epilogue(c):
        a = a_phase = 0
        for t in range(tiles):
            yield (("tfull", c, a), a_phase)
            assert acc[(c, a)] == [t, kblocks], ("epilogue reads", c, t, acc[(c, a)])
            bars[("tempty", 0, a)].arrive()
            a += 1
            if a == 2:
                a, a_phase = 0, a_phase ^ 1

    makers = [("mma", mma)] + [(f"{n}{c}", (lambda f, c: lambda: f(c))(f, c))
                                for c in cta for n, f in (("prod", producer), ("split", split), ("epi", epilogue))]
    actors = {k: [f(), None] for k, f in makers}
    for a in actors.values():
        a[1] = next(a[0], "done")
    while True:
        ready = [k for k, a in actors.items() if a[1] != "done" and bars[a[1][0]].done(a[1][1])]
        choices = ready + (["tensor"] if fifo else []) + (["tma"] if tma else [])
        if not choices:
            assert all(a[1] == "done" for a in actors.values()), {k: a[1] for k, a in actors.items()}
            return
        ch = rng.choice(choices)
        if ch == "tensor":
            tensor(fifo.pop(0))
        elif ch == "tma":
            c, s, v = tma.pop(rng.randrange(len(tma)))
            hi[(c, s)] = v
            bars[("full", c, s)].arrive()
        else:
            actors[ch][1] = next(actors[ch][0], "done")


@pytest.mark.parametrize("seed", range(4))
def test_tf32_pair_gemm_protocol_under_random_schedules(seed):
    rng = random.Random(seed)
    for trial in range(200):
        simulate(rng.randint(1, 6), rng.randint(1, 8), seed * 1000 + trial)
