"""The barrier protocol of attn_tf32_kernel (attention_tf32.cu), modelled on
the CPU: its four roles (the Q/K load warp, the MMA thread, the transposer,
the softmax) as the kernel orders them, mbarriers with the hardware's phase
and parity semantics (try_wait.parity(p) succeeds once the phase of parity p
has completed, i.e. while the current phase's parity differs from p), MMAs
executing in issue order, TMA loads completing in any order. Under random
schedules no role may wait forever and every read of a shared-memory or
tensor-memory buffer must see the version the protocol promises. The same
model fails on the two protocols the kernel had before (one P V barrier with
one final wait reads O early; one P V barrier with a two-step final wait
deadlocks), which is how both were found."""
import random

import pytest


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


def simulate(units_nch, seed, rescale_p=0.3):
    rng = random.Random(seed)
    stream = [(u, j, n) for u, n in enumerate(units_nch) for j in range(n)]
    bars = {k: Bar(1) for k in ["q", "qf"] + [f"{x}{b}" for x in ("k", "kf", "v", "vf", "s", "p", "o") for b in (0, 1)]}
    st = dict(K=[None, None], Q=None, SP=[None, None], PL=[None, None], Vt=[None, None], O=None)
    fifo, tma = [], []

    def tensor(op):
        if op[0] == "S":
            z, b = op[1], op[2]
            assert st["K"][b] == z and st["Q"] == stream[z][0], ("S operands", z)
            st["SP"][b] = ("S", z)
        elif op[0] == "PV":
            y, b = op[1], op[2]
            assert st["SP"][b] == ("P", y) and st["PL"][b] == y and st["Vt"][b] == y, ("PV operands", y)
            u, j, _ = stream[y]
            if j == 0:
                st["O"] = (u, [y])
            else:
                assert st["O"][0] == u and st["O"][1][-1] == y - 1, ("PV accumulates", y)
                st["O"][1].append(y)
        else:
            bars[op[1]].arrive()

    def loader():
        z = qn = 0
        for u, j, _ in stream:
            if j == 0:
                if qn >= 1:
                    yield ("qf", (qn - 1) & 1)
                tma.append(("Q", u, "q"))
                qn += 1
            b = z & 1
            if z >= 2:
                yield (f"kf{b}", ((z >> 1) & 1) ^ 1)
            tma.append(("K", (b, z), f"k{b}"))
            z += 1

    def mma():
        state = dict(zs=0, qn=0, si=0)

        def issue_s():
            u, j, n = stream[state["si"]]
            b = state["zs"] & 1
            if j == 0:
                yield ("q", state["qn"] & 1)
                state["qn"] += 1
            yield (f"k{b}", (state["zs"] >> 1) & 1)
            fifo.extend([("S", state["zs"], b), ("commit", f"s{b}"), ("commit", f"kf{b}")])
            if j + 1 == n:
                fifo.append(("commit", "qf"))
            state["zs"] += 1
            state["si"] += 1

        for _ in range(2):
            if state["si"] < len(stream):
                yield from issue_s()
        for y in range(len(stream)):
            b = y & 1
            yield (f"p{b}", (y >> 1) & 1)
            yield (f"v{b}", (y >> 1) & 1)
            fifo.extend([("PV", y, b), ("commit", f"o{b}"), ("commit", f"vf{b}")])
            if state["si"] < len(stream):
                yield from issue_s()

    def transposer():
        for y in range(len(stream)):
            b = y & 1
            if y >= 2:
                yield (f"vf{b}", ((y >> 1) & 1) ^ 1)
            st["Vt"][b] = y
            bars[f"v{b}"].arrive()

    def softmax():
        g = 0
        for u, j, n in stream:
            sb = g & 1
            yield (f"s{sb}", (g >> 1) & 1)
            assert st["SP"][sb] == ("S", g), ("softmax reads S", g)
            if j > 0 and rng.random() < rescale_p:  # O rescaled in tensor memory
                yield (f"o{(g - 1) & 1}", ((g - 1) >> 1) & 1)
                assert st["O"] == (u, list(range(g - j, g))), ("rescale reads O", g)
            st["SP"][sb], st["PL"][sb] = ("P", g), g
            bars[f"p{sb}"].arrive()
            g += 1
            if j + 1 == n:
                yield (f"o{(g - 1) & 1}", ((g - 1) >> 1) & 1)
                assert st["O"] == (u, list(range(g - n, g))), ("final O", g)

    actors = {k: [f(), None] for k, f in (("load", loader), ("mma", mma), ("tr", transposer), ("sm", softmax))}
    for a in actors.values():
        a[1] = next(a[0], "done")
    while True:
        ready = [k for k, a in actors.items() if a[1] != "done" and bars[a[1][0]].done(a[1][1])]
        choices = ready + (["tensor"] if fifo else []) + (["tma"] if tma else [])
        if not choices:
            assert all(a[1] == "done" for a in actors.values()), {k: a[1] for k, a in actors.items()}
            return
        c = rng.choice(choices)
        if c == "tensor":
            tensor(fifo.pop(0))
        elif c == "tma":
            kind, val, bar = tma.pop(rng.randrange(len(tma)))
            if kind == "Q":
                st["Q"] = val
            else:
                st["K"][val[0]] = val[1]
            bars[bar].arrive()
        else:
            actors[c][1] = next(actors[c][0], "done")


@pytest.mark.parametrize("seed", range(4))
def test_tf32_attention_protocol_under_random_schedules(seed):
    rng = random.Random(seed)
    for trial in range(300):
        units = [rng.randint(1, 6) for _ in range(rng.randint(1, 7))]
        simulate(units, seed * 1000 + trial)
