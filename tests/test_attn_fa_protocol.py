"""The barrier protocol of attn_fa_kernel (attention_fa.cu), modelled on the
CPU: its roles (the load warp, the MMA thread, the two softmax warpgroups)
as the kernel orders them, mbarriers with the hardware's phase and parity
semantics (try_wait.parity(p) succeeds once the phase of parity p has
completed, i.e. while the current phase's parity differs from p), MMAs
executing in issue order, TMA loads completing in any order. Units carry two
tiles, the second absent in some (an odd last head, or a row's last 128
queries alone). Under random schedules no role may wait forever, and every
read of a shared-memory or tensor-memory buffer must see the version the
protocol promises. The same model fails on a variant with one O barrier a
tile (a final wait two phases behind reads O before its last P V) and on
one with one P barrier a tile (the softmax writes P(c + 1) before the MMA
thread waits for P(c): two phases, and the wait never returns)."""
import random

import pytest

NKV = 3


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


def simulate(units, seed, rescale_p=0.3, one_o_barrier=False, one_p_barrier=False):
    """units: [(nch, has1)], the CTA's units in order."""
    rng = random.Random(seed)
    stream = [(u, j, n, h1) for u, (n, h1) in enumerate(units) for j in range(n)]
    names = ["qf0", "qf1", "qe0", "qe1"] + [f"{x}{i}" for x in ("kf", "ke", "vf", "ve") for i in range(NKV)]
    for t in (0, 1):
        names += [f"s{t}_0", f"s{t}_1", f"p{t}_0", f"p{t}_1", f"o{t}_0", f"o{t}_1"]
    bars = {k: Bar(1) for k in names}
    st = dict(Q=[None, None], K=[None] * NKV, V=[None] * NKV, S={(t, b): None for t in (0, 1) for b in (0, 1)},
              O=[None, None])
    fifo, tma = [], []
    obar = (lambda t, g: f"o{t}_0") if one_o_barrier else (lambda t, g: f"o{t}_{g & 1}")
    pbar = (lambda t, g: f"p{t}_0") if one_p_barrier else (lambda t, g: f"p{t}_{g & 1}")
    ppar = (lambda g: g & 1) if one_p_barrier else (lambda g: (g >> 1) & 1)
    # Tile 1's chunk index of each stream chunk.
    g1_of, g1 = [], 0
    for u, j, n, h1 in stream:
        g1_of.append(g1 if h1 else None)
        g1 += 1 if h1 else 0

    def tensor(op):
        kind = op[0]
        if kind == "S":
            t, c, g = op[1], op[2], op[3]
            u = stream[c][0]
            assert st["Q"][u & 1] == u and st["K"][c % NKV] == c, ("S operands", t, c)
            st["S"][(t, g & 1)] = ("S", g)
        elif kind == "PV":
            t, c, g = op[1], op[2], op[3]
            u, j = stream[c][0], stream[c][1]
            assert st["S"][(t, g & 1)] == ("P", g) and st["V"][c % NKV] == c, ("PV operands", t, c)
            if j == 0:
                st["O"][t] = (u, [g])
            else:
                assert st["O"][t][0] == u and st["O"][t][1][-1] == g - 1, ("PV accumulates", t, c)
                st["O"][t][1].append(g)
        else:
            bars[op[1]].arrive()

    def loader():
        c = 0
        for u, (n, h1) in enumerate(units):
            qb = u & 1
            if u >= 2:
                yield (f"qe{qb}", ((u >> 1) - 1) & 1)
            tma.append(("Q", qb, u, f"qf{qb}"))
            for j in range(n):
                s = c % NKV
                if c >= NKV:
                    yield (f"ke{s}", ((c // NKV) - 1) & 1)
                tma.append(("K", s, c, f"kf{s}"))
                if c >= NKV:
                    yield (f"ve{s}", ((c // NKV) - 1) & 1)
                tma.append(("V", s, c, f"vf{s}"))
                c += 1

    def mma():
        cur = dict(s=0)

        def issue_s():
            c = cur["s"]
            u, j, n, h1 = stream[c]
            if j == 0:
                yield (f"qf{u & 1}", (u >> 1) & 1)
            yield (f"kf{c % NKV}", (c // NKV) & 1)
            for t in (0, 1):
                if t == 1 and not h1:
                    break
                g = c if t == 0 else g1_of[c]
                fifo.extend([("S", t, c, g), ("commit", f"s{t}_{g & 1}")])
            fifo.append(("commit", f"ke{c % NKV}"))
            if j + 1 == n:
                fifo.append(("commit", f"qe{u & 1}"))
            cur["s"] += 1

        for _ in range(2):
            if cur["s"] < len(stream):
                yield from issue_s()
        for c, (u, j, n, h1) in enumerate(stream):
            yield (f"vf{c % NKV}", (c // NKV) & 1)
            for t in (0, 1):
                if t == 1 and not h1:
                    break
                g = c if t == 0 else g1_of[c]
                yield (pbar(t, g), ppar(g))
                fifo.extend([("PV", t, c, g), ("commit", obar(t, g))])
            fifo.append(("commit", f"ve{c % NKV}"))
            if cur["s"] < len(stream):
                yield from issue_s()

    def softmax(t):
        g = 0
        for c, (u, j, n, h1) in enumerate(stream):
            if t == 1 and not h1:
                continue
            sb = g & 1
            yield (f"s{t}_{sb}", (g >> 1) & 1)
            assert st["S"][(t, sb)] == ("S", g), ("softmax reads S", t, g)
            if j > 0 and rng.random() < rescale_p:  # O rescaled in tensor memory
                yield (obar(t, g - 1), ((g - 1) >> 1) & 1 if not one_o_barrier else (g - 1) & 1)
                assert st["O"][t] == (u, list(range(g - j, g))), ("rescale reads O", t, g)
            st["S"][(t, sb)] = ("P", g)
            bars[pbar(t, g)].arrive()
            g += 1
            if j + 1 == n:
                yield (obar(t, g - 1), ((g - 1) >> 1) & 1 if not one_o_barrier else (g - 1) & 1)
                assert st["O"][t] == (u, list(range(g - n, g))), ("final O", t, g)

    actors = {k: [f(), None] for k, f in (("load", loader), ("mma", mma), ("sm0", lambda: softmax(0)),
                                          ("sm1", lambda: softmax(1)))}
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
            kind, slot, val, bar = tma.pop(rng.randrange(len(tma)))
            st[kind][slot] = val
            bars[bar].arrive()
        else:
            actors[c][1] = next(actors[c][0], "done")


def random_units(rng):
    return [(rng.randint(1, 6), rng.random() < 0.8) for _ in range(rng.randint(1, 8))]


@pytest.mark.parametrize("seed", range(4))
def test_fa_attention_protocol_under_random_schedules(seed):
    rng = random.Random(seed)
    for trial in range(300):
        simulate(random_units(rng), seed * 1000 + trial)


def test_the_model_catches_a_single_o_barrier():
    # One O barrier a tile: a final wait after two P V completions aliases
    # the parity and reads O early, or never returns.
    rng = random.Random(7)
    failed = 0
    for trial in range(300):
        try:
            simulate(random_units(rng), 7000 + trial, rescale_p=0.0, one_o_barrier=True)
        except AssertionError:
            failed += 1
    assert failed > 0


def test_the_model_catches_a_single_p_barrier():
    rng = random.Random(8)
    failed = 0
    for trial in range(300):
        try:
            simulate(random_units(rng), 8000 + trial, one_p_barrier=True)
        except AssertionError:
            failed += 1
    assert failed > 0
