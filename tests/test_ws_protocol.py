"""CPU model of the warp-specialised kernel's mbarrier protocol (fused-lncc_b200/csrc/lncc_ws.cuh).

One cluster of CTAs; per CTA 4 A warps, 8 BC warps and 4 D warps walk the same step sequence with random
work times, and the halo bulk copies (one per A warp: warps 0-1 to the CTA above, 2-3 below) land after
random delays. Each D warp also boxes two of the five fields for its paired A warp (same rows): it
waits until the buffer is free and the pair's running sums are complete (ya), writes its fields and
signals xd, which the A warp waits for before announcing its rows and sending the halo; the D warps do
this for the first two steps of a segment, then for step s + 2 before the adjoints of step s.
Barriers are modelled like mbarriers
(arrival count, pending count, transaction bytes, phase). Every arrival and every completed copy is
tagged with the phase it is meant for; a tag different from the barrier's current phase is a protocol
violation (the hardware would count it silently in the wrong phase), and actors left waiting at the end
are a deadlock.

The kernel sends the halo rows on every step, planes outside the volume included. The model shows why:
sending them only for planes inside the volume lets a neighbour run two steps ahead across the padding
steps at a volume boundary and arrive on the wrong phase.
"""
import heapq
import random


class Bar:
    def __init__(self, count):
        self.count = count
        self.pending = count
        self.tx = 0
        self.phase = 0

    def _maybe_complete(self):
        if self.pending == 0 and self.tx == 0:
            self.phase += 1
            self.pending = self.count


def simulate(ncta, steps_valid, always_send, seed, slow_cta=None, seg_len=None):
    rnd = random.Random(seed)
    nsteps = len(steps_valid)
    seg_len = seg_len or nsteps
    seg_start = [s - s % seg_len for s in range(nsteps)]  # first step of each step's segment
    bars = {}
    for j in range(ncta):
        nb = 8 * (1 + (j > 0) + (j < ncta - 1))
        for i in range(2):
            bars[(j, "full", i)] = Bar(4)
            bars[(j, "empty", i)] = Bar(nb)
            bars[(j, "ahfull", i)] = Bar(8)
            bars[(j, "ahempty", i)] = Bar(4)
        for w in range(4):
            bars[(j, "xd", w)] = Bar(1)
            bars[(j, "ya", w)] = Bar(1)
    violations = []
    t = [0.0]
    events = []  # (time, seq, fn)
    seq = [0]

    def at(time, fn):
        seq[0] += 1
        heapq.heappush(events, (time, seq[0], fn))

    def arrive(key, tag, tx=0):
        b = bars[key]
        if tag != b.phase:
            violations.append((key, tag, b.phase))
        b.tx += tx
        b.pending -= 1
        b._maybe_complete()

    def complete_tx(key, tag, n):
        b = bars[key]
        if tag != b.phase:
            violations.append((key, "tx", tag, b.phase))
        b.tx -= n
        b._maybe_complete()

    def done(key, phase):  # phase `phase` has completed
        return bars[key].phase > phase

    HALO = 100

    def dur(j):
        d = rnd.expovariate(1.0)
        if slow_cta is not None and j == slow_cta and rnd.random() < 0.3:
            d *= 20
        return d

    # actor state machines: generators yielding ("wait", key, phase) or ("work", dt)
    def A(j, w):
        for s in range(nsteps):
            i, u = s & 1, s >> 1
            if s == seg_start[s]:  # warm-up of the segment's running sums
                yield ("work", dur(j))
                arrive((j, "ya", w), s)
            if s >= 2:
                yield ("wait", (j, "empty", i), u - 1)
            yield ("work", dur(j))
            yield ("wait", (j, "xd", w), s)
            valid = steps_valid[s]
            send = always_send or valid
            ntx = HALO * ((j > 0) + (j < ncta - 1))
            arrive((j, "full", i), u, tx=(ntx if (w == 0 and send) else 0))
            # each warp sends its own halo rows: warps 0, 1 to the CTA above, warps 2, 3 below
            nb = j - 1 if w < 2 else j + 1
            if send and 0 <= nb < ncta:
                at(t[0] + rnd.expovariate(0.5), lambda nb=nb, i=i, u=u: complete_tx((nb, "full", i), u, HALO // 2))
            if s + 1 < nsteps and seg_start[s + 1] == seg_start[s]:
                yield ("work", dur(j) * 0.5)  # running sums of the next step
                arrive((j, "ya", w), s + 1)

    def BC(j, w):
        for s in range(nsteps):
            i, u = s & 1, s >> 1
            yield ("wait", (j, "full", i), u)
            if s >= 2:
                yield ("wait", (j, "ahempty", i), u - 1)
            yield ("work", dur(j) * 2)
            for nb in (j - 1, j, j + 1):
                if 0 <= nb < ncta:
                    arrive((nb, "empty", i), u)
            arrive((j, "ahfull", i), u)

    def d_part(j, w, st):
        if st >= 2:
            yield ("wait", (j, "empty", st & 1), (st >> 1) - 1)
        yield ("wait", (j, "ya", w), st)
        yield ("work", dur(j) * 0.3)
        arrive((j, "xd", w), st)

    def D(j, w):
        for s in range(nsteps):
            i, u = s & 1, s >> 1
            if s == seg_start[s]:
                for st in (s, s + 1):
                    yield from d_part(j, w, st)
            if s + 2 < nsteps and seg_start[s + 2] == seg_start[s]:
                yield from d_part(j, w, s + 2)
            yield ("wait", (j, "ahfull", i), u)
            yield ("work", dur(j))
            arrive((j, "ahempty", i), u)

    actors = []
    for j in range(ncta):
        actors += [A(j, w) for w in range(4)] + [BC(j, w) for w in range(8)] + [D(j, w) for w in range(4)]
    waiting = {}  # actor index -> (key, phase)

    def step(k):
        g = actors[k]
        try:
            op = next(g)
        except StopIteration:
            waiting.pop(k, None)
            return
        if op[0] == "work":
            at(t[0] + op[1], lambda k=k: step(k))
        else:
            waiting[k] = (op[1], op[2])

    for k in range(len(actors)):
        at(0.0, lambda k=k: step(k))
    while True:
        # release satisfied waiters
        ready = [k for k, (key, ph) in waiting.items() if done(key, ph)]
        for k in ready:
            del waiting[k]
            at(t[0], lambda k=k: step(k))
        if not events:
            break
        t[0], _, fn = heapq.heappop(events)
        fn()
    return violations, len(waiting)


def _steps(R, nseg=3, inner=12):
    seg = [False] * R + [True] * inner + [False] * R
    return seg * nseg


def test_protocol_has_no_misaligned_arrivals_or_deadlock():
    for R in (1, 4):
        for seed in range(24):
            violations, waiting = simulate(8, _steps(R), True, seed, slow_cta=seed % 8, seg_len=12 + 2 * R)
            assert not violations, (R, seed, violations[:3])
            assert waiting == 0, (R, seed)


def test_protocol_with_16_ctas():
    # planes of 129 - 256 rows run as one chain of up to 16 CTAs (non-portable cluster)
    for seed in range(6):
        violations, waiting = simulate(16, _steps(3), True, seed, slow_cta=seed % 16, seg_len=12 + 2 * 3)
        assert not violations, (seed, violations[:3])
        assert waiting == 0, seed


def test_model_detects_halo_sent_only_for_valid_planes():
    # the rule the kernel does not use: the model must catch its misaligned arrivals
    hits = 0
    for seed in range(24):
        violations, _ = simulate(8, _steps(4), False, seed, slow_cta=seed % 8)
        hits += bool(violations)
    assert hits > 0
