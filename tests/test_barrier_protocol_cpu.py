"""The head kernel's mbarrier protocol (rust_ppocrv6_b200/csrc/rechead_kernels.cu) restated as
a discrete-event model of one CTA, run on the CPU.

Every role is a sequence of waits ("barrier b has completed at least n phases") and arrivals
(weighted by how many arrivals the kernel makes there: one per warp where a warp elects one
lane, one per thread otherwise). A barrier completes a phase when its arrivals reach its
expected count; an arrival beyond the count is an over-arrival, which on the GPU is undefined
behaviour. Counting barriers are monotone (a wait that can pass stays passable until it
passes), so one maximal run decides whether the protocol can deadlock: if every role finishes
in one run, none can block for ever in any interleaving.

The model covers the three weight forms (fp16 image: 4 weight stages; compact int8: 3 fp16
stages filled by the expander warps from 2 landing slots, with each unit's A conversion
placed before the expansion of the unit's tile kStages8 - 1; FP32: 2 stages), the three
accumulators, the class-table ring, the per-unit A hand-over and row de-scale slots, and the
epilogue's 64-column halves and end-of-unit merge, over unit shapes from one tile per unit to
whole class ranges.
"""
import itertools

import pytest

ACC_BUFS = 3
CTAB_SLOTS = 4
EPI_GROUPS = 6
EXPANDER_WARPS = 4
STAGES = {"image": 4, "compact": 3, "f32": 2}
I8_SLOTS = 2


class Barrier:
    def __init__(self, count):
        self.count, self.arrived, self.done = count, 0, 0

    def arrive(self, weight=1):
        self.arrived += weight
        assert self.arrived <= self.count, "over-arrival"
        if self.arrived == self.count:
            self.arrived = 0
            self.done += 1


def run_cta(units, form):
    """Runs one CTA over `units` (tiles per work unit); returns the roles left blocked."""
    S = STAGES[form]
    expand = form == "compact"
    bars = {}

    def bar(name, count):
        bars[name] = Barrier(count)

    for i in range(S):
        bar(("BFull", i), EXPANDER_WARPS if expand else 1)
        bar(("BEmpty", i), 1)
    for i in range(I8_SLOTS):
        bar(("I8Full", i), 1)
        bar(("I8Empty", i), EXPANDER_WARPS)
    for i in range(ACC_BUFS):
        bar(("AccFull", i), 1)
        bar(("AccEmpty", i), 8)  # two groups' halves x four warps, one arrival per warp
    for i in range(CTAB_SLOTS):
        bar(("CtabFull", i), 1)
        bar(("CtabEmpty", i), 8)
    bar("AFull", 128)
    bar("AEmpty", 1)
    for i in range(4):
        bar(("Rho", i), 128)
    for i in range(2):
        bar(("MFull", i), 128 * (EPI_GROUPS - 1))
        bar(("MEmpty", i), 128)
    first_tile = list(itertools.accumulate([0] + units))

    def producer():  # warp 0: one bulk copy per tile
        ring, full, empty = (I8_SLOTS, "I8Full", "I8Empty") if expand else (S, "BFull", "BEmpty")
        for t in range(first_tile[-1]):
            yield (empty, t % ring), t // ring
            bars[(full, t % ring)].arrive()

    def mma():  # warp 1: per tile, both commits after its MMAs
        t = 0
        for u, n in enumerate(units):
            yield "AFull", u + 1
            for _ in range(n):
                yield ("BFull", t % S), t // S + 1
                yield ("AccEmpty", t % ACC_BUFS), t // ACC_BUFS
                bars[("BEmpty", t % S)].arrive()
                bars[("AccFull", t % ACC_BUFS)].arrive()
                t += 1
            bars["AEmpty"].arrive()

    def class_table():  # warp 2: copy, convert, publish (one lane arrives)
        for t in range(first_tile[-1]):
            yield ("CtabEmpty", t % CTAB_SLOTS), t // CTAB_SLOTS
            bars[("CtabFull", t % CTAB_SLOTS)].arrive()

    def convert(u):  # warps 4-7: A of unit u into TMEM, then the row de-scale
        yield "AEmpty", u
        bars["AFull"].arrive(128)
        bars[("Rho", u % 4)].arrive(128)

    def converters():
        if not expand:
            for u in range(len(units)):
                yield from convert(u)
            return
        au, a_first = 0, 0
        for t in range(first_tile[-1]):
            if au < len(units) and t == a_first + S - 1:
                yield from convert(au)
                a_first += units[au]
                au += 1
            yield ("I8Full", t % I8_SLOTS), t // I8_SLOTS + 1
            yield ("BEmpty", t % S), t // S
            bars[("BFull", t % S)].arrive(EXPANDER_WARPS)
            bars[("I8Empty", t % I8_SLOTS)].arrive(EXPANDER_WARPS)
        for u in range(au, len(units)):
            yield from convert(u)

    def epilogue(g):  # one group = four warps, modelled together (each warp arrives once)
        for u, n in enumerate(units):
            yield ("Rho", u % 4), u // 4 + 1
            for h in range(g, 2 * n, EPI_GROUPS):
                t = first_tile[u] + h // 2
                yield ("CtabFull", t % CTAB_SLOTS), t // CTAB_SLOTS + 1
                yield ("AccFull", t % ACC_BUFS), t // ACC_BUFS + 1
                bars[("AccEmpty", t % ACC_BUFS)].arrive(4)
                bars[("CtabEmpty", t % CTAB_SLOTS)].arrive(4)
            if g != 0:
                yield ("MEmpty", u % 2), u // 2
                bars[("MFull", u % 2)].arrive(128)
            else:
                yield ("MFull", u % 2), u // 2 + 1
                bars[("MEmpty", u % 2)].arrive(128)

    roles = {"producer": producer(), "mma": mma(), "converters": converters(), "class_table": class_table()}
    for g in range(EPI_GROUPS):
        roles[f"epilogue{g}"] = epilogue(g)
    pending = {k: None for k in roles}
    alive = set(roles)
    progressed = True
    while alive and progressed:
        progressed = False
        for k in list(alive):
            while True:
                w = pending[k]
                if w is not None and bars[w[0]].done < w[1]:
                    break
                try:
                    pending[k] = next(roles[k])
                    progressed = True
                except StopIteration:
                    alive.discard(k)
                    progressed = True
                    break
    return {k: pending[k] for k in alive}


UNIT_SHAPES = {
    "cfg2 (two class halves)": [74, 73] * 7,
    "whole class range": [147] * 7,
    "one tile per unit": [1] * 20,
    "ragged": [2, 3, 1, 5, 8, 2, 1, 1, 13],
    "tiny head (K=80, N=6906)": [55] * 9,
    "split plans": [9] * 17 + [3],
    "cfg2 plan (six whole row blocks, then a split one)": [147] * 6 + [74],
}


@pytest.mark.parametrize("form", ["image", "compact", "f32"])
@pytest.mark.parametrize("shape", list(UNIT_SHAPES))
def test_protocol_finishes_without_deadlock_or_over_arrival(form, shape):
    blocked = run_cta(UNIT_SHAPES[shape], form)
    assert not blocked, f"{form} / {shape}: roles blocked for ever: {blocked}"


def test_model_detects_a_broken_protocol():
    """The checker is not vacuous: an expansion order that converts a unit's A after the
    expansion its own MMAs must free first deadlocks, and a barrier expecting one arrival
    where a whole warp arrives over-arrives."""
    # A converted only after all expansions of its unit: unit 0's tile 3 needs stage 0 freed by
    # MMA(0), which waits for A(0)
    assert run_cta_late_conversion([8, 8])
    b = Barrier(1)
    with pytest.raises(AssertionError):
        b.arrive(32)


def run_cta_late_conversion(units):
    """run_cta's compact form with each unit's A conversion moved after the unit's expansions."""
    S = STAGES["compact"]
    bars = {("BFull", i): Barrier(EXPANDER_WARPS) for i in range(S)}
    bars.update({("BEmpty", i): Barrier(1) for i in range(S)})
    bars.update({("I8Full", i): Barrier(1) for i in range(I8_SLOTS)})
    bars.update({("I8Empty", i): Barrier(EXPANDER_WARPS) for i in range(I8_SLOTS)})
    bars.update({"AFull": Barrier(1), "AEmpty": Barrier(1)})
    total = sum(units)

    def producer():
        for t in range(total):
            yield ("I8Empty", t % I8_SLOTS), t // I8_SLOTS
            bars[("I8Full", t % I8_SLOTS)].arrive()

    def mma():
        t = 0
        for u, n in enumerate(units):
            yield "AFull", u + 1
            for _ in range(n):
                yield ("BFull", t % S), t // S + 1
                bars[("BEmpty", t % S)].arrive()
                t += 1
            bars["AEmpty"].arrive()

    def converters():
        t = 0
        for u, n in enumerate(units):
            for _ in range(n):
                yield ("I8Full", t % I8_SLOTS), t // I8_SLOTS + 1
                yield ("BEmpty", t % S), t // S
                bars[("BFull", t % S)].arrive(EXPANDER_WARPS)
                bars[("I8Empty", t % I8_SLOTS)].arrive(EXPANDER_WARPS)
                t += 1
            yield "AEmpty", u
            bars["AFull"].arrive()

    roles = {"producer": producer(), "mma": mma(), "converters": converters()}
    pending = {k: None for k in roles}
    alive = set(roles)
    progressed = True
    while alive and progressed:
        progressed = False
        for k in list(alive):
            while True:
                w = pending[k]
                if w is not None and bars[w[0]].done < w[1]:
                    break
                try:
                    pending[k] = next(roles[k])
                    progressed = True
                except StopIteration:
                    alive.discard(k)
                    progressed = True
                    break
    return {k: pending[k] for k in alive}
