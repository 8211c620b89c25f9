"""Executable model of the persistent tree-attention CTA's barrier protocol.

Test infrastructure: a randomised discrete-event model of the warp roles of
`tree_attention_tm_kernel` (specgrove_b200/csrc/attention.cu) with mbarrier
semantics (arrival counts, phases, parity waits), asynchronous completions
(TMA loads land and tcgen05 commits fire at random later steps, commits in
issue order) and checks for deadlock, arrival overflow and tensor-memory /
shared-memory hazards.  Each softmax warp is one actor whose arrivals count
32 threads.

Roles, as in the kernel:
  scheduler + K producer  publishes work items into two slots, streams K tiles
  V producer              follows the items, streams V tiles
  MMA issuer              QK^T of tile g after K_g landed and S_{g-1} was read;
                          PV of tile g-1 after P_{g-1} was written and V landed
  softmax warps (8)       per tile: wait S, read S, release S, wait PV of the
                          previous tile, write P, release P; idle quarters take
                          the same barrier steps; the next item's Q is staged
                          at the current item's last tile; merge + epilogue.

`bugs` plants historical mistakes so the tests can show the model catches
them: "skip_idle" (idle quarters skip the per-tile barrier steps, relying on
a proxy arrival) and "no_v_wait" (tail-tile V zeroing without waiting for the
V tile).
"""
from __future__ import annotations

import random


class Hazard(Exception):
    """A data hazard or protocol violation found by the model."""


class Bar:
    """mbarrier: expected count, pending arrivals, completed-phase counter."""

    def __init__(self, name: str, count: int, arrivals: list):
        self.name, self.count, self.pending, self.phase = name, count, count, 0
        self._arrivals = arrivals

    def arrive(self, n: int = 1) -> None:
        self._arrivals[0] += 1
        self.pending -= n
        if self.pending < 0:
            raise Hazard(f"arrival overflow on {self.name} (phase {self.phase})")
        if self.pending == 0:
            self.phase += 1
            self.pending = self.count

    def done(self, parity: int) -> bool:
        """try_wait.parity: true once the phase with this parity completed."""
        return (self.phase & 1) != parity


def run(items, kst: int = 4, vst: int = 3, seed: int = 0, bugs: frozenset = frozenset()) -> int:
    """Simulate one CTA over `items` = [(tiles, active_quarters)]; returns steps."""
    rng = random.Random(seed)
    arrivals = [0]
    bars = {}

    def bar(name, count):
        bars[name] = Bar(name, count, arrivals)
        return bars[name]

    k_full = [bar(f"k_full{i}", 1) for i in range(kst)]
    k_empty = [bar(f"k_empty{i}", 1) for i in range(kst)]
    v_full = [bar(f"v_full{i}", 1) for i in range(vst)]
    v_empty = [bar(f"v_empty{i}", 1) for i in range(vst)]
    s_full, s_free, p_full, o_done, q_full = (bar("s_full", 1), bar("s_free", 256), bar("p_full", 256),
                                             bar("o_done", 1), bar("q_full", 256))
    merge = [bar(f"merge{q}", 64) for q in range(4)]
    item_full = [bar(f"item_full{i}", 1) for i in range(2)]
    item_empty = [bar(f"item_empty{i}", 2 + 256) for i in range(2)]
    slots = [None, None]
    loads = []      # (barrier, (ring, slot, tile)) landing at a random later step
    mma = []        # in-order tcgen05 work: (kind, tile, [barriers to arrive on])
    landed = {}     # (ring, slot) -> tile whose data is in that slot

    def wait(b, parity):
        while not b.done(parity):
            yield ("wait", b.name)

    def next_item(seq, n):
        yield from wait(item_full[seq & 1], (seq >> 1) & 1)
        it = slots[seq & 1]
        item_empty[seq & 1].arrive(n)
        return it

    def scheduler():
        gt = 0
        for seq in range(len(items) + 1):
            it = (tuple(items[seq]) + (seq,)) if seq < len(items) else None
            yield from wait(item_empty[seq & 1], ((seq >> 1) & 1) ^ 1)
            slots[seq & 1] = it
            item_full[seq & 1].arrive()
            yield ("step",)
            if it is None:
                return
            for _ in range(it[0]):
                s = gt % kst
                yield from wait(k_empty[s], ((gt // kst) & 1) ^ 1)
                loads.append((k_full[s], ("k", s, gt)))
                gt += 1
                yield ("step",)

    def v_producer():
        gt, seq = 0, 0
        while True:
            it = yield from next_item(seq, 1)
            if it is None:
                return
            for _ in range(it[0]):
                s = gt % vst
                yield from wait(v_empty[s], ((gt // vst) & 1) ^ 1)
                loads.append((v_full[s], ("v", s, gt)))
                gt += 1
                yield ("step",)
            seq += 1

    def mma_issuer():
        gt, seq = 0, 0
        while True:
            it = yield from next_item(seq, 1)
            if it is None:
                return
            tiles = it[0]
            yield from wait(q_full, seq & 1)
            for j in range(tiles + 1):
                g = gt + j
                if j < tiles:
                    s = g % kst
                    yield from wait(k_full[s], (g // kst) & 1)
                    if g > 0:
                        yield from wait(s_free, (g - 1) & 1)
                    if landed.get(("k", s)) != g:
                        raise Hazard(f"QK {g} reads K of tile {landed.get(('k', s))}")
                    mma.append(("qk", g, [k_empty[s], s_full]))
                    yield ("step",)
                if j > 0:
                    s = (g - 1) % vst
                    yield from wait(p_full, (g - 1) & 1)
                    yield from wait(v_full[s], ((g - 1) // vst) & 1)
                    if landed.get(("v", s)) != g - 1:
                        raise Hazard(f"PV {g - 1} reads V of tile {landed.get(('v', s))}")
                    mma.append(("pv", g - 1, [v_empty[s], o_done]))
                    yield ("step",)
            gt += tiles
            seq += 1

    def softmax(warp):
        quarter = warp & 3
        gt, merges, seq = 0, 0, 0
        it = yield from next_item(0, 32)
        if it is None:
            return
        if quarter < it[1]:
            if any(k == "qk" for k, _, _ in mma):
                raise Hazard("Q written while a QK^T is in flight")
            yield ("step",)
        q_full.arrive(32)
        while it is not None:
            tiles, aq = it[0], it[1]
            active = quarter < aq
            nx = None
            skip = "skip_idle" in bugs and not active
            proxy_extra = 64 * (4 - aq) if ("skip_idle" in bugs and warp == 4) else 0
            for j in range(tiles):
                g = gt + j
                if not skip:
                    yield from wait(s_full, g & 1)
                    if active and any(k == "qk" and t == g for k, t, _ in mma):
                        raise Hazard("S read before its QK^T completed")
                    yield ("step",)
                    s_free.arrive(32 + proxy_extra)
                if j == tiles - 1:
                    yield from wait(item_full[(seq + 1) & 1], ((seq + 1) >> 1) & 1)
                    nx = slots[(seq + 1) & 1]
                    if nx is not None:
                        if quarter < nx[1]:
                            if any(k == "qk" for k, _, _ in mma):
                                raise Hazard(f"warp {warp} stages the next Q while a QK^T is in flight")
                            yield ("step",)
                        q_full.arrive(32)
                if skip:
                    continue
                if j > 0:
                    yield from wait(o_done, (g - 1) & 1)
                if active and any(k == "pv" for k, _, _ in mma):
                    raise Hazard(f"warp {warp} writes P while a PV is in flight")
                if active and rng.random() < 0.3:  # a tail tile: zero stale V rows
                    s = g % vst
                    if "no_v_wait" not in bugs:
                        yield from wait(v_full[s], (g // vst) & 1)
                    if landed.get(("v", s)) != g:
                        raise Hazard(f"V zeroing of tile {g} sees V of tile {landed.get(('v', s))}")
                yield ("step",)
                p_full.arrive(32 + proxy_extra)
            if not skip:
                yield from wait(o_done, (gt + tiles - 1) & 1)
            if active:
                merge[quarter].arrive(32)
                yield from wait(merge[quarter], merges & 1)
                merges += 1
                if any(k == "pv" for k, _, _ in mma):
                    raise Hazard(f"warp {warp} reads O while a PV is in flight")
                yield ("step",)
            if slots[(seq + 1) & 1] is not nx:
                raise Hazard("next item's slot overwritten before its release")
            item_empty[(seq + 1) & 1].arrive(32)
            gt += tiles
            seq += 1
            it = nx

    actors = {"sched": scheduler(), "vprod": v_producer(), "mma": mma_issuer()}
    for w in range(3, 11):
        actors[f"softmax{w}"] = softmax(w)
    blocked = {}
    steps = 0
    while actors:
        steps += 1
        if steps > 400000:
            raise RuntimeError("model did not finish")
        choices = list(actors) + ["#load"] * (2 if loads else 0) + ["#mma"] * (2 if mma else 0)
        rng.shuffle(choices)
        before = arrivals[0]
        progressed = False
        for c in choices:
            if c == "#load":
                b, (ring, s, t) = loads.pop(rng.randrange(len(loads)))
                landed[(ring, s)] = t
                b.arrive()
                progressed = True
                break
            if c == "#mma":
                _, _, commits = mma.pop(0)
                for b in commits:
                    b.arrive()
                progressed = True
                break
            try:
                r = next(actors[c])
            except StopIteration:
                del actors[c]
                progressed = True
                break
            if r[0] == "wait":
                blocked[c] = r[1]
                if arrivals[0] != before:
                    progressed = True
                    break
                continue
            progressed = True
            break
        if not progressed:
            raise Hazard("deadlock: " + ", ".join(f"{k} waits {blocked.get(k)}" for k in actors))
    if loads or mma:
        raise Hazard("work still in flight at exit")
    return steps


def random_items(rng: random.Random):
    return [(rng.randint(1, 6), rng.randint(1, 4)) for _ in range(rng.randint(1, 10))]
