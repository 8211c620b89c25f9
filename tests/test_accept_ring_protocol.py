"""CPU model of the acceptance kernel's shared-memory ring (specgrove_b200/csrc/accept.cu).

Each CTA streams its slice of a probability row through `kSlots` 4 KB slots:
thread 0 issues the first fill of every slot at the start of a pass, block i
lands in slot i % kSlots and is reduced by warp i % kWarps, and the warp that
has read a slot issues its next fill.  A slot's mbarrier completes one phase
per fill and waiters use parity waits, which cannot tell phase k from phase
k - 2.  The model runs random interleavings of the warps and of the copies'
completions over several passes and checks that every wait returns only once
its own block has landed and that no slot is refilled while a fill is in
flight.  It reads the constants from the kernel source, and a layout whose
slot count is not a multiple of its warps (12 slots over 8 warps) must fail.
"""
from __future__ import annotations

import random
import re
from pathlib import Path

import pytest

SRC = Path(__file__).resolve().parents[1] / "specgrove_b200" / "csrc" / "accept.cu"


def kernel_constants():
    text = SRC.read_text()
    threads = int(re.search(r"constexpr int kThreads = (\d+);", text).group(1))
    slots = int(re.search(r"constexpr int kSlots = (\d+);", text).group(1))
    return threads // 32, slots


class ProtocolError(AssertionError):
    pass


def simulate(warps: int, slots: int, nb: int, passes: int, rng: random.Random) -> None:
    completed = [0] * slots          # completed phases per slot barrier
    pending = [None] * slots         # block whose copy is in flight
    content = [None] * slots         # block that has landed in the slot
    for p in range(passes):
        fills = [(nb - s + slots - 1) // slots if s < nb else 0 for s in range(slots)]

        def issue(block):
            s = block % slots
            if pending[s] is not None:
                raise ProtocolError(f"slot {s} refilled with block {block} while block {pending[s]} is in flight")
            pending[s] = block
            content[s] = None

        # per-warp programs; warp 0 first issues the initial fills
        programs = []
        for w in range(warps):
            ops = []
            if w == 0:
                ops += [("issue", s) for s in range(min(slots, nb))]
            for i in range(w, nb, warps):
                ops += [("wait", i), ("read", i)]
                if i + slots < nb:
                    ops.append(("issue", i + slots))
            programs.append(ops)
        pcs = [0] * warps
        while True:
            actors = []
            for w in range(warps):
                if pcs[w] < len(programs[w]):
                    kind, i = programs[w][pcs[w]]
                    if kind == "wait":
                        s = i % slots
                        parity = (p * fills[s] + i // slots) & 1
                        if (completed[s] & 1) == parity:   # the awaited phase is still in progress
                            continue
                    actors.append(("warp", w))
            actors += [("copy", s) for s in range(slots) if pending[s] is not None]
            if not actors:
                break
            kind, who = rng.choice(actors)
            if kind == "copy":
                content[who] = pending[who]
                pending[who] = None
                completed[who] += 1
                continue
            op, i = programs[who][pcs[who]]
            pcs[who] += 1
            if op == "issue":
                issue(i)
            elif op == "read":
                if content[i % slots] != i:
                    raise ProtocolError(f"warp {who} read slot {i % slots} for block {i}, "
                                        f"which holds {content[i % slots]}")
        if any(pc < len(prog) for pc, prog in zip(pcs, programs)):
            raise ProtocolError("deadlock")
        if any(x is not None for x in pending):
            raise ProtocolError("a fill is still in flight at the end of the pass")


@pytest.mark.parametrize("nb", [1, 5, 12, 16, 19, 35, 38, 75, 149])
def test_ring_protocol_holds(nb):
    warps, slots = kernel_constants()
    rng = random.Random(nb)
    for _ in range(300):
        simulate(warps, slots, nb, passes=3, rng=rng)


def test_shared_slots_are_caught():
    rng = random.Random(7)
    with pytest.raises(ProtocolError):
        for _ in range(2000):
            simulate(8, 12, 38, passes=3, rng=rng)
