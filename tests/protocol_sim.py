"""A small model of the peer-memory flag protocols, for CPU tests.

Each rank is a generator of operations on shared state, executed in a random
interleaving (one operation of one runnable rank at a time):

* ``("write", owner, region, tag)``: store into ``owner``'s memory region;
* ``("read", region, tag)``: load from this rank's region; the value must be
  ``tag`` (a read that sees an older or newer write is a race);
* ``("read_peer", owner, region, tag)``: the same for a peer load from
  ``owner``'s memory;
* ``("signal", dst, channel, slot, seq)``: release-store ``seq`` into
  ``dst``'s flag (channel, slot);
* ``("wait", channel, slots, seq)``: block until this rank's flags
  (channel, s) have reached ``seq`` for every s in ``slots``;
* ``("collective", name)``: block until every rank has arrived (an NCCL
  collective such as the gradient-norm all-reduce);
* ``("record", name)`` / ``("wait_event", name)``: a CUDA event recorded on
  one of the rank's streams and waited for on another.

A kernel's stores are visible to a peer once the peer has observed the flag
the kernel released after them, which is what the release/acquire pairs of
the CUDA code give; the interleaving explores how far ranks can drift apart.
``run`` raises on a race or a deadlock.
"""

from __future__ import annotations

import random
from typing import Callable, Dict, Iterator, List, Tuple


class ProtocolError(AssertionError):
    pass


def run(actors: List, seed: int, max_ops: int = 1_000_000) -> Dict[str, int]:
    """``actors``: one operation generator per rank, or (rank, generator)
    pairs when a rank has several CUDA streams (each stream is an actor of
    that rank; they share its memory, flags and events)."""
    rng = random.Random(seed)
    items = [a if isinstance(a, tuple) else (i, a) for i, a in enumerate(actors)]
    rank_of = [rk for rk, _ in items]
    gens = [g for _, g in items]
    n = len(items)
    world = len(set(rank_of))
    mem: Dict[Tuple[int, object], object] = {}
    flags: Dict[Tuple[int, object, int], int] = {}
    events: set = set()
    arrived: Dict[str, set] = {}
    pending: List[object] = [None] * n
    done = [False] * n
    stats = {"ops": 0, "waits_blocked": 0}

    def runnable(i: int) -> bool:
        op = pending[i]
        if op is None:
            return True
        kind, r = op[0], rank_of[i]
        if kind == "wait":
            _, ch, slots, seq = op
            return all(flags.get((r, ch, s), 0) >= seq for s in slots)
        if kind == "collective":
            return len(arrived.get(op[1], ())) == world
        if kind == "wait_event":
            return (r, op[1]) in events
        return True

    for _ in range(max_ops):
        live = [i for i in range(n) if not done[i]]
        if not live:
            return stats
        ready = [i for i in live if runnable(i)]
        if not ready:
            raise ProtocolError("deadlock: " + ", ".join(
                f"rank {rank_of[i]} (actor {i}) at {pending[i]}" for i in live))
        i = rng.choice(ready)
        r = rank_of[i]
        op = pending[i]
        if op is None:
            try:
                op = next(gens[i])
            except StopIteration:
                done[i] = True
                continue
            pending[i] = op
            if op[0] == "collective":
                arrived.setdefault(op[1], set()).add(r)
            if not runnable(i):
                stats["waits_blocked"] += 1
                continue
        pending[i] = None
        stats["ops"] += 1
        kind = op[0]
        if kind == "write":
            _, owner, region, tag = op
            mem[(owner, region)] = tag
        elif kind in ("read", "read_peer"):
            owner, region, tag = (r,) + op[1:] if kind == "read" else op[1:]
            got = mem.get((owner, region))
            if got != tag:
                raise ProtocolError(f"race: rank {r} read {region!r} of rank {owner} = {got!r}, "
                                    f"expected {tag!r}")
        elif kind == "signal":
            _, dst, ch, slot, seq = op
            key = (dst, ch, slot)
            flags[key] = max(flags.get(key, 0), seq)
        elif kind == "record":
            events.add((r, op[1]))
        elif kind in ("wait", "collective", "wait_event"):
            pass
        else:
            raise ValueError(op)
    raise ProtocolError("operation budget exhausted")


def explore(make_ranks: Callable[[], List[Iterator]], schedules: int = 200) -> None:
    """Run the protocol under ``schedules`` random interleavings."""
    for seed in range(schedules):
        run(make_ranks(), seed)
