"""A small model of the synchronisation the tcgen05 kernels use, for CPU model checks of their protocols.

* `Barrier` is an mbarrier: a phase completes once its expected arrivals have been made and its transaction count
  (bytes announced by `arrive.expect_tx`, retired by TMA copies) is back to zero; byte completions may come before
  the announcement, as they may on the hardware. `parity_done(P)` is `mbarrier.try_wait.parity P`: true as soon as
  the current phase's parity differs from P.
* `Pipe` is a tensor pipe (or a TMA engine): work is completed in issue order, and a commit placed after some work
  arrives on its barrier once that work has completed (`tcgen05.commit`).
* `run` interleaves role generators and pipes at random: a role yields whenever it may be overtaken, and spins by
  yielding until its wait succeeds.
"""

from __future__ import annotations

import random
from typing import Callable, Iterator


class Violation(AssertionError):
    """A role touched shared state its protocol had not yet made safe."""


def check(condition: bool, what: str) -> None:
    if not condition:
        raise Violation(what)


class Barrier:
    def __init__(self, count: int, name: str = "") -> None:
        self.count, self.pending, self.tx, self.phase, self.name = count, 0, 0, 0, name

    def _maybe_complete(self) -> None:
        if self.pending == self.count and self.tx == 0:
            self.pending = 0
            self.phase += 1

    def arrive(self, expect_tx: int = 0) -> None:
        check(self.pending < self.count, f"{self.name}: more arrivals than expected in one phase")
        self.tx += expect_tx
        self.pending += 1
        self._maybe_complete()

    def complete_tx(self, nbytes: int) -> None:
        self.tx -= nbytes
        self._maybe_complete()

    def parity_done(self, parity: int) -> bool:
        return (self.phase & 1) != parity


class Pipe:
    """Asynchronous work: ("op", key) items mark `key` done; ("commit", barrier) items arrive;
    ("bytes", barrier, n, key) items retire n bytes on a barrier and mark `key` landed. A tensor pipe completes its
    items in order; TMA copies (ordered=False) complete in any order."""

    def __init__(self, rng: random.Random | None = None, ordered: bool = True) -> None:
        self.queue: list[tuple] = []
        self.done: set = set()
        self.rng, self.ordered = rng, ordered

    def push(self, *items: tuple) -> None:
        self.queue.extend(items)

    def step(self) -> None:
        index = 0 if self.ordered else self.rng.randrange(len(self.queue))
        item = self.queue.pop(index)
        if item[0] == "op":
            self.done.add(item[1])
        elif item[0] == "commit":
            item[1].arrive()
        else:
            _, bar, nbytes, key = item
            self.done.add(key)
            bar.complete_tx(nbytes)


def run(roles: dict[str, Iterator], pipes: list[Pipe], rng: random.Random, limit: int = 400000) -> None:
    live = dict(roles)
    for _ in range(limit):
        actors: list = list(live)
        actors += [pipe for pipe in pipes if pipe.queue for _ in range(2)]
        if not actors:
            return
        actor = rng.choice(actors)
        if isinstance(actor, Pipe):
            actor.step()
            continue
        try:
            next(live[actor])
        except StopIteration:
            del live[actor]
    raise Violation("the schedule did not finish (a wait that never succeeds)")


def wait(predicate: Callable[[], bool]) -> Iterator[None]:
    """Spin until `predicate` holds (use as `yield from wait(...)`)."""
    while not predicate():
        yield
