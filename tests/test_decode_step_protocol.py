"""CPU model check of the persistent decode step's grid barrier (`csrc/decode_step.cu`, `GridBarrier`).

The barrier is a 64-bit arrival counter that only grows. At entry every CTA's thread 0 reads the counter and rounds it
down to a multiple of the grid size (the launch's base); barrier b of the launch (b = 1, 2, ...) is one arrival (a
release add) followed by a poll until the counter reaches base + b x grid. The model runs whole launches back to back,
as a stream runs them (launch L + 1 starts once every CTA of launch L has returned), with the CTAs of a launch starting
at random moments, so a slow CTA may read the counter after fast ones have arrived at the first barrier. It checks
that no CTA leaves a barrier before every CTA has arrived at it, that every launch ends, and that the counter ends at
launches x barriers x grid. It also models the last-CTA pattern that ends the step (every CTA counts itself out after
writing its LM-head partials; the last one alone reduces them and resets the count).

Planted mistakes are caught: a base taken without rounding down (the slow CTA then waits for an arrival that never
comes), a target one barrier short (a CTA leaves before the others arrive), and a launch in which one CTA skips the
last barrier (the next launch's base is then wrong).
"""

from __future__ import annotations

import random

import pytest

from _protocol import Violation, check, run


class Counter:
    def __init__(self) -> None:
        self.value = 0


def cta(counter: Counter, grid: int, index: int, barriers: int, arrived: list[set[int]], passed: list[set[int]],
        no_round: bool = False, short: bool = False, skip_last: bool = False):
    for _ in range(random.Random(index).randrange(4)):
        yield                                            # a CTA starts late
    seen = counter.value
    base = seen if no_round else (seen // grid) * grid
    yield
    for b in range(1, barriers + 1):
        if skip_last and index == 0 and b == barriers:
            return
        arrived[b].add(index)
        counter.value += 1                               # red.release.add: one indivisible step
        yield
        target = base + (b - 1 if short else b) * grid
        while counter.value < target:
            yield
        check(arrived[b] == set(range(grid)), f"CTA {index} left barrier {b} before every CTA arrived")
        passed[b].add(index)
        yield


def launches(grid: int, barriers: int, count: int, seed: int, **mistake) -> None:
    counter = Counter()
    rng = random.Random(seed)
    for launch in range(count):
        arrived = [set() for _ in range(barriers + 1)]
        passed = [set() for _ in range(barriers + 1)]
        roles = {f"cta{i}": cta(counter, grid, i, barriers, arrived, passed, **mistake) for i in range(grid)}
        run(roles, [], rng, limit=200000)
        check(all(passed[b] == set(range(grid)) for b in range(1, barriers + 1)),
              f"launch {launch}: a CTA never passed a barrier")
    check(counter.value == count * barriers * grid, "the counter does not count every arrival")


@pytest.mark.parametrize("seed", range(60))
def test_grid_barrier_holds_across_launches(seed: int) -> None:
    launches(grid=2 + seed % 7, barriers=5, count=3, seed=seed)


def test_base_without_rounding_is_caught() -> None:
    with pytest.raises(Violation):
        for seed in range(200):
            launches(grid=4, barriers=4, count=2, seed=seed, no_round=True)


def test_target_one_barrier_short_is_caught() -> None:
    with pytest.raises(Violation):
        for seed in range(50):
            launches(grid=3, barriers=4, count=1, seed=seed, short=True)


def test_a_skipped_barrier_breaks_the_next_launch() -> None:
    with pytest.raises(Violation):
        for seed in range(50):
            launches(grid=3, barriers=4, count=2, seed=seed, skip_last=True)


def test_last_cta_reduces_only_complete_partials() -> None:
    for seed in range(200):
        rng = random.Random(seed)
        ctas = 2 + seed % 9
        written: set[int] = set()
        state = {"count": 0, "reducer": None}

        def finisher(i):
            written.add(i)                    # its tiles' partials, then the fence
            yield
            old = state["count"]
            state["count"] += 1               # atomicAdd
            yield
            if old == ctas - 1:
                state["count"] = 0
                check(written == set(range(ctas)), "the last CTA reduced before every partial was written")
                state["reducer"] = i

        run({f"cta{i}": finisher(i) for i in range(ctas)}, [], rng)
        assert state["reducer"] is not None and state["count"] == 0
