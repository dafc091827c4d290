"""CPU model check of the persistent decode step's grid barrier (`csrc/decode_step.cu`, `grid_barrier`).

Every CTA's thread 0 reads the generation word, arrives on the arrival counter, and either (the last to arrive)
resets the counter and then publishes generation + 1, or spins until the generation word moves. The model runs that
protocol for several CTAs through several consecutive barriers under random schedules, each read, atomic and store
one step, and checks that no CTA leaves a barrier before every CTA has arrived at it (so whatever a CTA wrote before
arriving is complete when any CTA passes) and that the counter is back at zero whenever a barrier opens. It also
models the last-CTA pattern that ends the step (every CTA counts itself out after writing its LM-head partials; the
last one alone reduces them). Two planted mistakes are caught: the generation read after the arrival, and the
counter reset after the generation is published.
"""

from __future__ import annotations

import random

import pytest

from _protocol import Violation, check, run


class Memory:
    def __init__(self) -> None:
        self.count = 0
        self.generation = 0


def cta(mem: Memory, ctas: int, index: int, barriers: int, arrived: list[set[int]], passed: list[set[int]],
        read_late: bool = False, reset_late: bool = False):
    for b in range(barriers):
        if not read_late:
            gen = mem.generation
            yield
        arrived[b].add(index)
        old = mem.count
        mem.count += 1                       # atomicAdd: one indivisible step
        yield
        if read_late:
            gen = mem.generation
            yield
        if old == ctas - 1:
            if reset_late:
                mem.generation = gen + 1
                yield
                mem.count = 0
                yield
            else:
                mem.count = 0
                yield
                mem.generation = gen + 1     # st.release after the reset
                yield
        else:
            while mem.generation == gen:
                yield
        check(arrived[b] == set(range(ctas)), f"CTA {index} left barrier {b} before every CTA arrived")
        passed[b].add(index)
        yield


def schedule(ctas: int, barriers: int, seed: int, **mistake) -> None:
    mem = Memory()
    arrived = [set() for _ in range(barriers)]
    passed = [set() for _ in range(barriers)]
    roles = {f"cta{i}": cta(mem, ctas, i, barriers, arrived, passed, **mistake) for i in range(ctas)}
    run(roles, [], random.Random(seed), limit=200000)
    check(all(p == set(range(ctas)) for p in passed), "a CTA never passed a barrier")
    check(mem.count == 0, "the arrival counter is not back at zero")
    check(mem.generation == barriers, "the generation did not advance once per barrier")


@pytest.mark.parametrize("seed", range(60))
def test_grid_barrier_holds_under_random_schedules(seed: int) -> None:
    schedule(ctas=2 + seed % 7, barriers=6, seed=seed)


@pytest.mark.parametrize("seed", range(40))
def test_reading_the_generation_after_arriving_is_caught(seed: int) -> None:
    with pytest.raises(Violation):
        for extra in range(10):
            schedule(ctas=3 + seed % 4, barriers=5, seed=seed * 31 + extra, read_late=True)


def test_resetting_the_counter_after_publishing_is_caught() -> None:
    with pytest.raises(Violation):
        for seed in range(400):
            schedule(ctas=4, barriers=8, seed=seed, reset_late=True)


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
