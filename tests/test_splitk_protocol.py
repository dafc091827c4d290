"""CPU model check of the split-K GEMM's reduction protocol (`csrc/gemm.cu`, `gemm_splitk_kernel`).

A cluster of SPLITS CTAs shares one output tile; CTA r owns rows [r * 128 / SPLITS, (r + 1) * 128 / SPLITS). Thread 0
of every CTA initialises its `red_full` mbarrier and announces, with its single arrival, the bytes the other CTAs will
send it; every thread arrives on the cluster barrier. Each of the 8 epilogue warps (TMEM lane quarter q, column half
h) waits for the cluster, writes the rows it owns straight into its own reduction buffer, stages the others in the
operand ring and issues one bulk copy per remote owner, which lands after a random latency, in any order,
completing its bytes on the owner's `red_full`. The warps of a CTA then meet on a named barrier (their own rows are
in place), wait for `red_full`, read every partial of their rows and store the outputs; a final cluster barrier
precedes the exit.

Each run interleaves the CTAs' warps and the copy engine at random and checks: a copy is issued only once its
destination CTA has started, it reads a staging tile whose CTA has not exited and writes into a CTA that has not
exited, and an owner reads its rows only when all SPLITS partials of them are there. Planted mistakes are caught: no
wait for `red_full`, a byte announcement one piece short, and no final cluster barrier.
"""

from __future__ import annotations

import random

import pytest

from _protocol import Barrier, Violation, check, run, wait


def splitk(splits: int, seed: int, wait_red: bool = True, short: bool = False, final_barrier: bool = True) -> None:
    rng = random.Random(seed)
    rows_per = 128 // splits
    piece_rows = min(rows_per, 32)
    remote_units = (splits - 1) * rows_per * 2           # bytes counted as (row, half) units
    red_full = [Barrier(1, f"red_full{r}") for r in range(splits)]
    started: set[int] = set()
    exited: set[int] = set()
    at_final: set[int] = set()
    present = [set() for _ in range(splits)]              # owner -> {(src, row, half)} in its buffer
    staged: dict[tuple, bool] = {}
    in_flight: list[tuple] = []
    local_bar = [0] * splits
    warps_done = [0] * splits

    def cta(rank: int):
        red_full[rank].arrive(expect_tx=remote_units - (piece_rows if short else 0))
        started.add(rank)
        yield
        epilogue = [warp(rank, w) for w in range(2, 10)]
        live = list(epilogue)
        while live:                                      # the CTA's epilogue warps, interleaved
            g = rng.choice(live)
            try:
                next(g)
            except StopIteration:
                live.remove(g)
            yield
        if final_barrier:
            at_final.add(rank)
            yield from wait(lambda: len(at_final) == splits)
        exited.add(rank)

    def warp(rank: int, w: int):
        quarter, half = w & 3, (w - 2) >> 2
        yield from wait(lambda: len(started) == splits)  # the cluster barrier at entry
        rows = [32 * quarter + lane for lane in range(32)]
        for row in rows:
            owner = row // rows_per
            if owner == rank:
                present[rank].add((rank, row, half))
            else:
                staged[(rank, row, half)] = True
            yield
        for first in range(0, 32, piece_rows):
            owner = rows[first] // rows_per
            if owner != rank:
                check(owner in started, "a copy into a CTA that has not started")
                in_flight.append((rank, owner, tuple(rows[first:first + piece_rows]), half, rng.randrange(400)))
        local_bar[rank] += 1
        yield from wait(lambda: local_bar[rank] == 8)
        if wait_red:
            yield from wait(lambda: red_full[rank].parity_done(0))
        mine = range(rank * rows_per, (rank + 1) * rows_per)
        for row in mine:
            for src in range(splits):
                check((src, row, half) in present[rank], f"CTA {rank} read row {row} before CTA {src}'s partial landed")
        warps_done[rank] += 1

    def copy_engine():
        # every copy takes a random number of the engine's turns (its latency) and lands in any order
        while len(exited) < splits:
            for i in range(len(in_flight)):
                src, owner, rows, half, left = in_flight[i]
                in_flight[i] = (src, owner, rows, half, left - 1)
            ready = [i for i, c in enumerate(in_flight) if c[4] <= 0]
            if ready:
                src, owner, rows, half, _ = in_flight.pop(rng.choice(ready))
                check(src not in exited, f"a copy read the staging of CTA {src} after it exited")
                check(owner not in exited, f"a copy wrote into CTA {owner} after it exited")
                for row in rows:
                    check(staged.get((src, row, half), False), "a copy of rows that were never staged")
                    present[owner].add((src, row, half))
                red_full[owner].complete_tx(len(rows))
            yield

    roles = {f"cta{r}": cta(r) for r in range(splits)}
    roles["copies"] = copy_engine()
    run(roles, [], rng, limit=400000)
    check(all(d == 8 for d in warps_done), "an owner never finished")
    check(not in_flight, "copies left in flight")


@pytest.mark.parametrize("splits", [2, 4, 8])
@pytest.mark.parametrize("seed", range(12))
def test_splitk_reduction_protocol(splits: int, seed: int) -> None:
    splitk(splits, seed)


@pytest.mark.parametrize("splits", [2, 4, 8])
def test_reading_without_waiting_for_the_copies_is_caught(splits: int) -> None:
    with pytest.raises(Violation):
        for seed in range(40):
            splitk(splits, seed, wait_red=False)


@pytest.mark.parametrize("splits", [2, 8])
def test_a_short_byte_announcement_is_caught(splits: int) -> None:
    with pytest.raises(Violation):
        for seed in range(40):
            splitk(splits, seed, short=True)


def test_leaving_without_the_final_cluster_barrier_is_caught() -> None:
    with pytest.raises(Violation):
        for seed in range(200):
            splitk(4, seed, final_barrier=False)
