"""CPU model checks of the barrier protocols of the two persistent tcgen05 GEMM kernels (`csrc/gemm.cu`).

`gemm_rowmajor_kernel`: one producer thread fills a ring of operand stages (the first tile's weight halves are issued
before the dependent-launch wait, their activation halves after it), one MMA thread consumes the stages into one of
two TMEM accumulators and commits each stage and each finished accumulator, and the epilogue warps drain an
accumulator and release it. With a folded LayerNorm (one tile per CTA) the epilogue warps also read the first tile's
stages for the rows' statistics, and a stage is free only once the MMA and every warp are done with it.

`gemm_pair_kernel`: two CTAs on two SMs. Each CTA's producer copies its halves into its own stages, completing on the
leader's full barrier, whose bytes the leader alone announces; the leader's MMA thread consumes both CTAs' stages and
commits the stage and accumulator barriers of both CTAs; every epilogue warp of either CTA releases the accumulator on
the leader's barrier.

Each run interleaves the roles at random, with TMA copies landing in any order and the tensor pipe lagging, and checks
every access against what it needs: an MMA reads only landed operands, a copy overwrites a stage only after every
reader of its previous contents is done, an epilogue reads an accumulator only after its tile's MMAs completed, and an
MMA overwrites an accumulator only after every epilogue warp has drained it.
"""

from __future__ import annotations

import random

import pytest

from _protocol import Barrier, Pipe, Violation, check, run, wait


def rowmajor(tiles: int, kblocks: int, stages: int, warps: int, ln: bool, seed: int,
             ln_release: bool = True) -> None:
    rng = random.Random(seed)
    tma, tensor = Pipe(rng, ordered=False), Pipe()
    full = [Barrier(1, f"full{s}") for s in range(stages)]
    empty = [Barrier(1 + warps if ln and ln_release else 1, f"empty{s}") for s in range(stages)]
    acc_full = [Barrier(1, "acc_full0"), Barrier(1, "acc_full1")]
    acc_empty = [Barrier(warps, "acc_empty0"), Barrier(warps, "acc_empty1")]
    final = Barrier(1, "final")
    occupant: dict[int, tuple] = {}          # stage -> (tile, kb) last loaded
    ln_read: dict[tuple, set[int]] = {}       # (tile, kb) -> warps that read it for the statistics
    drained: dict[int, set[int]] = {}        # tile -> warps that drained its accumulator
    units = [(t, kb) for t in range(tiles) for kb in range(kblocks)]

    def load(stage: int, unit: tuple, half: str) -> None:
        if half == "B" and stage in occupant:
            previous = occupant[stage]
            check(("mma",) + previous in tensor.done, f"stage {stage} refilled before the MMA read {previous}")
            if ln and previous[0] == 0:
                check(ln_read.get(previous, set()) == set(range(warps)), f"stage {stage} refilled before the "
                                                                       f"statistics read {previous}")
        if half == "B":
            occupant[stage] = unit
        tma.push(("bytes", full[stage], 1, (half,) + unit))

    def producer():
        early = min(kblocks, stages)
        for kb in range(early):  # the first tile's weights, before the dependent-launch wait
            full[kb].arrive(expect_tx=2)
            load(kb, (0, kb), "B")
            yield
        stage = phase = 0
        used: dict[int, int] = {}
        for t in range(tiles):
            for kb in range(kblocks):
                if not (t == 0 and kb < early):
                    yield from wait(lambda s=stage, p=phase: empty[s].parity_done(p ^ 1))
                    full[stage].arrive(expect_tx=2)
                    load(stage, (t, kb), "B")
                load(stage, (t, kb), "A")
                used[stage] = phase
                stage, phase = (0, phase ^ 1) if stage + 1 == stages else (stage + 1, phase)
                yield
        for s, p in used.items():  # every copy landed before exit
            yield from wait(lambda s=s, p=p: full[s].parity_done(p))

    def mma():
        stage = phase = acc = acc_phase = 0
        for t in range(tiles):
            yield from wait(lambda a=acc, p=acc_phase: acc_empty[a].parity_done(p ^ 1))
            if t >= 2:
                check(drained.get(t - 2, set()) == set(range(warps)), f"tile {t} overwrote an undrained accumulator")
            for kb in range(kblocks):
                yield from wait(lambda s=stage, p=phase: full[s].parity_done(p))
                check(("A", t, kb) in tma.done and ("B", t, kb) in tma.done, f"MMA read ({t}, {kb}) before it landed")
                check(occupant[stage] == (t, kb), f"stage {stage} holds {occupant[stage]}, not ({t}, {kb})")
                tensor.push(("op", ("mma", t, kb)), ("commit", empty[stage]))
                stage, phase = (0, phase ^ 1) if stage + 1 == stages else (stage + 1, phase)
                yield
            tensor.push(("commit", acc_full[acc]))
            acc, acc_phase = (0, acc_phase ^ 1) if acc == 1 else (1, acc_phase)
        tensor.push(("commit", final))
        yield from wait(lambda: final.parity_done(0))

    def epilogue(w: int):
        if ln:  # the first tile's statistics from its stages as they stream in
            stage = phase = 0
            for kb in range(kblocks):
                yield from wait(lambda s=stage, p=phase: full[s].parity_done(p))
                check(("A", 0, kb) in tma.done, f"warp {w} read the statistics of (0, {kb}) before it landed")
                ln_read.setdefault((0, kb), set()).add(w)
                if ln_release:
                    empty[stage].arrive()
                stage, phase = (0, phase ^ 1) if stage + 1 == stages else (stage + 1, phase)
                yield
        acc = acc_phase = 0
        for t in range(tiles):
            yield from wait(lambda a=acc, p=acc_phase: acc_full[a].parity_done(p))
            check(("mma", t, kblocks - 1) in tensor.done, f"warp {w} drained tile {t} before its MMAs completed")
            yield
            drained.setdefault(t, set()).add(w)
            acc_empty[acc].arrive()
            acc, acc_phase = (0, acc_phase ^ 1) if acc == 1 else (1, acc_phase)
            yield

    roles = {"producer": producer(), "mma": mma(), **{f"epi{w}": epilogue(w) for w in range(warps)}}
    run(roles, [tma, tensor], rng)
    check(all(("mma",) + u in tensor.done for u in units), "an MMA never ran")


def pair(tiles: int, kblocks: int, stages: int, warps: int, seed: int, announced: int = 4) -> None:
    rng = random.Random(seed)
    tma, tensor = Pipe(rng, ordered=False), Pipe()
    ctas = range(2)
    full = [[Barrier(1, f"full{s}@{r}") for s in range(stages)] for r in ctas]  # only the leader's is used
    empty = [[Barrier(1, f"empty{s}@{r}") for s in range(stages)] for r in ctas]
    acc_full = [[Barrier(1, f"acc_full{a}@{r}") for a in range(2)] for r in ctas]
    acc_empty = [Barrier(2 * warps, f"acc_empty{a}@leader") for a in range(2)]
    final = Barrier(1, "final")
    occupant: dict[tuple, tuple] = {}  # (cta, stage) -> (tile, kb)
    drained: dict[int, set] = {}

    def producer(r: int):
        stage = phase = 0
        used: dict[int, int] = {}
        for t in range(tiles):
            for kb in range(kblocks):
                yield from wait(lambda s=stage, p=phase: empty[r][s].parity_done(p ^ 1))
                if (r, stage) in occupant:
                    previous = occupant[(r, stage)]
                    check(("mma",) + previous in tensor.done, f"CTA {r} refilled stage {stage} before the MMA read "
                                                             f"{previous}")
                if r == 0:
                    full[0][stage].arrive(expect_tx=announced)  # both CTAs' A and B halves: 4
                occupant[(r, stage)] = (t, kb)
                yield
                tma.push(("bytes", full[0][stage], 1, ("A", r, t, kb)))
                tma.push(("bytes", full[0][stage], 1, ("B", r, t, kb)))
                used[stage] = phase
                stage, phase = (0, phase ^ 1) if stage + 1 == stages else (stage + 1, phase)
                yield
        for s, p in used.items():  # the copies landed once the MMA released the stage's last use
            yield from wait(lambda s=s, p=p: empty[r][s].parity_done(p))

    def mma():
        stage = phase = acc = acc_phase = 0
        for t in range(tiles):
            yield from wait(lambda a=acc, p=acc_phase: acc_empty[a].parity_done(p ^ 1))
            if t >= 2:
                check(drained.get(t - 2, set()) == {(r, w) for r in ctas for w in range(warps)},
                      f"tile {t} overwrote an undrained accumulator")
            for kb in range(kblocks):
                yield from wait(lambda s=stage, p=phase: full[0][s].parity_done(p))
                for r in ctas:
                    check(("A", r, t, kb) in tma.done and ("B", r, t, kb) in tma.done,
                          f"MMA read ({t}, {kb}) before CTA {r}'s halves landed")
                    check(occupant[(r, stage)] == (t, kb), f"CTA {r} stage {stage} holds another k-block")
                tensor.push(("op", ("mma", t, kb)), ("commit", empty[0][stage]), ("commit", empty[1][stage]))
                stage, phase = (0, phase ^ 1) if stage + 1 == stages else (stage + 1, phase)
                yield
            tensor.push(("commit", acc_full[0][acc]), ("commit", acc_full[1][acc]))
            acc, acc_phase = (0, acc_phase ^ 1) if acc == 1 else (1, acc_phase)
        tensor.push(("commit", final))
        yield from wait(lambda: final.parity_done(0))

    def epilogue(r: int, w: int):
        acc = acc_phase = 0
        for t in range(tiles):
            yield from wait(lambda a=acc, p=acc_phase: acc_full[r][a].parity_done(p))
            check(("mma", t, kblocks - 1) in tensor.done, f"CTA {r} warp {w} drained tile {t} early")
            yield
            drained.setdefault(t, set()).add((r, w))
            acc_empty[acc].arrive()
            acc, acc_phase = (0, acc_phase ^ 1) if acc == 1 else (1, acc_phase)
            yield

    roles = {"producer0": producer(0), "producer1": producer(1), "mma": mma(),
             **{f"epi{r}.{w}": epilogue(r, w) for r in ctas for w in range(warps)}}
    run(roles, [tma, tensor], rng)


SHAPES = [(1, 1, 2), (1, 5, 3), (3, 2, 2), (4, 3, 5), (5, 12, 4), (2, 7, 5)]  # (tiles, k-blocks, stages)


@pytest.mark.parametrize(("tiles", "kblocks", "stages"), SHAPES)
def test_rowmajor_gemm_protocol(tiles: int, kblocks: int, stages: int) -> None:
    for seed in range(60):
        rowmajor(tiles, kblocks, stages, warps=4, ln=False, seed=seed)


@pytest.mark.parametrize(("kblocks", "stages"), [(1, 3), (4, 4), (12, 5), (3, 5)])
def test_rowmajor_gemm_with_folded_layernorm_protocol(kblocks: int, stages: int) -> None:
    for seed in range(60):
        rowmajor(1, kblocks, stages, warps=4, ln=True, seed=seed)  # one tile per CTA, as the host guarantees


@pytest.mark.parametrize(("tiles", "kblocks", "stages"), SHAPES)
def test_pair_gemm_protocol(tiles: int, kblocks: int, stages: int) -> None:
    for seed in range(60):
        pair(tiles, kblocks, stages, warps=3, seed=seed)


def test_sixteen_epilogue_warps() -> None:
    for seed in range(10):
        rowmajor(3, 4, 4, warps=16, ln=False, seed=seed)
        pair(3, 4, 4, warps=16, seed=seed)


def test_a_missing_release_is_caught() -> None:
    """The checker bites: with the stage barriers counting the MMA alone (the folded LayerNorm's warps not
    releasing the stages they read, a planted mistake), a refill overtakes a statistics read under some schedule."""
    caught = []
    for seed in range(300):
        try:
            rowmajor(1, 6, 2, warps=4, ln=True, seed=seed, ln_release=False)
        except Violation as error:
            caught.append(str(error))
            break
    assert caught and "statistics" in caught[0], caught


def test_a_short_byte_announcement_is_caught() -> None:
    """The checker bites on the pair kernel too: a leader announcing only one CTA's worth of bytes (a planted
    mistake) lets its MMA read a stage before both CTAs' halves have landed under some schedule."""
    caught = []
    for seed in range(300):
        try:
            pair(2, 4, 3, warps=2, seed=seed, announced=2)
        except Violation as error:
            caught.append(str(error))
            break
    assert caught and "halves landed" in caught[0], caught
