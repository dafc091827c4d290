"""A model check, on the CPU, of the barrier protocol of the persistent prefill attention kernel.

`tempo_compiler_b200/csrc/attention_prefill.cu` runs four roles per CTA over a sequence of (query tile, head,
sequence) items: one thread loads each item's Q into one of two buffers and the key / value tiles into a ring of
stages (TMA copies, landing in any order), one thread issues the tensor-core work (S = Q K^T into two alternating
TMEM buffers, then O += P V), four softmax warps turn each S into P in place and may rescale O, and the tensor pipe
completes the issued work in order, each `tcgen05.commit` arriving on its mbarrier once everything issued before it
has completed. The waits are
parity waits: `mbarrier.try_wait.parity P` succeeds as soon as the barrier's current phase parity differs from P,
so a wait is only right while the barrier is at most one phase short of the phase it means.

The model below restates that protocol (issue order, the barriers, their arrival counts and the parities each role
waits for) and runs it under many random schedules in which the warps drift apart and the tensor pipe lags. Every
shared-state access is checked against what it needs: an S or P V is issued only once its Q, K or V has landed, a
Q buffer or stage is refilled only after the products reading it completed, a warp reads S_g only once S_g has
completed and before S_{g+2} is issued over it, P V_g is issued only once every warp has written P_g, a rescale touches O only between P V_{g-1}'s
completion and P V_g's issue, and an item's output read sees every P V of the item completed.

The kernel's final O read waits on `o_done`, committed once per item after the item's last P V. An earlier form waited
on the per-tile O barrier with the last tile's parity; a warp that finished the last tile while another was still on
the one before then saw the phase completed two steps back and read O early. The model finds that schedule, so the
check is shown to bite.
"""

from __future__ import annotations

import random

import pytest

from _protocol import Barrier, Pipe, Violation, check, run, wait


def run_schedule(items: list[int], warps: int, seed: int, final_wait: str, stages: int = 4) -> None:
    """Runs one CTA's items (key tiles per item) under a random schedule; raises Violation on a bad access."""
    rng = random.Random(seed)
    tma, tensor = Pipe(rng, ordered=False), Pipe()
    q_full = [Barrier(1, "q_full0"), Barrier(1, "q_full1")]
    q_empty = [Barrier(1, "q_empty0"), Barrier(1, "q_empty1")]
    kv_full = [Barrier(1, f"kv_full{i}") for i in range(stages)]
    kv_empty = [Barrier(1, f"kv_empty{i}") for i in range(stages)]
    s_full = [Barrier(1, "s_full0"), Barrier(1, "s_full1")]
    p_full = [Barrier(warps, "p_full0"), Barrier(warps, "p_full1")]
    o_full, o_done = Barrier(1, "o_full"), Barrier(1, "o_done")
    issued: set[tuple] = set()  # ("S", g) / ("PV", g) issued
    p_written: dict[int, set[int]] = {}
    first_tile = [sum(items[:k]) for k in range(len(items))]
    item_of = [k for k, tiles in enumerate(items) for _ in range(tiles)]
    q_holds: dict[int, int] = {}      # Q buffer -> item loaded into it
    stage_holds: dict[int, int] = {}  # K/V stage -> key tile loaded into it

    def issue(op: tuple, *commits: Barrier) -> None:
        kind, g = op
        if kind == "S":
            check(g < 2 or ("PV", g - 2) in issued, f"S_{g} issued over P_{g - 2} before its P V")
            k = item_of[g]
            check(("Q", k) in tma.done and q_holds.get(k & 1) == k, f"S_{g} issued before item {k}'s Q landed")
            check(("K", g) in tma.done and stage_holds.get(g % stages) == g, f"S_{g} issued before K_{g} landed")
        else:
            check(p_written.get(g, set()) == set(range(warps)), f"P V_{g} issued before every warp wrote P")
            check(("V", g) in tma.done and stage_holds.get(g % stages) == g, f"P V_{g} issued before V_{g} landed")
        issued.add(op)
        tensor.push(("op", op), *(("commit", bar) for bar in commits))

    def producer():
        g = 0
        for k, tiles in enumerate(items):
            yield from wait(lambda k=k: q_empty[k & 1].parity_done(((k >> 1) & 1) ^ 1))
            if k >= 2:
                last = first_tile[k - 2] + items[k - 2] - 1
                check(all(("S", t) in tensor.done for t in range(first_tile[k - 2], last + 1)),
                      f"item {k}'s Q loaded over item {k - 2}'s before its S completed")
            q_full[k & 1].arrive(expect_tx=1)
            q_holds[k & 1] = k
            tma.push(("bytes", q_full[k & 1], 1, ("Q", k)))
            yield
            for _ in range(tiles):
                st, ph = g % stages, (g // stages) & 1
                yield from wait(lambda st=st, ph=ph: kv_empty[st].parity_done(ph ^ 1))
                if g >= stages:
                    check(("S", g - stages) in tensor.done and ("PV", g - stages) in tensor.done,
                          f"tile {g} loaded over tile {g - stages} before its products completed")
                kv_full[st].arrive(expect_tx=2)
                stage_holds[st] = g
                tma.push(("bytes", kv_full[st], 1, ("K", g)), ("bytes", kv_full[st], 1, ("V", g)))
                g += 1
                yield

    def mma():
        g = 0

        def issue_s(g: int):
            yield from wait(lambda: kv_full[g % stages].parity_done((g // stages) & 1))
            issue(("S", g), s_full[g & 1])

        for k, tiles in enumerate(items):
            yield from wait(lambda k=k: q_full[k & 1].parity_done((k >> 1) & 1))
            yield from issue_s(g)
            for j in range(tiles):
                if j + 1 < tiles:
                    yield from issue_s(g + 1)
                else:
                    tensor.push(("commit", q_empty[k & 1]))
                yield from wait(lambda g=g: p_full[g & 1].parity_done((g >> 1) & 1))
                commits = [o_full, o_done] if j + 1 == tiles else [o_full]
                issue(("PV", g), *commits, kv_empty[g % stages])
                g += 1
                yield

    def softmax(w: int):
        g = 0
        for k, tiles in enumerate(items):
            for j in range(tiles):
                yield from wait(lambda g=g: s_full[g & 1].parity_done((g >> 1) & 1))
                check(("S", g) in tensor.done, f"warp {w} read S_{g} before it completed")
                check(("S", g + 2) not in issued, f"warp {w} read S_{g} after S_{g + 2} was issued over it")
                yield
                p_written.setdefault(g, set()).add(w)
                if j >= 1 and rng.random() < 0.3:  # the row maximum grew: rescale O
                    yield from wait(lambda g=g: o_full.parity_done((g - 1) & 1))
                    check(("PV", g - 1) in tensor.done, f"warp {w} rescaled O before P V_{g - 1} completed")
                    check(("PV", g) not in issued, f"warp {w} rescaled O after P V_{g} was issued")
                    yield
                p_full[g & 1].arrive()
                g += 1
                yield
            if final_wait == "o_done":
                yield from wait(lambda k=k: o_done.parity_done(k & 1))
            else:  # the earlier form: the per-tile O barrier with the last tile's parity
                yield from wait(lambda g=g: o_full.parity_done((g - 1) & 1))
            for t in range(first_tile[k], g):
                check(("PV", t) in tensor.done, f"warp {w} read item {k}'s O before P V_{t} completed")
            yield

    run({"producer": producer(), "mma": mma(), **{f"warp{w}": softmax(w) for w in range(warps)}}, [tma, tensor], rng)
    check(all(("PV", g) in tensor.done for g in range(sum(items))), "P V missing")


ITEM_SETS = [[2], [3], [4, 2], [2, 2, 2], [5, 1, 3], [1, 1, 1, 1]]


@pytest.mark.parametrize("items", ITEM_SETS)
def test_final_read_waits_for_every_p_v(items: list[int]) -> None:
    for seed in range(300):
        run_schedule(items, warps=4, seed=seed, final_wait="o_done")


@pytest.mark.parametrize("stages", [2, 3])
def test_shallower_rings_keep_the_protocol(stages: int) -> None:
    """The kernel's ring holds four stages; the protocol does not depend on the depth."""
    for seed in range(200):
        run_schedule([3, 1, 4, 2], warps=4, seed=seed, final_wait="o_done", stages=stages)


def test_the_per_tile_barrier_final_wait_is_caught() -> None:
    """The earlier final wait reads O early under some schedule; the model finds it."""
    found = []
    for seed in range(2000):
        try:
            run_schedule([3, 2], warps=4, seed=seed, final_wait="o_full")
        except Violation as error:
            found.append(str(error))
            break
    assert found and "O before P V" in found[0], found
