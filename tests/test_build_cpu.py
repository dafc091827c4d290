"""The in-tree build when several processes find the library stale at once (one rank per GPU, each loading the
library): one builds under the lock, the others wait for it and find the library fresh. Modelled with threads, each
opening the lock file on its own (flock locks belong to the open file, so they exclude each other as processes do),
over a fake compile step; nothing is compiled."""

from __future__ import annotations

import threading
import time

from tempo_compiler_b200 import build


def test_concurrent_builders_build_once(monkeypatch) -> None:
    state = {"stale": True, "builds": 0, "inside": 0, "overlap": False}
    guard = threading.Lock()

    def fake_build(verbose_ptxas: bool):
        with guard:
            state["inside"] += 1
            state["overlap"] |= state["inside"] > 1
        time.sleep(0.2)
        with guard:
            state["builds"] += 1
            state["stale"] = False
            state["inside"] -= 1
        return build.LIBRARY

    monkeypatch.setattr(build, "_stale", lambda: state["stale"])
    monkeypatch.setattr(build, "_build_locked", fake_build)
    results = []
    threads = [threading.Thread(target=lambda: results.append(build.build())) for _ in range(4)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=30)
    assert len(results) == 4 and all(r == build.LIBRARY for r in results)
    assert state["builds"] == 1 and not state["overlap"]


def test_force_rebuilds_even_when_fresh(monkeypatch) -> None:
    calls = []
    monkeypatch.setattr(build, "_stale", lambda: False)
    monkeypatch.setattr(build, "_build_locked", lambda verbose_ptxas: calls.append(1) or build.LIBRARY)
    assert build.build() == build.LIBRARY and calls == []
    assert build.build(force=True) == build.LIBRARY and calls == [1]
