"""Parity figures the GPU tests measure, appended as JSON lines to the file named by TEMPO_PARITY_LOG (when set), so
a run can keep them beside its pass/fail record."""

from __future__ import annotations

import json
import os


def record(name: str, **fields) -> None:
    path = os.environ.get("TEMPO_PARITY_LOG")
    if not path:
        return
    with open(path, "a") as f:
        f.write(json.dumps({"test": name, **fields}) + "\n")
