"""The reference's own drivers and board checks on the B200: ``board_package/board_checks.py`` imported with
``tempo_compiler_b200.runtime`` installed as its ``runtime`` module (the seam ``tools/emulators/emulate_board_checks.py:
21-23`` uses), and its ten checks run (``board_checks.py:557-576``) against this repository's image set.

It needs the reference project's checkout, named by the environment variable TEMPO_REFERENCE_DIR, and a GPU; it is
skipped without either. The GPT-2 checks read the reference's exported weights file when the checkout holds one, and
otherwise seeded random weights in the same naming (tempo_compiler_b200.weights.random_gpt2)."""

from __future__ import annotations

import os
import pathlib
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = pathlib.Path(__file__).resolve().parents[1]

_SCRIPT = r"""
import pathlib, sys
root, reference = pathlib.Path(sys.argv[1]), pathlib.Path(sys.argv[2])
sys.path.insert(0, str(root))
import tempo_compiler_b200.runtime as b200_runtime
from tempo_compiler_b200 import images
sys.modules["runtime"] = b200_runtime
sys.path.insert(0, str(reference / "board_package"))
import board_checks, gpt2_inference
gpt2_inference._IMAGE_DIRECTORY = images.ensure_image_set()
checks = [("Halt", board_checks.check_halt), ("COPY round trip", board_checks.check_copy_argument),
          ("Full GEMM", board_checks.check_full_gemm), ("Elementwise add", board_checks.check_elementwise_add),
          ("Decode attention", board_checks.check_decode_attention), ("LayerNorm", board_checks.check_layernorm),
          ("KV cache", board_checks.check_kv_cache), ("Transformer block", board_checks.check_transformer_block)]
if not (reference / "board_package" / "weights" / "gpt2_weights.npz").exists():
    from tempo_compiler_b200.weights import random_gpt2
    board_checks.load_gpt2_weights = lambda *_, **__: random_gpt2(7)
checks += [("GPT-2 prefill", board_checks.check_gpt2_prefill), ("GPT-2 decode", board_checks.check_gpt2_decode)]
results = [board_checks.run_check(name=name, check=check) for name, check in checks]
sys.exit(0 if all(results) else 1)
"""


def test_reference_board_checks_pass_over_the_b200_runtime() -> None:
    reference = os.environ.get("TEMPO_REFERENCE_DIR")
    if not reference or not (pathlib.Path(reference) / "board_package" / "board_checks.py").exists():
        pytest.skip("TEMPO_REFERENCE_DIR does not name the reference project's checkout")
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    result = subprocess.run([sys.executable, "-c", _SCRIPT, str(ROOT), reference], capture_output=True, text=True,
                            timeout=1800)
    assert result.returncode == 0, result.stdout[-4000:] + result.stderr[-4000:]
