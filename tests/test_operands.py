"""The operand-discrimination guard, ported from the reference's board test (board_package/tests/test_operands.py).

Identical token rows, or weights constant along the contraction, let a GEMM that drops or confuses a 32-deep block
still produce the right product; the guard rejects such operand pairs before they are used as evidence."""

from __future__ import annotations

import numpy as np
import pytest

from oracle.bf16 import BLOCK_DEPTH, bf16_grid, check_operands_discriminating

TOKENS, DEPTH, COLUMNS = 32, 192, 16


def _varying(depth: int = DEPTH):
    rng = np.random.default_rng(0)
    return (bf16_grid(rng.standard_normal((TOKENS, depth)).astype(np.float32)),
            bf16_grid(rng.standard_normal((depth, COLUMNS)).astype(np.float32)))


def test_varying_operands_are_accepted() -> None:
    check_operands_discriminating(*_varying())


def test_identical_token_rows_are_rejected() -> None:
    _, weights = _varying()
    with pytest.raises(ValueError, match="tokens"):
        check_operands_discriminating(np.tile(np.arange(DEPTH, dtype=np.float32), (TOKENS, 1)), weights)


def test_weights_constant_along_the_contraction_are_rejected() -> None:
    activations, _ = _varying()
    weights = np.broadcast_to(np.arange(1, COLUMNS + 1, dtype=np.float32), (DEPTH, COLUMNS)).astype(np.float32)
    with pytest.raises(ValueError, match="contraction blocks"):
        check_operands_discriminating(activations, weights)


def test_identical_output_columns_are_rejected() -> None:
    activations, _ = _varying()
    weights = np.repeat(np.arange(DEPTH, dtype=np.float32).reshape(DEPTH, 1), COLUMNS, axis=1)
    with pytest.raises(ValueError, match="output columns"):
        check_operands_discriminating(activations, weights)


def test_two_contraction_blocks_are_accepted() -> None:
    check_operands_discriminating(*_varying(depth=2 * BLOCK_DEPTH))
