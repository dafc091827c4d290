"""The board checks' criteria catch planted mistakes (the counterpart of the reference's emulator mutation test,
tests/test_emulator.py:28-60, which flips vadd to vsub in the add image and expects the check to fail).

Each case computes a result through the oracle with one mistake planted on the CPU -- never on the device -- and
applies the same criterion the GPU checks apply to the device result (tests/test_dropin_gpu.py, following
board_package/board_checks.py): exactness for add, bias add, the structured GEMM and the KV cache; the relative
bounds of 1 % (GEMM), 5 % (decode attention, block) and 2 % (LayerNorm). A criterion that let these through would
not discriminate the device results either.
"""

from __future__ import annotations

import numpy as np

from oracle import bf16 as ob
from oracle import references as orf


def _rows(seed: int, shape, scale: float = 1.0):
    rng = np.random.default_rng(seed)
    return ob.bf16_grid((rng.standard_normal(shape) * scale).astype(np.float32))


def test_add_check_rejects_a_subtraction() -> None:
    """vadd -> vsub, as the reference's mutation test plants it."""
    left, right = _rows(53, (32, 768)), _rows(54, (32, 768))
    expected = ob.bf16_grid(left + right)
    assert np.array_equal(ob.bf16_grid(left + right), expected)
    assert not np.array_equal(ob.bf16_grid(left - right), expected)


def test_bias_add_check_rejects_a_bias_of_the_wrong_row() -> None:
    left, bias = _rows(55, (32, 768)), _rows(56, (768,))
    expected = ob.bf16_grid(left + bias)
    assert not np.array_equal(ob.bf16_grid(left + np.roll(bias, 1)), expected)


def test_structured_gemm_check_rejects_a_dropped_contraction_block() -> None:
    """The structured operands make every 16-deep block of the contraction visible in the exact product."""
    left, right = ob.build_operands(32, 768, 3072, kind="structured", seed=0)
    expected = left @ right
    dropped = left[:, 16:] @ right[16:]
    assert not np.array_equal(dropped, expected)


def test_varying_gemm_bound_rejects_a_dropped_block_and_a_mis_tiled_operand() -> None:
    left, right = ob.build_operands(32, 768, 3072, kind="varying", seed=0)
    exact = orf.gemm_f64(left, right)
    assert orf.relative_error(orf.gemm_f64(left, right), exact) < 0.01
    # one 16-deep block of the 768-deep contraction lost
    assert orf.relative_error(orf.gemm_f64(left[:, 16:], right[16:]), exact) > 0.01
    # the weights' 16-column tiles read in the wrong order
    mis_tiled = np.ascontiguousarray(right.reshape(768, 16, 192).transpose(0, 2, 1).reshape(768, 3072))
    assert orf.relative_error(orf.gemm_f64(left, mis_tiled), exact) > 0.01


def test_decode_attention_bound_rejects_the_wrong_head_and_a_missing_scale() -> None:
    query, keys, values = _rows(19, (1, 768)), _rows(20, (49, 768)), _rows(21, (49, 768))

    def heads(q, k, v):
        return np.concatenate([orf.attention_f64(q[:, h * 64:(h + 1) * 64], k[:, h * 64:(h + 1) * 64],
                                                 v[:, h * 64:(h + 1) * 64]) for h in range(12)], axis=1)

    expected = heads(query / 8.0, keys, values)
    assert orf.relative_error(heads(query / 8.0, keys, values), expected) < 0.05
    assert orf.relative_error(heads(query / 8.0, keys, np.roll(values, 64, axis=1)), expected) > 0.05
    assert orf.relative_error(heads(query * 2.0, keys, values), expected) > 0.05


def test_layernorm_bound_rejects_swapped_gamma_and_beta() -> None:
    values = _rows(0, (32, 768), 2.0)
    rng = np.random.default_rng(1)
    gamma = ob.bf16_grid((1.0 + 0.1 * rng.standard_normal(768)).astype(np.float32))
    beta = ob.bf16_grid((0.1 * rng.standard_normal(768)).astype(np.float32))
    expected = orf.layernorm_device(values, gamma, beta)
    assert orf.relative_error(orf.layernorm_device(values, beta, gamma), expected) > 0.02


def test_block_bound_rejects_a_dropped_residual() -> None:
    rng = np.random.default_rng(2)

    def normal(shape, scale):
        return ob.bf16_grid((rng.standard_normal(shape) * scale).astype(np.float32))

    model = 768
    ones = ob.bf16_grid(np.ones(model, dtype=np.float32))
    weights = {"ln_1.g": ones, "ln_1.b": normal((model,), 0.02), "attn.qkv.w": normal((model, 3 * model), 0.02),
               "attn.qkv.b": normal((3 * model,), 0.02), "attn.proj.w": normal((model, model), 0.02),
               "attn.proj.b": normal((model,), 0.02), "ln_2.g": ones.copy(), "ln_2.b": normal((model,), 0.02),
               "mlp.fc.w": normal((model, 4 * model), 0.02), "mlp.fc.b": normal((4 * model,), 0.02),
               "mlp.proj.w": normal((4 * model, model), 0.02), "mlp.proj.b": normal((model,), 0.02)}
    hidden = _rows(3, (32, model), 0.5)
    expected = orf.block_device(hidden, weights)
    # the block's output without its input added back: the residual stream is lost
    assert orf.relative_error(expected - hidden, expected) > 0.05


def test_kv_cache_check_rejects_an_off_by_one_append() -> None:
    prefill, step = _rows(31, (64, 3 * 768)), _rows(32, (32, 3 * 768))
    expected = np.concatenate([prefill[:, 768:], step[:1, 768:]])
    off_by_one = np.concatenate([prefill[:, 768:], step[1:2, 768:]])
    assert not np.array_equal(off_by_one, expected)
