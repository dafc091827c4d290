"""The persistent decode step (tempo_decode_step: one cooperative kernel per step for at most 8 sequences) against the
kernel-per-op decode it replaces: same weights, same prompts, the tokens and every layer's key and value caches
bit for bit, across the row counts its templates cover (1, 2, 4 and 8 rows, and 3 and 5 padded up) and the attention
chunkings the capacity selects (one stretch per (sequence, head) up to eight)."""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    yield
    from tempo_compiler_b200 import ops
    torch.cuda.synchronize()
    assert ops.watchdog() == 0


@pytest.fixture(scope="module")
def model():
    from tempo_compiler_b200.weights import GPT2Shape, random_gpt2
    return random_gpt2(71, GPT2Shape(layers=3, positions=1152))


def _run(layers, shared, ids, capacity, steps, persistent, graph=True):
    from tempo_compiler_b200.engine import Engine
    engine = Engine(layers, shared, batch=ids.shape[0], prompt=ids.shape[1], capacity=capacity,
                    persistent_decode=persistent)
    assert engine.persistent_decode == persistent
    assert Engine(layers, shared, batch=1, prompt=4, capacity=8).persistent_decode is False  # off unless asked
    tokens = engine.generate(ids, steps, graph=graph)
    caches = [(k.clone(), v.clone()) for k, v in zip(engine.k_cache, engine.v_cache)]
    return tokens, caches


@pytest.mark.parametrize("rows,prompt,capacity,steps", [
    (1, 64, 96, 24),      # one row; 12 pairs split in 2 stretches by the small capacity
    (1, 128, 1152, 12),   # one row, 8 stretches per pair
    (2, 32, 384, 16),
    (3, 96, 1152, 10),    # 3 rows on the 4-row template
    (4, 64, 512, 10),
    (5, 32, 256, 8),      # 5 rows on the 8-row template
    (8, 32, 64, 20),      # 96 pairs with one stretch each (the capacity allows no split)
    (8, 256, 1152, 6),
])
def test_persistent_step_matches_the_kernel_per_op_decode(model, rows, prompt, capacity, steps) -> None:
    from tempo_compiler_b200.weights import random_token_ids
    layers, shared = model
    ids = np.stack([random_token_ids(900 + 7 * rows + s, prompt) for s in range(rows)]).astype(np.int32)
    fused, fused_caches = _run(layers, shared, ids, capacity, steps, persistent=True)
    plain, plain_caches = _run(layers, shared, ids, capacity, steps, persistent=False)
    np.testing.assert_array_equal(fused, plain)
    for (kf, vf), (kp, vp) in zip(fused_caches, plain_caches):
        used = prompt + steps
        assert torch.equal(kf[:, :, :used], kp[:, :, :used])
        assert torch.equal(vf[:, :, :used], vp[:, :, :used])


def test_persistent_step_replayed_in_a_graph_equals_eager(model) -> None:
    from tempo_compiler_b200.weights import random_token_ids
    layers, shared = model
    ids = np.stack([random_token_ids(40 + s, 64) for s in range(2)]).astype(np.int32)
    graphed, _ = _run(layers, shared, ids, 96, 20, persistent=True, graph=True)
    eager, _ = _run(layers, shared, ids, 96, 20, persistent=True, graph=False)
    np.testing.assert_array_equal(graphed, eager)


def test_workspace_and_row_limits_are_checked() -> None:
    from tempo_compiler_b200 import ops
    assert ops.decode_step_workspace_bytes(8, 768, 12, 50257) > ops.decode_step_workspace_bytes(1, 768, 12, 50257)
    with pytest.raises(ValueError):
        ops.decode_step_workspace_bytes(9, 768, 12, 50257)
