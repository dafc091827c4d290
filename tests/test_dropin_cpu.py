"""The block driver (tempo_compiler_b200.dropin) on the CPU, over a host model of the runtime whose image kinds run the
oracle's arithmetic (tests/_image_model.py): its layouts, addresses, cache positions and launch order are checked
against the oracle's own GPT-2 chain without a GPU."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import bf16 as ob
from oracle import references as orf
from oracle.model import CachedChain
from tests._image_model import ImageModelRuntime


@pytest.fixture()
def d(monkeypatch):
    from tempo_compiler_b200 import dropin
    model = ImageModelRuntime()
    monkeypatch.setattr(dropin, "rt", model)
    dropin.image_model = model
    return dropin


@pytest.fixture(scope="module")
def small_model():
    from tempo_compiler_b200.weights import GPT2Shape, random_gpt2
    return random_gpt2(17, GPT2Shape(layers=2, vocab=300, positions=128))


def test_block_product_through_the_image_model(d) -> None:
    left, right = ob.build_operands(64, 768, 768, kind="varying", seed=3)
    got = d.block_product(left, right)
    assert orf.relative_error(got, orf.gemm_f64(left, right)) < 5e-3
    assert d.image_model.launches == ["gemm_bias", "gemm_bias"]


def test_prefill_and_steps_follow_the_oracle_chain(d, small_model) -> None:
    layers, shared = small_model
    ids = np.random.default_rng(2).integers(0, 300, size=40)
    observed: list[tuple[int, tuple, tuple]] = []
    net = d.PackedGPT2(layers, shared, capacity=128)
    logits = net.prefill(ids, observe=lambda i, x, y: observed.append((i, x.shape, y.shape)))
    assert observed == [(0, (40, 768), (40, 768)), (1, (40, 768), (40, 768))]
    # 64 padded tokens = 2 blocks: 9 block ops x 2 blocks + 2 cache copies + 1 attention per layer, then the final
    # LayerNorm of the last row's block
    assert len(d.image_model.launches) == 2 * 19 + 1
    # The oracle's exact chain rounds each residual sum once (bias and residual added before one rounding), where the
    # block images round the projection before the add image: a few BF16 steps of difference, far below what a wrong
    # address or cache position would give.
    chain = CachedChain(layers, shared, mode="exact")
    expected = chain.prefill(list(ids))
    assert orf.relative_error(logits, expected) < 2e-2
    token = int(np.argmax(logits))
    for step in range(3):
        before = len(d.image_model.launches)
        logits = net.step(token)
        assert len(d.image_model.launches) - before == 2 * 10 + 1
        expected = chain.step(token)
        assert orf.relative_error(logits, expected) < 2e-2, step
        token = int(np.argmax(logits))
    assert [cache.length for cache in net.caches] == [43, 43]
    net.close()
    assert not d.image_model.live


def test_generate_stops_at_the_cache_capacity(d, small_model) -> None:
    layers, shared = small_model
    net = d.PackedGPT2(layers, shared, capacity=64)
    with pytest.raises(ValueError):
        net.generate(np.arange(60), 8)
    net.close()


def test_packed_rows_round_trip(d) -> None:
    values = ob.bf16_grid(np.random.default_rng(4).standard_normal((70, 48)).astype(np.float32))
    with d.Session() as session:
        tensor = session.rows_in(values)
        assert (tensor.tokens, tensor.blocks) == (96, 3)
        back = session.rows_out(tensor)
        np.testing.assert_array_equal(back[:70], values)
        np.testing.assert_array_equal(back[70:], 0)
        np.testing.assert_array_equal(session.rows_out(tensor, blocks=range(1, 2)), values[32:64])


def test_reference_board_checks_over_the_image_model() -> None:
    """The reference's own driver and board checks (``board_package/board_checks.py:557-576``), unmodified, launching
    this repository's image set through the host model of the runtime: the manifest's kinds and fields and the
    argument slots agree with what the reference's driver stages and passes. Needs the reference's checkout, named by
    TEMPO_REFERENCE_DIR; skipped without it."""
    import importlib
    import os
    import pathlib
    import sys
    root = os.environ.get("TEMPO_REFERENCE_DIR")
    if not root or not (pathlib.Path(root) / "board_package" / "board_checks.py").exists():
        pytest.skip("TEMPO_REFERENCE_DIR does not name the reference project's checkout")
    from tempo_compiler_b200 import images
    from tempo_compiler_b200.weights import random_gpt2
    board = str(pathlib.Path(root) / "board_package")
    names = ("runtime", "gpt2_inference", "board_checks", "bf16", "references", "tokenizer")
    saved = {name: sys.modules.get(name) for name in names}
    model = ImageModelRuntime()
    sys.modules["runtime"] = model.as_module()
    sys.path.insert(0, board)
    try:
        for name in names[1:]:
            sys.modules.pop(name, None)
        gpt2_inference = importlib.import_module("gpt2_inference")
        board_checks = importlib.import_module("board_checks")
        gpt2_inference._IMAGE_DIRECTORY = images.ensure_image_set()
        board_checks.load_gpt2_weights = lambda *_, **__: random_gpt2(7)
        checks = [board_checks.check_halt, board_checks.check_copy_argument, board_checks.check_full_gemm,
                  board_checks.check_elementwise_add, board_checks.check_decode_attention,
                  board_checks.check_layernorm, board_checks.check_kv_cache, board_checks.check_transformer_block,
                  board_checks.check_gpt2_prefill, board_checks.check_gpt2_decode]
        for check in checks:
            check()
    finally:
        sys.path.remove(board)
        for name, value in saved.items():
            if value is None:
                sys.modules.pop(name, None)
            else:
                sys.modules[name] = value
