"""The KV-cached host chain equals the reference's full recompute, so it can stand in for it on long decodes."""

from __future__ import annotations

import numpy as np
import pytest

from oracle.model import CachedChain, forward_logits
from tempo_compiler_b200.weights import GPT2Shape, random_gpt2


@pytest.mark.parametrize("mode", ["device", "exact"])
def test_cached_decode_equals_full_recompute(mode: str) -> None:
    layers, shared = random_gpt2(11, GPT2Shape(layers=2))
    prompt = [464, 3139, 286, 4881, 318, 17, 9]
    chain = CachedChain(layers, shared, mode=mode)
    logits = chain.prefill(prompt)
    sequence = list(prompt)
    for _ in range(3):
        full = forward_logits(sequence, layers, shared, mode=mode)
        np.testing.assert_allclose(logits, full, rtol=0, atol=1e-5 if mode == "device" else 1e-9)
        assert int(np.argmax(logits)) == int(np.argmax(full))
        token = int(np.argmax(logits))
        sequence.append(token)
        logits = chain.step(token)
    assert chain.length == len(sequence)


def test_greedy_generate_reports_margins() -> None:
    layers, shared = random_gpt2(12, GPT2Shape(layers=1))
    tokens, margins = CachedChain(layers, shared, mode="exact").generate([1, 2, 3, 4], new_tokens=3)
    assert len(tokens) == 3 and len(margins) == 3 and min(margins) >= 0.0
