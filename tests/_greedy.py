"""Greedy-token parity of a generated sequence against the oracle's GPT-2 chain, teacher-forced on that sequence.

At every step the oracle (oracle.model.CachedChain) sees the same prefix as the generator did, so each generated token
is judged on its own: in exact mode (float64 ops, BF16 storage, the arithmetic the B200 kernels carry out) the token
must be the oracle's best wherever the best clears the runner-up by more than the tie margin, and within the margin
of the best otherwise; in device mode (the reference NPU's BF16 accumulation and table GELU) agreement is measured,
and the first step where the reference's semantics would pick another token is the first divergence a free-running
comparison would show.
"""

from __future__ import annotations

import numpy as np

from oracle.model import CachedChain

TIE_MARGIN = 0.02


def teacher_forced(layers, shared, prompt, tokens, *, margin: float = TIE_MARGIN) -> dict:
    """Checks every token against the exact oracle; returns the number of near-ties and the smallest top-2 gap.

    Raises:
        AssertionError: At the first step whose token the oracle ranks more than `margin` below its best, or that is
            not the oracle's best although the best clears the runner-up by more than `margin`.
    """
    chain = CachedChain(layers, shared, mode="exact")
    logits = chain.prefill([int(t) for t in prompt])
    ties, smallest = 0, float("inf")
    exact_logits = []
    for step, token in enumerate(tokens):
        token = int(token)
        best = int(np.argmax(logits))
        top = np.sort(logits)[-2:]
        gap = float(top[1] - top[0])
        smallest = min(smallest, gap)
        exact_logits.append(logits)
        if gap > margin:
            assert token == best, f"step {step}: token {token}, oracle's best {best} clears the runner-up by {gap:.4f}"
        else:
            ties += 1
            assert logits[best] - logits[token] <= margin, f"step {step}: {logits[best] - logits[token]:.4f} below"
        if step + 1 < len(tokens):
            logits = chain.step(token)
    return {"steps": len(tokens), "near_ties": ties, "smallest_gap": smallest, "exact_logits": exact_logits}


def device_agreement(layers, shared, prompt, tokens, exact_logits=None) -> dict:
    """Teacher-forced agreement with the reference's device semantics (BF16 accumulation, table GELU).

    Returns the steps where the device chain's best token equals the generated one, the first step where it does
    not (None if never: the free-running sequences would be identical), and at each disagreement the device chain's
    gap between its own pick and the generated token, the exact chain's gap the other way, and the RMS and largest
    difference between the two chains' logits at that step.
    """
    chain = CachedChain(layers, shared, mode="device")
    logits = chain.prefill([int(t) for t in prompt])
    agree, disagreements = 0, []
    for step, token in enumerate(tokens):
        token = int(token)
        pick = int(np.argmax(logits))
        if pick == token:
            agree += 1
        else:
            entry = {"step": step, "device_gap": float(logits[pick] - logits[token])}
            if exact_logits is not None:
                exact = np.asarray(exact_logits[step], np.float64)
                diff = np.asarray(logits, np.float64) - exact
                entry.update(exact_gap=float(exact[token] - exact[pick]), rms_diff=float(np.sqrt((diff ** 2).mean())),
                             max_diff=float(np.abs(diff).max()))
            disagreements.append(entry)
        if step + 1 < len(tokens):
            logits = chain.step(token)
    first = disagreements[0]["step"] if disagreements else None
    return {"agree": agree, "steps": len(tokens), "first_divergence": first, "disagreements": disagreements}
