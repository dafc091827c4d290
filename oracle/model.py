"""GPT-2 small on the host, chained from the per-op references: full recompute and a KV-cached restatement.

Test infrastructure only (see ``oracle/__init__.py``).

The full-recompute chain is the one the reference's decode check runs (board_package/board_checks.py:467-474):
``embed`` -> every ``transformer_block_reference`` -> ``layernorm_reference`` on the last row -> ``lm_head``.
The reference has no KV-cached host decode; :class:`CachedChain` restates one from the same primitives, and
tests/test_oracle_model.py proves it equal to the full recompute on a few steps.

``mode="device"`` uses the NPU rounding model (references.py semantics, GELU table, BF16 accumulation);
``mode="exact"`` uses float64 ops with BF16 storage, the arithmetic the B200 kernels carry out.
"""

from __future__ import annotations

import math

import numpy as np
from numpy.typing import NDArray

from oracle.bf16 import bf16_grid, gelu_exact_bf16
from oracle.references import (
    attention_decode_device,
    block_device,
    block_exact,
    device_product,
    gemm_f64,
    gelu_device,
    layernorm_device,
    layernorm_f64,
    widened,
)

END_OF_TEXT: int = 50256
"""GPT-2's end-of-text token, which the reference's ``generate`` stops at (board_package/gpt2_inference.py:93)."""


def embed(token_ids, shared: dict, *, start: int = 0) -> NDArray[np.float32]:
    """Token plus position embeddings (``embed``, board_package/gpt2_inference.py:800-812)."""
    ids = np.asarray(token_ids, dtype=np.int64)
    positions = start + np.arange(len(ids))
    return (shared["wte"][ids] + shared["wpe"][positions]).astype(np.float32)


def final_norm(rows, shared: dict, mode: str) -> NDArray[np.float32]:
    """GPT-2's final LayerNorm (board_package/gpt2_inference.py:890-912)."""
    if mode == "device":
        return layernorm_device(rows, shared["ln_f.g"], shared["ln_f.b"])
    return bf16_grid(layernorm_f64(bf16_grid(rows), shared["ln_f.g"], shared["ln_f.b"]))


def lm_head(normalised, shared: dict, mode: str) -> NDArray:
    """Logits through the tied embedding (``lm_head``, board_package/gpt2_inference.py:915-925): float32 on the host
    in device mode as the reference does, float64 in exact mode."""
    if mode == "device":
        return np.asarray(normalised, dtype=np.float32) @ shared["wte"].T
    return widened(shared["wte"]) @ np.asarray(normalised, dtype=np.float64)


def block(rows, weights: dict, mode: str) -> NDArray[np.float32]:
    """One block in the chosen mode."""
    return block_device(rows, weights) if mode == "device" else block_exact(rows, weights)


def forward_logits(token_ids, layers: list[dict], shared: dict, *, mode: str = "device") -> NDArray:
    """Logits after the last token, recomputing the whole sequence (board_package/board_checks.py:469-474)."""
    rows = embed(token_ids, shared)
    for weights in layers:
        rows = block(rows, weights, mode)
    return lm_head(final_norm(rows[-1:], shared, mode)[0], shared, mode)


def greedy_full_recompute(token_ids, layers, shared, *, new_tokens: int, mode: str = "device") -> list[int]:
    """Greedy continuation by full recompute per token; slow, used on short sequences to pin :class:`CachedChain`."""
    sequence = list(int(t) for t in token_ids)
    out: list[int] = []
    for _ in range(new_tokens):
        token = int(np.argmax(forward_logits(sequence, layers, shared, mode=mode)))
        out.append(token)
        sequence.append(token)
    return out


class CachedChain:
    """GPT-2 with per-layer key/value caches on the host, built only from the per-op references.

    Prefill runs every layer over the prompt and keeps each layer's keys and values; a decode step runs the new
    token alone through every layer, attending over the cache. The result equals :func:`forward_logits` over the
    whole sequence, because every op but attention is row-wise and the newest query masks nothing.
    """

    def __init__(self, layers: list[dict], shared: dict, *, mode: str = "device", heads: int = 12) -> None:
        self.layers = layers
        self.shared = shared
        self.mode = mode
        self.heads = heads
        self.keys: list[NDArray[np.float32]] = []
        self.values: list[NDArray[np.float32]] = []
        self.length = 0

    # -- one layer over rows that attend causally to themselves and to the cache ------------------------------

    def _qkv(self, rows, weights):
        if self.mode == "device":
            normed = layernorm_device(rows, weights["ln_1.g"], weights["ln_1.b"])
            return bf16_grid(device_product(normed, weights["attn.qkv.w"]) + weights["attn.qkv.b"])
        normed = bf16_grid(layernorm_f64(bf16_grid(rows), weights["ln_1.g"], weights["ln_1.b"]))
        return bf16_grid(gemm_f64(normed, weights["attn.qkv.w"], bias=weights["attn.qkv.b"]))

    def _attend_row(self, query, keys, values) -> NDArray[np.float32]:
        width = query.shape[0]
        head = width // self.heads
        out = np.empty(width, dtype=np.float32)
        for h in range(self.heads):
            cols = slice(h * head, (h + 1) * head)
            if self.mode == "device":
                out[cols] = attention_decode_device(query[cols], keys[:, cols], values[:, cols])
            else:
                q = bf16_grid(query[cols] / math.sqrt(head)).astype(np.float64)
                scores = keys[:, cols].astype(np.float64) @ q
                weights = np.exp(scores - scores.max())
                out[cols] = (weights / weights.sum()) @ values[:, cols].astype(np.float64)
        return out

    def _finish(self, rows, gathered, weights):
        if self.mode == "device":
            attended = bf16_grid(device_product(bf16_grid(gathered), weights["attn.proj.w"]) + weights["attn.proj.b"])
            residual = bf16_grid(rows + attended)
            normed = layernorm_device(residual, weights["ln_2.g"], weights["ln_2.b"])
            expanded = bf16_grid(device_product(normed, weights["mlp.fc.w"]) + weights["mlp.fc.b"])
            contracted = bf16_grid(device_product(gelu_device(expanded), weights["mlp.proj.w"]) + weights["mlp.proj.b"])
            return bf16_grid(residual + contracted)
        residual = bf16_grid(bf16_grid(rows) + gemm_f64(bf16_grid(gathered), weights["attn.proj.w"],
                                                        bias=weights["attn.proj.b"]))
        normed = bf16_grid(layernorm_f64(residual, weights["ln_2.g"], weights["ln_2.b"]))
        expanded = gelu_exact_bf16(bf16_grid(gemm_f64(normed, weights["mlp.fc.w"], bias=weights["mlp.fc.b"])))
        return bf16_grid(residual + gemm_f64(expanded, weights["mlp.proj.w"], bias=weights["mlp.proj.b"]))

    def prefill(self, token_ids) -> NDArray:
        """Runs the prompt through every layer, filling the caches, and returns the logits after its last token."""
        rows = embed(token_ids, self.shared)
        self.keys, self.values = [], []
        for weights in self.layers:
            fused = self._qkv(rows, weights)
            width = rows.shape[1]
            self.keys.append(fused[:, width:2 * width].copy())
            self.values.append(fused[:, 2 * width:].copy())
            rows = block(rows, weights, self.mode)
        self.length = len(token_ids)
        return lm_head(final_norm(rows[-1:], self.shared, self.mode)[0], self.shared, self.mode)

    def step(self, token_id: int) -> NDArray:
        """Runs one new token through every layer, appending to each cache, and returns the next logits."""
        row = embed([token_id], self.shared, start=self.length)
        for index, weights in enumerate(self.layers):
            fused = self._qkv(row, weights)
            width = row.shape[1]
            self.keys[index] = np.concatenate([self.keys[index], fused[:, width:2 * width]], axis=0)
            self.values[index] = np.concatenate([self.values[index], fused[:, 2 * width:]], axis=0)
            gathered = self._attend_row(fused[0, :width], self.keys[index], self.values[index])[None, :]
            row = self._finish(row, gathered, weights)
        self.length += 1
        return lm_head(final_norm(row, self.shared, self.mode)[0], self.shared, self.mode)

    def generate(self, token_ids, *, new_tokens: int, stop_at_end: bool = False) -> tuple[list[int], list[float]]:
        """Greedy continuation (``generate``, board_package/gpt2_inference.py:941-978).

        Returns the tokens and, per step, the gap between the best and second-best logit (the tie margin).
        """
        logits = self.prefill(token_ids)
        tokens: list[int] = []
        margins: list[float] = []
        while len(tokens) < new_tokens:
            order = np.argsort(logits)
            token = int(np.argmax(logits))
            tokens.append(token)
            margins.append(float(logits[order[-1]] - logits[order[-2]]))
            if (stop_at_end and token == END_OF_TEXT) or len(tokens) == new_tokens:
                break
            logits = self.step(token)
        return tokens, margins
