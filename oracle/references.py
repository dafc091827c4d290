"""Per-op host references: the NPU's rounding model ("device") and float64 checks ("exact").

Test infrastructure only (see ``oracle/__init__.py``).

The "device" functions restate ``board_package/references.py``: they round to BF16 wherever the NPU writes a
register, so they reproduce the reference's own host references bit for bit (pinned by tests/golden).
The "exact" functions restate the reference's float64 checks (board_package/board_checks.py:238,319-327;
board_package/bf16.py:228-245; tests/test_mlir_gemm.py:96-101): float64 math with BF16 rounding only where a
tensor is stored as BF16, which is also what the B200 kernels compute (fp32 accumulate, BF16 storage).
"""

from __future__ import annotations

import math

import numpy as np
from numpy.typing import NDArray

from oracle.bf16 import (
    BLOCK_DEPTH,
    LN_EPSILON,
    MASKED_SCORE,
    TILE,
    bf16_bits,
    bf16_grid,
    bf16_values,
    gelu_exact_bf16,
    gelu_lut_bits,
)

# ----------------------------------------------------------------------------------------------------------------
# Device rounding model (board_package/references.py)
# ----------------------------------------------------------------------------------------------------------------


_WIDE: dict[int, tuple[NDArray, NDArray[np.float64]]] = {}


def widened(matrix) -> NDArray[np.float64]:
    """A weight matrix in float64, widened once and kept while the same array object is alive in the cache (the
    oracle's chains multiply by the same weights at every decode step)."""
    if not isinstance(matrix, np.ndarray) or matrix.size < (1 << 20):
        return np.asarray(matrix, dtype=np.float64)
    cached = _WIDE.get(id(matrix))
    if cached is None or cached[0] is not matrix:
        if len(_WIDE) >= 64:
            _WIDE.clear()
        cached = (matrix, matrix.astype(np.float64))
        _WIDE[id(matrix)] = cached
    return cached[1]


def device_product(left, right) -> NDArray[np.float32]:
    """A product summed as the NPU sums it: each 32-deep partial exact then rounded to BF16, added into a BF16
    running sum (``_device_product``, board_package/references.py:119-140)."""
    left = np.asarray(left, dtype=np.float32).astype(np.float64)
    wide = widened(right) if isinstance(right, np.ndarray) else np.asarray(right, dtype=np.float32).astype(np.float64)
    running = np.zeros((left.shape[0], wide.shape[1]), dtype=np.float32)
    for start in range(0, left.shape[1], BLOCK_DEPTH):
        stop = start + BLOCK_DEPTH
        partial = (left[:, start:stop] @ wide[start:stop]).astype(np.float32)
        running = bf16_grid(running + bf16_grid(partial))
    return running


def layernorm_device(rows, gamma, beta) -> NDArray[np.float32]:
    """LayerNorm rounded to BF16 after every step: BF16 sums scaled by a BF16 1/width, BF16 rsqrt, BF16 affine
    (``layernorm_reference``, board_package/references.py:28-46)."""
    x = bf16_grid(rows)
    inverse = bf16_grid(np.float32(1.0 / x.shape[1]))
    mean = bf16_grid(x.sum(axis=1, keepdims=True, dtype=np.float32) * inverse)
    centred = bf16_grid(x - mean)
    squares = bf16_grid(centred * centred)
    variance = bf16_grid(squares.sum(axis=1, keepdims=True, dtype=np.float32) * inverse)
    scale = bf16_grid(1.0 / np.sqrt(bf16_grid(variance + LN_EPSILON)))
    return bf16_grid(bf16_grid(centred * scale) * bf16_grid(gamma) + bf16_grid(beta))


def softmax_device(scores) -> NDArray[np.float32]:
    """Row softmax rounded to BF16 at the shift, the exponential, the sum and the product
    (``softmax_reference``, board_package/references.py:49-67)."""
    x = bf16_grid(scores)
    shifted = bf16_grid(x - x.max(axis=1, keepdims=True))
    weights = bf16_grid(np.exp(shifted, dtype=np.float32))
    totals = bf16_grid(weights.sum(axis=1, keepdims=True, dtype=np.float32))
    return bf16_grid(weights * bf16_grid(1.0 / totals))


def attention_device(query, key, value, *, causal: bool = False) -> NDArray[np.float32]:
    """One head's attention as the NPU computes it (``attention_reference``, board_package/references.py:93-116).

    The query is scaled by 1/sqrt(head) and rounded, the float64 scores are rounded, later keys are replaced by
    -1e30 when causal, the softmax is :func:`softmax_device`, and the weighted sum is float64 (not rounded).
    """
    head = query.shape[1]
    scaled = bf16_grid((np.asarray(query, dtype=np.float32) / math.sqrt(head)).astype(np.float32))
    scores = bf16_grid((scaled.astype(np.float64) @ bf16_grid(key).T.astype(np.float64)).astype(np.float32))
    if causal:
        later = np.arange(key.shape[0])[None, :] > np.arange(query.shape[0])[:, None]
        scores = np.where(later, np.float32(MASKED_SCORE), scores)
    weights = softmax_device(scores)
    return (weights.astype(np.float64) @ bf16_grid(value).astype(np.float64)).astype(np.float32)


def attention_decode_device(query_row, keys, values) -> NDArray[np.float32]:
    """The last row of :func:`attention_device` with ``causal=True`` when the query is the newest of ``keys``.

    Every cached key is at or before the query, so no mask applies; this is the KV-cached form the decode oracle
    uses, equal bit for bit to recomputing the whole causal attention and keeping the last row.
    """
    return attention_device(np.asarray(query_row, dtype=np.float32).reshape(1, -1), keys, values, causal=False)[0]


def gelu_device(values) -> NDArray[np.float32]:
    """The SFU's table GELU applied to BF16 values (board_package/references.py:88)."""
    return bf16_values(gelu_lut_bits(bf16_bits(values)).astype(np.uint16)).reshape(np.shape(values))


def _split_heads(matrix: NDArray[np.float32], heads: int) -> list[NDArray[np.float32]]:
    width = matrix.shape[1] // heads
    return [np.ascontiguousarray(matrix[:, h * width:(h + 1) * width]) for h in range(heads)]


def block_device(hidden, weights: dict, *, heads: int = 12) -> NDArray[np.float32]:
    """One GPT-2 block as the NPU computes it (``transformer_block_reference``, board_package/references.py:70-90)."""
    hidden = np.asarray(hidden, dtype=np.float32)
    normed = layernorm_device(hidden, weights["ln_1.g"], weights["ln_1.b"])
    fused = bf16_grid(device_product(normed, weights["attn.qkv.w"]) + weights["attn.qkv.b"])
    query, key, value = np.split(fused, 3, axis=1)
    heads_out = [attention_device(q, k, v, causal=True)
                 for q, k, v in zip(_split_heads(query, heads), _split_heads(key, heads), _split_heads(value, heads))]
    gathered = bf16_grid(np.concatenate(heads_out, axis=1))
    attended = bf16_grid(device_product(gathered, weights["attn.proj.w"]) + weights["attn.proj.b"])
    residual = bf16_grid(hidden + attended)
    normed = layernorm_device(residual, weights["ln_2.g"], weights["ln_2.b"])
    expanded = bf16_grid(device_product(normed, weights["mlp.fc.w"]) + weights["mlp.fc.b"])
    activated = gelu_device(expanded)
    contracted = bf16_grid(device_product(activated, weights["mlp.proj.w"]) + weights["mlp.proj.b"])
    return bf16_grid(residual + contracted)


# ----------------------------------------------------------------------------------------------------------------
# float64 references (the checks the reference's board and compiler tests hold devices to)
# ----------------------------------------------------------------------------------------------------------------


def attention_f64(query, key, value, *, mask=None) -> NDArray[np.float64]:
    """float64 softmax attention with an optional additive mask (``attention_reference``, board_package/bf16.py:228-245)."""
    scores = np.asarray(query, dtype=np.float64) @ np.asarray(key, dtype=np.float64).T
    if mask is not None:
        scores = scores + mask
    weights = np.exp(scores - scores.max(axis=1, keepdims=True))
    return (weights / weights.sum(axis=1, keepdims=True)) @ np.asarray(value, dtype=np.float64)


def attention_tiles_device(query, key, value, *, initial_maximum: float, mask=None) -> NDArray[np.float32]:
    """One attention block as the image computes it, 16 keys at a time with a BF16 online softmax
    (``attention_bf16_reference``, board_package/bf16.py:248-291)."""
    query = np.asarray(query, dtype=np.float32)
    key = np.asarray(key, dtype=np.float32)
    value = np.asarray(value, dtype=np.float32)
    rows, head = query.shape
    maximum = np.full((rows, 1), initial_maximum, dtype=np.float32)
    total = np.zeros((rows, 1), dtype=np.float32)
    out = np.zeros((rows, head), dtype=np.float32)
    for start in range(0, key.shape[0], TILE):
        keys, values = key[start:start + TILE], value[start:start + TILE]
        scores = np.zeros((rows, TILE), dtype=np.float32)
        for step in range(0, head, TILE):
            piece = bf16_grid(query[:, step:step + TILE] @ keys[:, step:step + TILE].T)
            scores = piece if step == 0 else bf16_grid(scores + piece)
        if mask is not None:
            scores = bf16_grid(scores + mask[:, start:start + TILE])
        new_max = bf16_grid(np.maximum(maximum, scores.max(axis=1, keepdims=True)))
        alpha = bf16_grid(np.exp(bf16_grid(maximum - new_max)))
        maximum = new_max
        probabilities = bf16_grid(np.exp(bf16_grid(scores - new_max)))
        total = bf16_grid(bf16_grid(total * alpha) + bf16_grid(probabilities.sum(axis=1, keepdims=True)))
        out = bf16_grid(out * alpha)
        for tile in range(0, head, TILE):
            piece = bf16_grid(probabilities @ values[:, tile:tile + TILE])
            out[:, tile:tile + TILE] = bf16_grid(out[:, tile:tile + TILE] + piece)
    return bf16_grid(out * bf16_grid(1.0 / total))


def gemm_f64(left, right, *, bias=None, activate: bool = False) -> NDArray[np.float64]:
    """[GELU](left) @ right (+ bias) in float64, GELU exact-erf on BF16 inputs rounded back to BF16 as the staging
    leaves them (board_package/board_checks.py:238; tests/test_mlir_gemm.py:96-101; tests/test_mlir_padding.py:159-162)."""
    staged = gelu_exact_bf16(left) if activate else np.asarray(left, dtype=np.float32)
    product = staged.astype(np.float64) @ widened(right)
    if bias is not None:
        product = product + np.asarray(bias, dtype=np.float64)
    return product


def layernorm_f64(rows, gamma, beta, *, epsilon: float = LN_EPSILON) -> NDArray[np.float64]:
    """float64 LayerNorm (tests/test_mlir_layernorm.py:84-86)."""
    values = np.asarray(rows, dtype=np.float64)
    centred = values - values.mean(axis=1, keepdims=True)
    return centred / np.sqrt((centred ** 2).mean(axis=1, keepdims=True) + epsilon) * gamma + beta


def causal_attention_f64(query, key, value) -> NDArray[np.float64]:
    """float64 causal attention of one head whose queries already carry 1/sqrt(head)
    (tests/test_mlir_attention.py:165-175)."""
    scores = np.asarray(query, dtype=np.float64) @ np.asarray(key, dtype=np.float64).T
    scores = np.where(np.tril(np.ones_like(scores, dtype=bool)), scores, -np.inf)
    weights = np.exp(scores - scores.max(axis=1, keepdims=True))
    return (weights / weights.sum(axis=1, keepdims=True)) @ np.asarray(value, dtype=np.float64)


def relative_error(actual, expected) -> float:
    """Relative Frobenius error, the metric every reference check gates on (board_package/board_checks.py:239)."""
    expected = np.asarray(expected, dtype=np.float64)
    return float(np.linalg.norm(np.asarray(actual, dtype=np.float64) - expected) / np.linalg.norm(expected))


def max_relative_error(actual, expected) -> float:
    """Elementwise max |error| over max |expected|, reported beside the norm-wise figure."""
    expected = np.asarray(expected, dtype=np.float64)
    return float(np.abs(np.asarray(actual, dtype=np.float64) - expected).max() / np.abs(expected).max())


# ----------------------------------------------------------------------------------------------------------------
# Exact-mode block: float64 per op, BF16 where the B200 path stores BF16
# ----------------------------------------------------------------------------------------------------------------


def block_exact(hidden, weights: dict, *, heads: int = 12) -> NDArray[np.float32]:
    """One GPT-2 block with float64 arithmetic inside every op and BF16 rounding at every stored tensor, the way the
    B200 native path stores them: LN out, QKV, attention out, each residual sum (bias and residual added before the
    one rounding), the FC output (rounded, then exact-erf GELU, rounded again).

    The op order is ``_run_layer``'s (board_package/gpt2_inference.py:1133-1189)."""
    x = bf16_grid(hidden)
    width = x.shape[1]
    head = width // heads
    normed = bf16_grid(layernorm_f64(x, weights["ln_1.g"], weights["ln_1.b"]))
    fused = bf16_grid(gemm_f64(normed, weights["attn.qkv.w"], bias=weights["attn.qkv.b"]))
    query = bf16_grid(fused[:, :width] / math.sqrt(head))
    key, value = fused[:, width:2 * width], fused[:, 2 * width:]
    gathered = np.concatenate([causal_attention_f64(query[:, h * head:(h + 1) * head],
                                                    key[:, h * head:(h + 1) * head],
                                                    value[:, h * head:(h + 1) * head]) for h in range(heads)], axis=1)
    gathered = bf16_grid(gathered)
    residual = bf16_grid(x + gemm_f64(gathered, weights["attn.proj.w"], bias=weights["attn.proj.b"]))
    normed = bf16_grid(layernorm_f64(residual, weights["ln_2.g"], weights["ln_2.b"]))
    expanded = gelu_exact_bf16(bf16_grid(gemm_f64(normed, weights["mlp.fc.w"], bias=weights["mlp.fc.b"])))
    return bf16_grid(residual + gemm_f64(expanded, weights["mlp.proj.w"], bias=weights["mlp.proj.b"]))
