"""BF16 arithmetic, the NPU's packed layouts and the operand builders, restated from the reference's host code.

Test infrastructure only (see ``oracle/__init__.py``). Each function names the reference function it restates,
by its path and line inside the yeungn523/tempo-compiler project.
"""

from __future__ import annotations

import math

import numpy as np
from numpy.typing import NDArray

# Geometry of the reference NPU, which the packed drop-in layouts are defined in (board_package/bf16.py:21-79).
TILE: int = 16
"""Edge of one MXU tile: the packed layouts group features in runs of this many BF16 values (32 bytes)."""

BLOCK_TOKENS: int = 32
"""Token rows one launch of a per-block image covers (board_package/bf16.py:51)."""

BLOCK_DEPTH: int = 32
"""Contraction depth whose partial the NPU sums exactly before a BF16 accumulate (board_package/bf16.py:54)."""

SUBLANES: int = 4
"""Times each bias tile repeats in the packed bias (board_package/bf16.py:57)."""

VREG_ELEMENTS: int = 64
"""Values a LayerNorm scalar is broadcast across in the constants block (board_package/bf16.py:72)."""

ZERO_TILE_WORDS: int = TILE * TILE
"""Words of the zeroed clearing tile that heads every packed block (board_package/bf16.py:66)."""

ZERO_TILE_BYTES: int = 2 * ZERO_TILE_WORDS
"""Bytes of that tile."""

MODEL_WIDTH: int = 768
"""GPT-2 small's width (board_package/bf16.py:75)."""

LN_EPSILON: float = 1e-5
"""LayerNorm's variance floor (board_package/bf16.py:78)."""

GELU_TABLE_ENTRIES: int = 2048
"""Entries of the NPU's GELU lookup table (board_package/bf16.py:30)."""

GELU_LIMIT_Q7: int = 8 * 128
"""Q7 magnitude at which the table saturates, i.e. 8.0 (board_package/bf16.py:33)."""

MASKED_SCORE: float = -1.0e30
"""Score a mask tile adds to an excluded key (board_package/bf16.py:205, references.py:114)."""


def bf16_bits(values) -> NDArray[np.uint16]:
    """Rounds float32 values to BF16 words, nearest-even on the bit pattern.

    Restates ``as_bf16_words`` (board_package/bf16.py:82-97): add 0x7FFF plus the kept LSB to the float32 bits
    in wrapping 32-bit arithmetic and keep the high half.
    """
    bits = np.ascontiguousarray(values, dtype="<f4").view("<u4")
    keep = (bits >> np.uint32(16)) & np.uint32(1)
    rounded = bits + np.uint32(0x7FFF) + keep
    return (rounded >> np.uint32(16)).astype("<u2")


def bf16_values(words) -> NDArray[np.float32]:
    """Widens BF16 words to the float32 values they hold (board_package/bf16.py:100-102)."""
    return (np.asarray(words).astype("<u4") << np.uint32(16)).view("<f4")


def bf16_grid(values) -> NDArray[np.float32]:
    """Rounds values onto the BF16 grid, keeping their shape (``_on_bf16_grid``, board_package/bf16.py:402-412)."""
    array = np.asarray(values, dtype=np.float32)
    return bf16_values(bf16_bits(array.reshape(-1))).reshape(array.shape)


def _round_one(value: float) -> int:
    """Nearest-even BF16 bits of one Python float, narrowed through float32 (board_package/bf16.py:436-446)."""
    bits = int(np.array([value], dtype="<f4").view("<u4")[0])
    return ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16) & 0xFFFF


_GELU_TABLE_CACHE: list[NDArray[np.uint16]] = []


def gelu_table() -> NDArray[np.uint16]:
    """The NPU's 2048-entry GELU ROM: exact-erf GELU at the centre of each 1/128-wide bin over [-8, 8), in BF16.

    Restates ``_gelu_table`` (board_package/bf16.py:395-399).
    """
    if not _GELU_TABLE_CACHE:
        entries = []
        for index in range(GELU_TABLE_ENTRIES):
            centre = -8.0 + (index + 0.5) / 128.0
            entries.append(_round_one(0.5 * centre * (1.0 + math.erf(centre / math.sqrt(2.0)))))
        _GELU_TABLE_CACHE.append(np.array(entries, dtype="<u2"))
    return _GELU_TABLE_CACHE[0]


def _magnitude_q7(magnitude_bits: NDArray[np.uint32]) -> NDArray[np.int64]:
    """Float32 magnitudes (sign already cleared) as truncated Q7 integers, saturated at 0x1FFF.

    Restates ``_fp32_abs_q7`` (board_package/bf16.py:415-433): value*128 is the 24-bit significand shifted right
    by 16 - unbiased exponent; a shift of 24 or more truncates to zero, one of 10 or less saturates the 13-bit field.
    """
    exponent = ((magnitude_bits >> np.uint32(23)) & np.uint32(0xFF)).astype(np.int64)
    significand = ((magnitude_bits & np.uint32(0x7FFFFF)) | np.uint32(1 << 23)).astype(np.int64)
    shift = 16 - (exponent - 127)
    truncated = significand >> np.clip(shift, 0, 63)
    q7 = np.where(shift <= 10, 0x1FFF, truncated)
    return np.where((exponent == 0) | (shift >= 24), 0, q7)


def gelu_lut_bits(words) -> NDArray[np.uint32]:
    """The NPU SFU's table GELU over BF16 words (``gelu_lut_reference``, board_package/bf16.py:105-121).

    The table address is 1024 + q7 for a positive input and 1023 - q7 for a negative one; at or past 8.0 in
    magnitude the unit passes a positive input through and flushes a negative one to zero, and a zero stays zero.
    """
    words32 = np.asarray(words).astype("<u4")
    operand = words32 << np.uint32(16)
    negative = (operand >> np.uint32(31)).astype(bool)
    magnitude_bits = operand & np.uint32(0x7FFFFFFF)
    q7 = _magnitude_q7(magnitude_bits)
    address = np.where(negative, GELU_LIMIT_Q7 - 1 - q7, GELU_LIMIT_Q7 + q7)
    looked_up = gelu_table()[np.clip(address, 0, GELU_TABLE_ENTRIES - 1)].astype("<u4")
    passed = np.where(negative, np.uint32(0), words32)
    result = np.where(q7 >= GELU_LIMIT_Q7, passed, looked_up)
    return np.where(magnitude_bits == 0, np.uint32(0), result).astype("<u4")


def gelu_exact_bf16(values) -> NDArray[np.float32]:
    """Exact-erf GELU in float64 of BF16 values, rounded back to BF16.

    This is what the reference's own float64 checks apply to staged activations (tests/test_mlir_padding.py:159-162,
    tests/test_mlir_gemm.py:98-101) and what the B200 kernels compute (fp32 erf of a BF16 input, rounded to BF16).
    """
    from scipy.special import erf

    widened = np.asarray(values, dtype=np.float64)
    return bf16_grid((0.5 * widened * (1.0 + erf(widened / math.sqrt(2.0)))).astype(np.float32))


def _pad_last(values: NDArray[np.float32]) -> NDArray[np.float32]:
    """Zero-pads the last axis to whole tiles (``_padded_columns``, board_package/bf16.py:124-130)."""
    short = -values.shape[-1] % TILE
    if not short:
        return values
    return np.pad(values, [(0, 0)] * (values.ndim - 1) + [(0, short)])


def pack_activations(activations) -> NDArray[np.uint16]:
    """[tokens, depth] -> BF16 words laid out [depth/16][tokens][16] (board_package/bf16.py:133-156).

    Raises:
        ValueError: If the tokens are not a whole number of 16-row groups.
    """
    activations = np.asarray(activations, dtype=np.float32)
    tokens = activations.shape[0]
    if tokens % TILE:
        raise ValueError(f"Unable to pack activations of shape {list(activations.shape)}: the token rows must be a "
                         f"whole number of {TILE}.")
    padded = _pad_last(activations)
    words = bf16_bits(padded).reshape(tokens, padded.shape[1] // TILE, TILE)
    return np.ascontiguousarray(words.transpose(1, 0, 2)).reshape(-1)


def unpack_activations(words, *, tokens: int, features: int) -> NDArray[np.float32]:
    """Inverse of :func:`pack_activations` for one packed run: [features/16][tokens][16] words -> [tokens, features]."""
    tiles = bf16_values(np.asarray(words)[: tokens * features]).reshape(features // TILE, tokens, TILE)
    return np.ascontiguousarray(tiles.transpose(1, 0, 2)).reshape(tokens, features)


def pack_bias(bias) -> NDArray[np.uint16]:
    """One feature row -> [features/16][4][16] words, each tile repeated four times (board_package/bf16.py:159-175).

    Raises:
        ValueError: If the bias is not one row.
    """
    bias = np.asarray(bias, dtype=np.float32)
    if bias.ndim != 1:
        raise ValueError(f"Unable to pack a bias of shape {bias.shape}: it must be one row.")
    tiles = bf16_bits(_pad_last(bias)).reshape(-1, TILE)
    return np.ascontiguousarray(np.repeat(tiles, SUBLANES, axis=0)).reshape(-1)


def pack_weights(weights) -> NDArray[np.uint16]:
    """[depth, columns] -> BF16 words laid out [columns/16][depth][16] (board_package/bf16.py:178-192)."""
    weights = np.asarray(weights, dtype=np.float32)
    padded = _pad_last(_pad_last(weights).T).T
    depth, columns = padded.shape
    words = bf16_bits(padded).reshape(depth, columns // TILE, TILE)
    return np.ascontiguousarray(words.transpose(1, 0, 2)).reshape(-1)


def decode_mask_tiles(*, keys: int, length: int) -> NDArray[np.float32]:
    """Mask tiles a decode step adds: 0 for the first ``length`` of ``keys`` keys, -1e30 past them.

    Shaped [1, keys/16, 16 queries, 16 keys], every query row the same (board_package/bf16.py:195-207).
    """
    row = np.where(np.arange(keys) < length, np.float32(0.0), np.float32(MASKED_SCORE)).astype(np.float32)
    return np.ascontiguousarray(np.broadcast_to(row.reshape(1, keys // TILE, 1, TILE), (1, keys // TILE, TILE, TILE)))


def pack_attention_constants(*, initial_maximum: float, constants: tuple[float, ...], masks) -> NDArray[np.uint16]:
    """The constants block of an attention image, per query block: a tile of the entering maximum, a tile of zeros,
    a tile per stated number, then that block's mask tiles; all as BF16 words, shape [rows, 16].

    Restates ``pack_attention_constants`` and ``_attention_constants`` (board_package/bf16.py:210-225,364-371).
    """
    masks = np.asarray(masks, dtype=np.float32)
    per_block = []
    for block in range(masks.shape[0]):
        rows = [np.full((TILE, TILE), initial_maximum, dtype=np.float32), np.zeros((TILE, TILE), dtype=np.float32)]
        rows += [np.full((TILE, TILE), number, dtype=np.float32) for number in constants]
        rows += list(masks[block])
        per_block.append(np.concatenate(rows, axis=0))
    return bf16_bits(np.concatenate(per_block, axis=0))


def causal_constants_words() -> NDArray[np.uint16]:
    """The constants block a causal attention image reads: entering-maximum tile, zero tile, then the diagonal mask
    tile laid out keys by queries, -1e30 where the key is past the query (mlir/lib/tempo/manifest.cpp:197-222)."""
    key = np.arange(TILE)[:, None]
    query = np.arange(TILE)[None, :]
    diagonal = np.where(key > query, np.float32(MASKED_SCORE), np.float32(0.0))
    tiles = [np.full((TILE, TILE), MASKED_SCORE, dtype=np.float32), np.zeros((TILE, TILE), dtype=np.float32), diagonal]
    return bf16_bits(np.concatenate(tiles, axis=0)).reshape(-1)


def _moved_permutation(rng: np.random.Generator, count: int):
    """A permutation of ``count`` positions that moves at least one, or None below two (board_package/bf16.py:374-392)."""
    if count < 2:
        return None
    identity = np.arange(count)
    order = rng.permutation(count)
    while np.array_equal(order, identity):
        order = rng.permutation(count)
    return order


def check_operands_discriminating(activations, weights) -> None:
    """Rejects a GEMM operand pair whose product survives a permutation of tokens, contraction blocks or columns.

    Restates ``assert_operands_discriminating`` (board_package/bf16.py:294-329), including its draw order.

    Raises:
        ValueError: Naming the axis ("tokens", "contraction blocks" or "output columns") the product is blind to.
    """
    left = np.asarray(activations, dtype=np.float64)
    right = np.asarray(weights, dtype=np.float64)
    product = left @ right
    rng = np.random.default_rng(0)
    trials = []
    order = _moved_permutation(rng, left.shape[0])
    if order is not None:
        trials.append(("tokens", left[order] @ right))
    blocks = left.shape[1] // BLOCK_DEPTH
    order = _moved_permutation(rng, blocks)
    if order is not None:
        shuffled = left.reshape(left.shape[0], blocks, BLOCK_DEPTH)[:, order, :].reshape(left.shape)
        trials.append(("contraction blocks", shuffled @ right))
    order = _moved_permutation(rng, right.shape[1])
    if order is not None:
        trials.append(("output columns", left @ right[:, order]))
    for axis, permuted in trials:
        if np.array_equal(permuted, product):
            raise ValueError(f"Unable to use these operands as evidence: permuting their {axis} leaves the product "
                             f"unchanged, so a kernel confusing one for another would pass.")


def build_operands(tokens: int, depth: int, columns: int, *, kind: str, seed: int):
    """One GEMM operand pair: ``structured`` (exactly representable, identical token rows) or ``varying``.

    Restates ``build_operands`` (board_package/bf16.py:332-361).
    """
    if kind == "structured":
        left = (np.arange(tokens * depth, dtype=np.float32).reshape(tokens, depth) % 2).astype(np.float32)
        scales = (2.0 ** -(np.arange(columns) % 4)) / 16.0
        right = np.broadcast_to(scales, (depth, columns)).astype(np.float32)
        return left, right
    rng = np.random.default_rng(seed)
    left = bf16_grid(rng.standard_normal((tokens, depth)).astype(np.float32))
    right = bf16_grid(rng.standard_normal((depth, columns)).astype(np.float32))
    check_operands_discriminating(left, right)
    return left, right
