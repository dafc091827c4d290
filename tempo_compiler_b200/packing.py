"""BF16 conversion and the packed block layouts of the per-32-token launch contract, on the host.

The drop-in op surface keeps the reference NPU's packed device layouts so that its layer drivers need no change
(board_package/gpt2_inference.py:136-230, mlir/include/tempo/tempo/tempo_ops.td:228-330):

* activations of one 32-token block: ``[features/16][32 tokens][16]`` BF16, headed in a device tensor by a zeroed
  16x16 tile (512 bytes);
* weights: ``[columns/16][depth][16]`` BF16;
* a bias row: ``[columns/16][4][16]`` BF16, each 16-feature tile repeated four times;
* a LayerNorm constants block: gamma, beta, then 1/width and epsilon each repeated 64 times, BF16.

These helpers pack and unpack those layouts with torch (CPU or CUDA tensors) so the host side never round-trips
through Python loops.
"""

from __future__ import annotations

import numpy as np
import torch

TILE = 16
BLOCK_TOKENS = 32
ZERO_TILE_BYTES = 512
BIAS_REPEAT = 4
SCALAR_REPEAT = 64


def to_bf16(values) -> torch.Tensor:
    """Nearest-even BF16 of float32 values (torch's conversion is round-to-nearest-even)."""
    tensor = values if isinstance(values, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(values, np.float32))
    return tensor.to(torch.float32).to(torch.bfloat16)


def bf16_words(values) -> np.ndarray:
    """BF16 words (uint16) of float32 values, rounded to nearest even."""
    return to_bf16(values).view(torch.int16).numpy().view(np.uint16)


def words_to_float(words) -> np.ndarray:
    """float32 values of BF16 words."""
    return (np.asarray(words).astype(np.uint32) << 16).view(np.float32)


def pack_block_rows(rows: torch.Tensor) -> torch.Tensor:
    """[tokens, features] (tokens a multiple of 16, features of 16) -> [features/16, tokens, 16], contiguous."""
    tokens, features = rows.shape
    return rows.reshape(tokens, features // TILE, TILE).permute(1, 0, 2).contiguous()


def unpack_block_rows(tiles: torch.Tensor, tokens: int, features: int) -> torch.Tensor:
    """Inverse of :func:`pack_block_rows`."""
    return tiles.reshape(features // TILE, tokens, TILE).permute(1, 0, 2).reshape(tokens, features)


def pack_weight_tiles(weights: torch.Tensor) -> torch.Tensor:
    """[depth, columns] -> [columns/16, depth, 16], contiguous (columns a multiple of 16)."""
    depth, columns = weights.shape
    return weights.reshape(depth, columns // TILE, TILE).permute(1, 0, 2).contiguous()


def pack_bias_tiles(bias: torch.Tensor) -> torch.Tensor:
    """[columns] -> [columns/16, 4, 16]: each 16-feature tile repeated four times."""
    tiles = bias.reshape(-1, 1, TILE)
    return tiles.expand(-1, BIAS_REPEAT, TILE).contiguous()


def layernorm_constants(gamma, beta, scalars) -> torch.Tensor:
    """The LayerNorm constants block as BF16: gamma, beta, then every manifest scalar repeated 64 times
    (board_package/gpt2_inference.py:439-471)."""
    pieces = [torch.as_tensor(np.asarray(gamma, np.float32)), torch.as_tensor(np.asarray(beta, np.float32))]
    pieces += [torch.full((SCALAR_REPEAT,), float(s), dtype=torch.float32) for s in scalars]
    return torch.cat(pieces).to(torch.bfloat16)


def pad_to_tiles(values: np.ndarray) -> np.ndarray:
    """Zero-pads the last axis to whole 16-wide tiles."""
    short = -values.shape[-1] % TILE
    return values if not short else np.pad(values, [(0, 0)] * (values.ndim - 1) + [(0, short)])
