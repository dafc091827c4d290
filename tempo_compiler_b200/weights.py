"""Seeded random GPT-2 weights in the reference's naming scheme.

No checkpoint is reachable here, so every workload runs on random-init weights drawn from a seed: each matrix and
bias ~N(0, 0.02) and every LayerNorm with gamma = 1 and beta = 0, all on the BF16 grid. The names follow the export
the reference's drivers read (tools/board/export_gpt2_weights.py:43-53, board_package/gpt2_inference.py:315-342):
one dict per layer keyed ``ln_1.g``, ``attn.qkv.w`` ... ``mlp.proj.b``, and a shared dict keyed ``wte``, ``wpe``,
``ln_f.g``, ``ln_f.b``. Matrices are ``[in, out]``, as the reference multiplies ``hidden @ W``.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch


@dataclass(frozen=True)
class GPT2Shape:
    """The dimensions of a GPT-2 model."""

    layers: int = 12
    width: int = 768
    heads: int = 12
    vocab: int = 50257
    positions: int = 1024

    @property
    def ffn(self) -> int:
        return 4 * self.width

    @property
    def head(self) -> int:
        return self.width // self.heads


GPT2_SMALL = GPT2Shape()

LAYER_KEYS = ("ln_1.g", "ln_1.b", "attn.qkv.w", "attn.qkv.b", "attn.proj.w", "attn.proj.b",
              "ln_2.g", "ln_2.b", "mlp.fc.w", "mlp.fc.b", "mlp.proj.w", "mlp.proj.b")


def _grid(values: np.ndarray) -> np.ndarray:
    """Rounds float32 values onto the BF16 grid (nearest even)."""
    return torch.from_numpy(values).to(torch.bfloat16).to(torch.float32).numpy()


def random_gpt2(seed: int, shape: GPT2Shape = GPT2_SMALL, *, std: float = 0.02) -> tuple[list[dict], dict]:
    """Random-init GPT-2 weights on the BF16 grid, drawn from ``seed`` in a fixed order.

    Returns:
        One dict per layer and the shared dict, every value a float32 numpy array on the BF16 grid.
    """
    rng = np.random.default_rng(seed)
    width, ffn = shape.width, shape.ffn

    def normal(*dims: int) -> np.ndarray:
        return _grid((rng.standard_normal(dims, dtype=np.float32) * np.float32(std)).astype(np.float32))

    ones = np.ones(width, dtype=np.float32)
    zeros = np.zeros(width, dtype=np.float32)
    layers = []
    for _ in range(shape.layers):
        layers.append({
            "ln_1.g": ones.copy(), "ln_1.b": zeros.copy(),
            "attn.qkv.w": normal(width, 3 * width), "attn.qkv.b": normal(3 * width),
            "attn.proj.w": normal(width, width), "attn.proj.b": normal(width),
            "ln_2.g": ones.copy(), "ln_2.b": zeros.copy(),
            "mlp.fc.w": normal(width, ffn), "mlp.fc.b": normal(ffn),
            "mlp.proj.w": normal(ffn, width), "mlp.proj.b": normal(width),
        })
    shared = {"wte": normal(shape.vocab, width), "wpe": normal(shape.positions, width),
              "ln_f.g": ones.copy(), "ln_f.b": zeros.copy()}
    return layers, shared


def save_gpt2_npz(path, layers: list[dict], shared: dict) -> None:
    """Writes weights in the reference's export format: one BF16-word (uint16) array per tensor, per-layer names
    prefixed ``h.<layer>.`` (tools/board/export_gpt2_weights.py:43-53)."""
    arrays = {}
    for index, layer in enumerate(layers):
        for name, value in layer.items():
            arrays[f"h.{index}.{name}"] = _words(value)
    for name, value in shared.items():
        arrays[name] = _words(value)
    np.savez(path, **arrays)


def load_gpt2_npz(path) -> tuple[list[dict], dict]:
    """Reads the reference's exported weights (``gpt2_weights.npz``) as float32 arrays, split into per-layer dicts and
    the shared dict the way the reference's loader splits them (board_package/gpt2_inference.py:315-342).

    Raises:
        FileNotFoundError: If the file does not exist.
        ValueError: If a layer lacks one of the twelve tensors a GPT-2 block reads.
    """
    with np.load(path) as exported:
        weights = {name: (exported[name].astype(np.uint32) << 16).view(np.float32) for name in exported.files}
    layers: list[dict] = []
    while f"h.{len(layers)}.ln_1.g" in weights:
        prefix = f"h.{len(layers)}."
        layer = {name[len(prefix):]: value for name, value in weights.items() if name.startswith(prefix)}
        missing = [key for key in LAYER_KEYS if key not in layer]
        if missing:
            raise ValueError(f"layer {len(layers)} of {path} lacks {missing}")
        layers.append(layer)
    shared = {name: value for name, value in weights.items() if not name.startswith("h.")}
    return layers, shared


def _words(values: np.ndarray) -> np.ndarray:
    """BF16 words (nearest even) of float32 values."""
    return torch.from_numpy(np.ascontiguousarray(values, dtype=np.float32)).to(torch.bfloat16).view(torch.int16) \
        .numpy().view(np.uint16)


def random_token_ids(seed: int, count: int, vocab: int = GPT2_SMALL.vocab) -> np.ndarray:
    """Seeded token ids, uniform in [0, vocab)."""
    return np.random.default_rng(seed).integers(0, vocab, size=count, dtype=np.int64)
