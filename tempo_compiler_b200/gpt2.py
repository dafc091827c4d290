"""GPT-2 small's per-32-token-block layer drivers over the drop-in runtime: the reference-facing host path.

This mirrors the reference's ``board_package/gpt2_inference.py`` (names, argument meaning, device layouts and error
behaviour) so that its callers, and ports of its board checks, run unchanged on a B200: device tensors in the
packed block-major layout (``DeviceTensor``, gpt2_inference.py:136-196), slices of a fused QKV tensor
(``DeviceTensorSlice``, :199-230), the per-layer KV cache filled by copy images (``KVCache``, :233-302), one launch per
32-token block for the GEMM, LayerNorm and add images and one per sequence for attention. Every launch goes through
``tempo_compiler_b200.runtime.minitpuLaunchKernel``, i.e. through the C ABI, onto the B200 kernels.

The batched, resident-weight engine the benchmarks use is ``tempo_compiler_b200.engine``; this module is the drop-in.
"""

from __future__ import annotations

import json
import math
import pathlib
import time
from collections.abc import Callable

import numpy as np
from numpy.typing import NDArray

from tempo_compiler_b200 import images as _images
from tempo_compiler_b200.runtime import (
    MemcpyKind,
    minitpuFree,
    minitpuHostAlloc,
    minitpuHostReset,
    minitpuLaunchKernel,
    minitpuMalloc,
    minitpuMemcpy,
    minitpuSetDevice,
)

TILE = 16
BLOCK_TOKENS = 32
ELEMENT_BYTES = 2
ROW_BYTES = TILE * ELEMENT_BYTES
ZERO_TILE_WORDS = TILE * TILE
ZERO_TILE_BYTES = ZERO_TILE_WORDS * ELEMENT_BYTES
BLOCK_WEIGHT_BYTES = 2 * TILE * ROW_BYTES      # one 32-deep block of a weight column tile (bf16.py:63)
BLOCK_ACTIVATION_BYTES = 2 * 2 * TILE * ROW_BYTES
VREG_ELEMENTS = 64
MODEL_WIDTH = 768
MAX_CONTEXT = 1024
END_OF_TEXT = 50256
UIO_NAME = "minitpu"

IMAGE_DIRECTORY: pathlib.Path = _images.DEFAULT_DIRECTORY
"""The image set these drivers launch from; written on first use (tempo_compiler_b200/images.py)."""

_TENSOR_POOL: dict[tuple[int, int], list[int]] = {}
_RESIDENT_IMAGES: dict[bytes, int] = {}
_COMPILED_IMAGES: dict[tuple, tuple[bytes, dict]] = {}
_ATTENTION_CONSTANTS: dict[str, int] = {}
_DECODE_CONSTANTS: dict[int, int] = {}
_DEVICE_CLOCK: list[float] = [0.0]


# ---------------------------------------------------------------------------------------------------------------
# BF16 and the packed layouts on the host
# ---------------------------------------------------------------------------------------------------------------

def bf16_words(values) -> NDArray[np.uint16]:
    """Nearest-even BF16 words of float32 values."""
    bits = np.ascontiguousarray(values, dtype="<f4").view("<u4")
    return ((bits + np.uint32(0x7FFF) + ((bits >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype("<u2")


def bf16_floats(words) -> NDArray[np.float32]:
    return (np.asarray(words).astype("<u4") << np.uint32(16)).view("<f4")


def on_bf16_grid(values) -> NDArray[np.float32]:
    array = np.asarray(values, dtype=np.float32)
    return bf16_floats(bf16_words(array.reshape(-1))).reshape(array.shape)


def _padded(values: NDArray[np.float32]) -> NDArray[np.float32]:
    short = -values.shape[-1] % TILE
    return values if not short else np.pad(values, [(0, 0)] * (values.ndim - 1) + [(0, short)])


def pack_activations(activations) -> NDArray[np.uint16]:
    """[tokens, depth] -> [depth/16][tokens][16] words (bf16.py:133-156)."""
    activations = np.asarray(activations, dtype=np.float32)
    if activations.shape[0] % TILE:
        raise ValueError(f"Unable to pack an activation array of shape {list(activations.shape)}. Its rows must be a "
                         f"whole number of the {TILE} a token group holds.")
    padded = _padded(activations)
    words = bf16_words(padded).reshape(padded.shape[0], -1, TILE)
    return np.ascontiguousarray(words.transpose(1, 0, 2)).reshape(-1)


def pack_weights(weights) -> NDArray[np.uint16]:
    """[depth, columns] -> [columns/16][depth][16] words (bf16.py:178-192)."""
    padded = _padded(_padded(np.asarray(weights, dtype=np.float32)).T).T
    words = bf16_words(padded).reshape(padded.shape[0], -1, TILE)
    return np.ascontiguousarray(words.transpose(1, 0, 2)).reshape(-1)


def pack_bias(bias) -> NDArray[np.uint16]:
    """[columns] -> [columns/16][4][16] words (bf16.py:159-175)."""
    bias = np.asarray(bias, dtype=np.float32)
    if bias.ndim != 1:
        raise ValueError(f"Unable to pack a bias of shape {bias.shape}. It must be one row.")
    tiles = bf16_words(_padded(bias)).reshape(-1, TILE)
    return np.ascontiguousarray(np.repeat(tiles, 4, axis=0)).reshape(-1)


def decode_mask_tiles(*, keys: int, length: int) -> NDArray[np.float32]:
    """[1, keys/16, 16, 16] mask tiles keeping the first `length` keys (bf16.py:195-207)."""
    row = np.where(np.arange(keys) < length, np.float32(0.0), np.float32(-1.0e30)).astype(np.float32)
    return np.ascontiguousarray(np.broadcast_to(row.reshape(1, keys // TILE, 1, TILE), (1, keys // TILE, TILE, TILE)))


def pack_attention_constants(*, initial_maximum: float, constants: tuple[float, ...], masks) -> NDArray[np.uint16]:
    """Per query block: entering-maximum tile, zero tile, stated tiles, mask tiles; BF16 (bf16.py:210-225)."""
    blocks = []
    for block in np.asarray(masks, dtype=np.float32):
        tiles = [np.full((TILE, TILE), initial_maximum, np.float32), np.zeros((TILE, TILE), np.float32)]
        tiles += [np.full((TILE, TILE), c, np.float32) for c in constants]
        blocks.append(np.concatenate(tiles + list(block), axis=0))
    return bf16_words(np.concatenate(blocks, axis=0))


# ---------------------------------------------------------------------------------------------------------------
# Device tensors
# ---------------------------------------------------------------------------------------------------------------

class ResidentWeights:
    """A packed matrix (or bias row) resident in device memory (gpt2_inference.py:104-133)."""

    def __init__(self, address: int, depth: int, columns: int, nbytes: int) -> None:
        self.address, self.depth, self.columns, self.nbytes = address, depth, columns, nbytes

    @property
    def shape(self) -> tuple[int, int]:
        return (self.depth, self.columns)

    def free(self) -> None:
        if self.address is not None:
            minitpuFree(self.address)
            self.address = None


class DeviceTensor:
    """Packed activations: per 32-token block a zeroed 16x16 tile then [features/16][32][16] (gpt2_inference.py:136-196)."""

    def __init__(self, base: int, tokens: int, features: int) -> None:
        self.base, self.tokens, self.features = base, tokens, features

    @property
    def blocks(self) -> int:
        return self.tokens // BLOCK_TOKENS

    @property
    def block_bytes(self) -> int:
        return ZERO_TILE_BYTES + BLOCK_TOKENS * self.features * ELEMENT_BYTES

    def d_drain(self, block: int) -> int:
        return self.base + block * self.block_bytes

    def operand(self, block: int) -> int:
        return self.d_drain(block) + ZERO_TILE_BYTES

    @property
    def address(self) -> int:
        return self.operand(0)

    @property
    def shape(self) -> tuple[int, int]:
        return (self.tokens, self.features)

    @property
    def nbytes(self) -> int:
        return self.blocks * self.block_bytes

    def free(self) -> None:
        """Returns the tensor to the shape-keyed pool; its clearing tiles stay zero (gpt2_inference.py:186-196)."""
        if self.base is not None:
            _TENSOR_POOL.setdefault((self.tokens, self.features), []).append(self.base)
            self.base = None


class DeviceTensorSlice:
    """A run of feature tiles of a packed tensor, addressed in its parent's blocks (gpt2_inference.py:199-230)."""

    def __init__(self, d_parent: DeviceTensor, first_tile: int, features: int) -> None:
        self._d_parent = d_parent
        self._offset = first_tile * BLOCK_TOKENS * TILE * ELEMENT_BYTES
        self.tokens = d_parent.tokens
        self.features = features

    @property
    def blocks(self) -> int:
        return self._d_parent.blocks

    @property
    def shape(self) -> tuple[int, int]:
        return (self.tokens, self.features)

    def operand(self, block: int) -> int:
        return self._d_parent.operand(block) + self._offset


class KVCache:
    """One layer's keys then values per token, in the packed layout, filled by copy images (gpt2_inference.py:233-302)."""

    def __init__(self, capacity: int, model: int = MODEL_WIDTH) -> None:
        self.tensor = _allocate_tensor(capacity, 2 * model)
        self.length = 0

    def extend(self, d_fused: DeviceTensor, *, tokens: int | None = None) -> None:
        """Copies a prefill's keys and values after the tokens already held."""
        tokens = d_fused.tokens if tokens is None else tokens
        if self.length % BLOCK_TOKENS or self.length + d_fused.tokens > self.tensor.tokens:
            raise ValueError(f"Unable to extend a cache holding {self.length} of {self.tensor.tokens} tokens by "
                             f"{d_fused.tokens}. A prefill fills whole token blocks, so the cache must hold whole "
                             f"blocks and have room for them.")
        rows = self.tensor.features // TILE * BLOCK_TOKENS
        first = self.length // BLOCK_TOKENS
        for block in range(d_fused.blocks):
            _launch_copy(rows=rows, stride=ROW_BYTES, source=d_fused.operand(block) + self._keys_offset(d_fused),
                         destination=self.tensor.operand(first + block))
        self.length += tokens

    def append(self, d_fused: DeviceTensor) -> None:
        """Copies a decode step's new token (row 0 of its fused QKV) into the next slot."""
        if self.length >= self.tensor.tokens:
            raise ValueError(f"Unable to append to a cache holding all {self.tensor.tokens} tokens it has room for.")
        block, row = divmod(self.length, BLOCK_TOKENS)
        _launch_copy(rows=self.tensor.features // TILE, stride=BLOCK_TOKENS * ROW_BYTES,
                     source=d_fused.operand(0) + self._keys_offset(d_fused),
                     destination=self.tensor.operand(block) + row * ROW_BYTES)
        self.length += 1

    def free(self) -> None:
        self.tensor.free()

    @staticmethod
    def _keys_offset(d_fused: DeviceTensor) -> int:
        return d_fused.features // 3 // TILE * BLOCK_TOKENS * ROW_BYTES


# ---------------------------------------------------------------------------------------------------------------
# Uploads and downloads
# ---------------------------------------------------------------------------------------------------------------

def _upload_words(words: NDArray[np.uint16], extra: int = 0) -> int:
    minitpuSetDevice(UIO_NAME)
    host = minitpuHostAlloc(words.nbytes)
    host.view.view("<u2")[: words.size] = words
    address = minitpuMalloc(words.nbytes + extra)
    minitpuMemcpy(address, host, words.nbytes, MemcpyKind.HostToDevice)
    minitpuHostReset()
    return address


def upload_weights(h_weights) -> ResidentWeights:
    """Packs a [depth, columns] matrix and leaves it resident (gpt2_inference.py:345-364)."""
    words = pack_weights(on_bf16_grid(np.asarray(h_weights, dtype=np.float32)))
    address = _upload_words(words, BLOCK_WEIGHT_BYTES)
    return ResidentWeights(address=address, depth=h_weights.shape[0], columns=h_weights.shape[1], nbytes=words.nbytes)


def upload_bias(h_bias) -> ResidentWeights:
    """Uploads one feature row, each tile repeated four times (gpt2_inference.py:367-386)."""
    h_bias = np.asarray(h_bias)
    if h_bias.ndim != 1 or h_bias.size % TILE:
        raise ValueError(f"Unable to upload bias shape {h_bias.shape}. It must be one row of whole {TILE}-lane tiles.")
    words = pack_bias(on_bf16_grid(h_bias.astype(np.float32)))
    return ResidentWeights(address=_upload_words(words), depth=1, columns=h_bias.size, nbytes=words.nbytes)


def upload_activations(h_activations) -> DeviceTensor:
    """Packs [tokens, features] host activations into a resident tensor (gpt2_inference.py:389-407)."""
    h_activations = np.asarray(h_activations, dtype=np.float32)
    tokens, features = h_activations.shape
    grid = on_bf16_grid(h_activations)
    d_tensor = _allocate_tensor(tokens, features)
    for block in range(d_tensor.blocks):
        words = pack_activations(grid[block * BLOCK_TOKENS:(block + 1) * BLOCK_TOKENS])
        staging = minitpuHostAlloc(words.nbytes)
        staging.view.view("<u2")[: words.size] = words
        minitpuMemcpy(d_tensor.operand(block), staging, words.nbytes, MemcpyKind.HostToDevice)
    minitpuHostReset()
    return d_tensor


def download_activations(d_tensor) -> NDArray[np.float32]:
    """Reads a resident tensor back as row-major float32 (gpt2_inference.py:410-432)."""
    per_block = BLOCK_TOKENS * d_tensor.features
    out = np.empty((d_tensor.tokens, d_tensor.features), dtype=np.float32)
    for block in range(d_tensor.blocks):
        staging = minitpuHostAlloc(per_block * ELEMENT_BYTES)
        minitpuMemcpy(staging, d_tensor.operand(block), per_block * ELEMENT_BYTES, MemcpyKind.DeviceToHost)
        values = bf16_floats(staging.view.view("<u2")[:per_block])
        tiles = values.reshape(d_tensor.features // TILE, BLOCK_TOKENS, TILE)
        out[block * BLOCK_TOKENS:(block + 1) * BLOCK_TOKENS] = tiles.transpose(1, 0, 2).reshape(BLOCK_TOKENS, -1)
    minitpuHostReset()
    return out


def upload_layernorm_constants(h_gamma, h_beta) -> int:
    """Uploads gamma, beta and the manifest's scalars, each broadcast over 64 values (gpt2_inference.py:439-471)."""
    _, entry = _compiled_image(kind="layernorm", features=int(np.asarray(h_gamma).size))
    if entry["rows"] != ["gamma_pointer", "beta_pointer"]:
        raise ValueError(f"Unable to pack the constants of a LayerNorm image reading the rows {entry['rows']}.")
    broadcast = [np.full(VREG_ELEMENTS, s, dtype=np.float32) for s in entry["scalars"]]
    words = bf16_words(np.concatenate([np.asarray(h_gamma, np.float32), np.asarray(h_beta, np.float32), *broadcast]))
    return _upload_words(words)


# ---------------------------------------------------------------------------------------------------------------
# Resident ops: one launch per 32-token block
# ---------------------------------------------------------------------------------------------------------------

def layernorm_resident(d_rows: DeviceTensor, d_constants: int, *, d_out: DeviceTensor | None = None) -> DeviceTensor:
    """LayerNorm through the layernorm image, per block (gpt2_inference.py:474-503)."""
    image, _ = _compiled_image(kind="layernorm", features=d_rows.features)
    d_out = d_out or _allocate_tensor(d_rows.tokens, d_rows.features)
    d_image = _stage_image(image)
    for block in range(d_rows.blocks):
        _launch(d_image, len(image), args=[d_rows.operand(block), d_constants, d_out.operand(block)])
    return d_out


def add_resident(d_left, d_right, *, d_out: DeviceTensor | None = None) -> DeviceTensor:
    """Elementwise sum of two resident tensors, per block (gpt2_inference.py:506-541)."""
    if d_left.shape != d_right.shape:
        raise ValueError(f"Unable to add a {d_left.shape} tensor to a {d_right.shape} one. Elementwise addition needs "
                         f"the same shape.")
    image, _ = _compiled_image(kind="add", features=d_left.features)
    d_out = d_out or _allocate_tensor(d_left.tokens, d_left.features)
    d_image = _stage_image(image)
    for block in range(d_left.blocks):
        _launch(d_image, len(image), args=[d_left.operand(block), d_right.operand(block), d_out.operand(block)])
    return d_out


def add_bias_resident(d_left, d_bias: ResidentWeights, *, d_out: DeviceTensor | None = None) -> DeviceTensor:
    """Adds one resident bias row to every token row (gpt2_inference.py:544-571)."""
    if d_bias.depth != 1 or d_bias.columns != d_left.features:
        raise ValueError(f"Unable to broadcast bias {d_bias.shape} over {d_left.shape}. The bias must be one row with "
                         f"the tensor's feature width.")
    image, _ = _compiled_image(kind="add_bias", features=d_left.features)
    d_out = d_out or _allocate_tensor(d_left.tokens, d_left.features)
    d_image = _stage_image(image)
    for block in range(d_left.blocks):
        _launch(d_image, len(image), args=[d_left.operand(block), d_bias.address, d_out.operand(block)])
    return d_out


def gemm_resident(d_activations, d_weights: ResidentWeights, *, activate: bool = False,
                  d_bias: ResidentWeights | None = None, d_out: DeviceTensor | None = None) -> DeviceTensor:
    """Product of two resident operands, one launch per block (gpt2_inference.py:574-640)."""
    tokens, depth = d_activations.shape
    columns = d_weights.columns
    if depth != d_weights.depth:
        raise ValueError(f"Unable to multiply a [{tokens},{depth}] tensor by a [{d_weights.depth},{columns}] one. "
                         f"Their inner dimensions must agree.")
    for name, value, block in (("tokens", tokens, BLOCK_TOKENS), ("columns", columns, TILE)):
        if value % block:
            raise ValueError(f"Unable to multiply tensors with {name} of {value}. It must be a whole number of {block}, "
                             f"which is what one launch covers.")
    fused = d_bias is not None and _has_image(kind="gemm_bias", depth=depth, columns=columns, activate=activate)
    if d_bias is not None and not fused:
        d_product = gemm_resident(d_activations, d_weights, activate=activate)
        try:
            return add_bias_resident(d_product, d_bias, d_out=d_out)
        finally:
            d_product.free()
    image = _compiled_gemm(depth=depth, columns=columns, activate=activate, bias=fused)
    d_out = d_out or _allocate_tensor(tokens, columns)
    d_image = _stage_image(image)
    bias_args = [d_bias.address] if fused else []
    for block in range(tokens // BLOCK_TOKENS):
        _launch(d_image, len(image),
                args=[d_activations.operand(block), d_weights.address, d_out.d_drain(block), *bias_args])
    return d_out


def full_gemm(activations, weights, *, activate: bool = False) -> NDArray[np.float32]:
    """A host product through the GEMM image, one launch per 32-token block (gpt2_inference.py:643-746)."""
    activations = np.asarray(activations, dtype=np.float32)
    resident = weights if isinstance(weights, ResidentWeights) else None
    tokens, depth = activations.shape
    columns = weights.shape[1]
    if depth != weights.shape[0]:
        raise ValueError(f"Unable to multiply a [{tokens},{depth}] array by a [{weights.shape[0]},{columns}] array. "
                         f"Their inner dimensions must agree.")
    for name, value, block in (("tokens", tokens, BLOCK_TOKENS), ("depth", depth, 2 * TILE), ("columns", columns, TILE)):
        if value % block:
            raise ValueError(f"Unable to multiply arrays with {name} of {value}. It must be a whole number of {block}, "
                             f"which is what one launch covers.")
    fused = not _has_image(kind="gemm", depth=depth, columns=columns, activate=activate)
    image = _compiled_gemm(depth=depth, columns=columns, activate=activate, bias=fused)
    drain_words = ZERO_TILE_WORDS + columns // TILE * BLOCK_TOKENS * TILE
    result = np.empty((tokens, columns), dtype=np.float32)
    owned: list[int] = []
    try:
        d_bias = upload_bias(np.zeros(columns, dtype=np.float32)) if fused else None
        if d_bias is not None:
            owned.append(d_bias.address)
        d_image = _stage_image(image)
        if resident is not None:
            d_weights = resident.address
        else:
            d_weights = _upload_words(pack_weights(weights), BLOCK_WEIGHT_BYTES)
            owned.append(d_weights)
        d_drain = _upload_words(np.zeros(drain_words, dtype=np.uint16))
        owned.append(d_drain)
        d_acts = minitpuMalloc(BLOCK_TOKENS * depth * ELEMENT_BYTES + BLOCK_ACTIVATION_BYTES)
        owned.append(d_acts)
        for token in range(0, tokens, BLOCK_TOKENS):
            words = pack_activations(activations[token:token + BLOCK_TOKENS])
            staging = minitpuHostAlloc(words.nbytes)
            staging.view.view("<u2")[: words.size] = words
            minitpuMemcpy(d_acts, staging, words.nbytes, MemcpyKind.HostToDevice)
            _launch(d_image, len(image), args=[d_acts, d_weights, d_drain, *([d_bias.address] if fused else [])])
            drain = minitpuHostAlloc(drain_words * ELEMENT_BYTES)
            minitpuMemcpy(drain, d_drain, drain_words * ELEMENT_BYTES, MemcpyKind.DeviceToHost)
            tiles = bf16_floats(drain.view.view("<u2")[ZERO_TILE_WORDS:drain_words]).reshape(-1, BLOCK_TOKENS, TILE)
            result[token:token + BLOCK_TOKENS] = tiles.transpose(1, 0, 2).reshape(BLOCK_TOKENS, columns)
            minitpuHostReset()
    finally:
        for address in owned:
            minitpuFree(address)
        minitpuHostReset()
    return result


def attention(d_fused: DeviceTensor, *, heads: int = 12) -> DeviceTensorSlice:
    """Causal attention of every head in one launch, output over the queries (gpt2_inference.py:981-1003)."""
    image, entry = _compiled_image(kind="attention", tokens=d_fused.tokens, heads=heads)
    d_constants = _attention_constants(entry)
    _launch(_stage_image(image), len(image), args=[d_constants, 0, d_fused.operand(0)])
    return DeviceTensorSlice(d_fused, 0, d_fused.features // 3)


def decode_attention(d_fused: DeviceTensor, cache: KVCache, *, heads: int = 12) -> DeviceTensorSlice:
    """The step's token over the cache through the shortest decode image holding it (gpt2_inference.py:1006-1039)."""
    built = sorted(e["keys"] for e in _manifest().values() if e["kind"] == "decode_attention" and e["heads"] == heads)
    keys = next((k for k in built if k >= cache.length), None)
    if cache.length < 1 or keys is None or keys > cache.tensor.tokens:
        raise ValueError(f"Unable to attend over a cache holding {cache.length} of {cache.tensor.tokens} tokens with "
                         f"decode images over {built} keys.")
    image, entry = _compiled_image(kind="decode_attention", keys=keys, heads=heads)
    d_constants = _decode_constants(entry, length=cache.length)
    _launch(_stage_image(image), len(image), args=[d_constants, cache.tensor.operand(0), d_fused.operand(0)])
    return DeviceTensorSlice(d_fused, 0, d_fused.features // 3)


# ---------------------------------------------------------------------------------------------------------------
# Layers and the model
# ---------------------------------------------------------------------------------------------------------------

def _run_layer(hidden, weights: dict, *, heads: int, attend: Callable[[DeviceTensor], DeviceTensorSlice]):
    """One block around the given attention, every intermediate resident (gpt2_inference.py:1133-1189)."""
    hidden = np.asarray(hidden, dtype=np.float32)
    model = hidden.shape[1]
    scale = np.ones(3 * model, dtype=np.float32)
    scale[:model] = 1.0 / math.sqrt(model // heads)
    owned: list = []
    constants: list[int] = []

    def kept(item):
        owned.append(item)
        return item

    try:
        d_weights = {n: kept(upload_weights(weights[n] * (scale if n == "attn.qkv.w" else 1.0)))
                     for n in ("attn.qkv.w", "attn.proj.w", "mlp.fc.w", "mlp.proj.w")}
        d_biases = {n: kept(upload_bias(weights[n] * (scale if n == "attn.qkv.b" else 1.0)))
                    for n in ("attn.qkv.b", "attn.proj.b", "mlp.fc.b", "mlp.proj.b")}
        for gamma, beta in (("ln_1.g", "ln_1.b"), ("ln_2.g", "ln_2.b")):
            constants.append(upload_layernorm_constants(weights[gamma], weights[beta]))
        d_hidden = kept(upload_activations(hidden))
        d_normed = kept(layernorm_resident(d_hidden, constants[0]))
        d_fused = kept(gemm_resident(d_normed, d_weights["attn.qkv.w"], d_bias=d_biases["attn.qkv.b"]))
        d_attended = attend(d_fused)
        d_projected = kept(gemm_resident(d_attended, d_weights["attn.proj.w"], d_bias=d_biases["attn.proj.b"]))
        d_residual = kept(add_resident(d_hidden, d_projected))
        d_normed = kept(layernorm_resident(d_residual, constants[1]))
        d_wide = kept(gemm_resident(d_normed, d_weights["mlp.fc.w"], d_bias=d_biases["mlp.fc.b"]))
        d_narrow = kept(gemm_resident(d_wide, d_weights["mlp.proj.w"], activate=True, d_bias=d_biases["mlp.proj.b"]))
        return download_activations(kept(add_resident(d_residual, d_narrow)))
    finally:
        for item in owned:
            item.free()
        for address in constants:
            minitpuFree(address)


def transformer_block(hidden, weights: dict, *, heads: int = 12, cache: KVCache | None = None,
                      valid: int | None = None) -> NDArray[np.float32]:
    """One block over a sequence, filling the cache from its keys and values (gpt2_inference.py:749-772)."""
    def attend(d_fused: DeviceTensor) -> DeviceTensorSlice:
        if cache is not None:
            cache.extend(d_fused, tokens=valid)
        return attention(d_fused, heads=heads)
    return _run_layer(hidden, weights, heads=heads, attend=attend)


def decode_block(hidden, weights: dict, cache: KVCache, *, heads: int = 12) -> NDArray[np.float32]:
    """One new token through one block, padded to a 32-token block (gpt2_inference.py:775-797)."""
    padded = np.zeros((BLOCK_TOKENS, np.asarray(hidden).shape[-1]), dtype=np.float32)
    padded[0] = hidden

    def attend(d_fused: DeviceTensor) -> DeviceTensorSlice:
        cache.append(d_fused)
        return decode_attention(d_fused, cache, heads=heads)
    return _run_layer(padded, weights, heads=heads, attend=attend)[0]


def embed(token_ids, shared: dict, *, start: int = 0) -> NDArray[np.float32]:
    """Token plus position embeddings on the host (gpt2_inference.py:800-812)."""
    positions = start + np.arange(len(token_ids))
    return (shared["wte"][np.asarray(token_ids)] + shared["wpe"][positions]).astype(np.float32)


def prefill(token_ids, layers: list[dict], shared: dict, *, heads: int = 12, capacity: int = MAX_CONTEXT,
            observe=None) -> tuple[NDArray[np.float32], list[KVCache]]:
    """The prompt through every layer, padded to the shortest attention image, filling the caches
    (gpt2_inference.py:815-862)."""
    tokens = len(token_ids)
    lengths = sorted(e["tokens"] for e in _manifest().values() if e["kind"] == "attention")
    padded = next((length for length in lengths if length >= tokens), None)
    if padded is None or padded > capacity:
        raise ValueError(f"Unable to prefill a prompt of {tokens} tokens. A compiled attention image covers "
                         f"{', '.join(map(str, lengths))} tokens and the caches hold {capacity}.")
    ids = np.concatenate([np.asarray(token_ids, dtype=np.int64), np.full(padded - tokens, END_OF_TEXT, np.int64)])
    hidden = embed(ids, shared)
    caches = [KVCache(capacity=capacity) for _ in layers]
    try:
        for index, (weights, cache) in enumerate(zip(layers, caches, strict=True)):
            layer_input = hidden
            hidden = transformer_block(hidden, weights, heads=heads, cache=cache, valid=tokens)
            if observe is not None:
                observe(index, layer_input, hidden)
    except BaseException:
        for cache in caches:
            cache.free()
        raise
    return hidden[:tokens], caches


def decode_step(token_id: int, layers: list[dict], shared: dict, caches: list[KVCache], *, heads: int = 12,
                observe=None) -> NDArray[np.float32]:
    """One new token through every layer (gpt2_inference.py:865-887)."""
    hidden = embed(np.asarray([token_id]), shared, start=caches[0].length)[0]
    for index, (weights, cache) in enumerate(zip(layers, caches, strict=True)):
        layer_input = hidden
        hidden = decode_block(hidden, weights, cache, heads=heads)
        if observe is not None:
            observe(index, layer_input, hidden)
    return hidden


def final_layernorm(hidden, shared: dict) -> NDArray[np.float32]:
    """GPT-2's final LayerNorm on the device (gpt2_inference.py:890-912)."""
    hidden = np.asarray(hidden, dtype=np.float32)
    tokens = hidden.shape[0]
    padded = np.zeros((-(-tokens // BLOCK_TOKENS) * BLOCK_TOKENS, hidden.shape[1]), dtype=np.float32)
    padded[:tokens] = hidden
    d_rows, d_constants = upload_activations(padded), upload_layernorm_constants(shared["ln_f.g"], shared["ln_f.b"])
    try:
        d_normed = layernorm_resident(d_rows, d_constants)
        try:
            return download_activations(d_normed)[:tokens]
        finally:
            d_normed.free()
    finally:
        d_rows.free()
        minitpuFree(d_constants)


def lm_head(normalised, shared: dict) -> NDArray[np.float32]:
    """Logits through the tied embedding, on the host (gpt2_inference.py:915-925)."""
    return np.asarray(normalised, dtype=np.float32) @ shared["wte"].T


def next_token_logits(hidden, shared: dict) -> NDArray[np.float32]:
    return lm_head(final_layernorm(np.asarray(hidden)[None, :], shared)[0], shared)


def generate(token_ids, layers: list[dict], shared: dict, *, new_tokens: int, heads: int = 12,
             capacity: int = MAX_CONTEXT) -> list[int]:
    """Greedy continuation: prefill, then one decode step per token (gpt2_inference.py:941-978)."""
    if len(token_ids) + new_tokens > capacity:
        raise ValueError(f"Unable to generate {new_tokens} tokens after a {len(token_ids)}-token prompt. The caches "
                         f"hold {capacity} tokens, so ask for fewer.")
    hidden, caches = prefill(token_ids, layers, shared, heads=heads, capacity=capacity)
    generated: list[int] = []
    try:
        logits = next_token_logits(hidden[-1], shared)
        while len(generated) < new_tokens:
            token = int(np.argmax(logits))
            generated.append(token)
            if token == END_OF_TEXT or len(generated) == new_tokens:
                break
            logits = next_token_logits(decode_step(token, layers, shared, caches, heads=heads), shared)
    finally:
        for cache in caches:
            cache.free()
    return generated


def npu_seconds() -> float:
    """Seconds spent inside launches so far (gpt2_inference.py:305-307)."""
    return _DEVICE_CLOCK[0]


def halt_image() -> bytes:
    return _compiled_image(kind="halt")[0]


# ---------------------------------------------------------------------------------------------------------------
# Images
# ---------------------------------------------------------------------------------------------------------------

def _manifest() -> dict:
    directory = _images.ensure_image_set(IMAGE_DIRECTORY)
    return json.loads((directory / "manifest.json").read_text())


def _compiled_image(*, kind: str, **shape) -> tuple[bytes, dict]:
    """The image of one kind and shape and its manifest entry (gpt2_inference.py:1072-1102)."""
    key = (kind, *sorted(shape.items()))
    cached = _COMPILED_IMAGES.get(key)
    if cached is not None:
        return cached
    manifest = _manifest()
    found = next((name for name, entry in manifest.items()
                  if entry["kind"] == kind and all(entry.get(f) == v for f, v in shape.items())), None)
    if found is None:
        stated = ", ".join(f"{f}={v}" for f, v in shape.items())
        raise ValueError(f"Unable to launch the {kind} image with {stated}. No image in {IMAGE_DIRECTORY} covers that "
                         f"shape.")
    cached = ((IMAGE_DIRECTORY / found).read_bytes(), manifest[found])
    _COMPILED_IMAGES[key] = cached
    return cached


def _compiled_gemm(*, depth: int, columns: int, activate: bool, bias: bool = False) -> bytes:
    image, entry = _compiled_image(kind="gemm_bias" if bias else "gemm", depth=depth, columns=columns,
                                   activate=activate)
    expected = ZERO_TILE_WORDS + columns // TILE * BLOCK_TOKENS * TILE
    if entry["drain_words"] != expected:
        raise ValueError(f"Unable to launch the [{depth}, {columns}] GEMM image. A product drains {expected} words, "
                         f"but the image drains {entry['drain_words']}.")
    return image


def _has_image(*, kind: str, **shape) -> bool:
    return any(e["kind"] == kind and all(e.get(f) == v for f, v in shape.items()) for e in _manifest().values())


def _attention_constants(entry: dict) -> int:
    cached = _ATTENTION_CONSTANTS.get(entry["constants"])
    if cached is not None:
        return cached
    words = np.frombuffer((IMAGE_DIRECTORY / entry["constants"]).read_bytes(), dtype="<u2")
    address = _upload_words(words)
    _ATTENTION_CONSTANTS[entry["constants"]] = address
    return address


def _decode_constants(entry: dict, *, length: int) -> int:
    """Writes a decode step's constants, masking keys past `length` (gpt2_inference.py:1212-1237)."""
    keys = entry["keys"]
    masks = decode_mask_tiles(keys=keys, length=length)
    if entry.get("transposed_masks", False):
        masks = np.ascontiguousarray(masks.swapaxes(-1, -2))
    words = pack_attention_constants(initial_maximum=entry["entering"], constants=tuple(entry["stated"]),
                                     masks=masks).reshape(-1)
    address = _DECODE_CONSTANTS.get(keys)
    if address is None:
        address = minitpuMalloc(words.nbytes)
        _DECODE_CONSTANTS[keys] = address
    staging = minitpuHostAlloc(words.nbytes)
    staging.view.view("<u2")[: words.size] = words
    minitpuMemcpy(address, staging, words.nbytes, MemcpyKind.HostToDevice)
    minitpuHostReset()
    return address


def _stage_image(image: bytes) -> int:
    """Makes an image resident once, keyed by its bytes (gpt2_inference.py:1240-1259)."""
    resident = _RESIDENT_IMAGES.get(image)
    if resident is not None:
        return resident
    minitpuSetDevice(UIO_NAME)
    address = minitpuMalloc(len(image))
    host = minitpuHostAlloc(len(image))
    host.view[: len(image) // 4] = np.frombuffer(image, dtype="<u4")
    minitpuMemcpy(address, host, len(image), MemcpyKind.HostToDevice)
    _RESIDENT_IMAGES[image] = address
    return address


def _launch(image: int, size: int, *, args: list[int]) -> None:
    started = time.perf_counter()
    minitpuLaunchKernel(image, size, args=args)
    _DEVICE_CLOCK[0] += time.perf_counter() - started


def _launch_copy(*, rows: int, stride: int, source: int, destination: int) -> None:
    image, _ = _compiled_image(kind="copy", rows=rows, stride=stride)
    _launch(_stage_image(image), len(image), args=[source, 0, destination])


def _allocate_tensor(tokens: int, features: int) -> DeviceTensor:
    """A drain-shaped device tensor, from the pool when one waits; clearing tiles zeroed once (gpt2_inference.py:1262-1297)."""
    if tokens % BLOCK_TOKENS:
        raise ValueError(f"Unable to hold {tokens} rows in device memory. A tensor is a whole number of "
                         f"{BLOCK_TOKENS}-row blocks, which is what one launch covers.")
    waiting = _TENSOR_POOL.get((tokens, features))
    if waiting:
        return DeviceTensor(base=waiting.pop(), tokens=tokens, features=features)
    minitpuSetDevice(UIO_NAME)
    tensor = DeviceTensor(base=0, tokens=tokens, features=features)
    tensor.base = minitpuMalloc(tensor.nbytes)
    host = minitpuHostAlloc(ZERO_TILE_BYTES)
    host.view.view("<u2")[:ZERO_TILE_WORDS] = 0
    for block in range(tensor.blocks):
        minitpuMemcpy(tensor.d_drain(block), host, ZERO_TILE_BYTES, MemcpyKind.HostToDevice)
    minitpuHostReset()
    return tensor


def reset_state() -> None:
    """Forgets every cached device address (after the runtime's device reset)."""
    for table in (_TENSOR_POOL, _RESIDENT_IMAGES, _ATTENTION_CONSTANTS, _DECODE_CONSTANTS):
        table.clear()
