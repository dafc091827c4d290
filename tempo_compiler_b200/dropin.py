"""GPT-2 small driven through the drop-in runtime, one image launch per 32-token block.

The reference runs GPT-2 from a numpy driver (``board_package/gpt2_inference.py``) that stages images and launches
them through a module named ``runtime`` with packed block-major operands. That driver runs unchanged over
``tempo_compiler_b200.runtime`` (installed as ``sys.modules["runtime"]`` before it is imported). This module drives
the same launch contract from this project's side, so the contract can be exercised and used where the reference's
tree is not installed. Its shape is its own:

* every layout of the contract is one of three host transforms (``tile_major``, ``bias_rows``, ``mask_tiles``);
* ``ImageSet`` looks images up by manifest kind and fields and stages each one once;
* ``Session`` scopes device memory: everything it allocates is released by ``close()``;
* ``PackedGPT2`` uploads a model's weights once, keeps the hidden state resident from the embedding to the final
  LayerNorm (only the last row block comes back for the LM head), reuses one workspace per padded token count and
  runs each layer as a list of (image, arguments) launches.

Launch contract (``mlir/lib/tempo/manifest.cpp:103-167``; argument slots as the runtime's dispatcher binds them):
``gemm_bias`` [A rows, weights, output drain, bias]; ``add`` / ``add_bias`` [left, right or bias, out];
``layernorm`` [rows, constants, out]; ``attention`` [constants, 0, fused rows]; ``decode_attention``
[constants, cache rows, fused rows]; ``copy`` [source, 0, destination].
"""

from __future__ import annotations

import json
import math
import pathlib
from collections.abc import Callable
from dataclasses import dataclass, field

import numpy as np
from numpy.typing import NDArray

from tempo_compiler_b200 import images as _images
from tempo_compiler_b200 import runtime as rt

LANES = 16                 # values in one 32-byte row of a tile: the unit every packed layout is built from
BLOCK = 32                 # token rows one block launch covers
CLEAR_BYTES = 512          # the zeroed 16 x 16 tile heading every packed block (a GEMM's drain target)
WIDTH = 768                # GPT-2 small's model width
HEAD = 64
CONTEXT = 1024             # learned positions, hence the longest sequence
END_OF_TEXT = 50256        # the token prompts are padded with
MASKED = -1.0e30           # the score a mask tile adds to an excluded key

Observer = Callable[[int, NDArray[np.float32], NDArray[np.float32]], None]


# ---------------------------------------------------------------------------------------------------------------
# Host side of the layouts
# ---------------------------------------------------------------------------------------------------------------

def to_words(values) -> NDArray[np.uint16]:
    """Nearest-even BF16 words of float32 values (ties to the even word)."""
    bits = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32)
    return ((bits + ((bits >> 16) & 1) + 0x7FFF) >> 16).astype(np.uint16)


def to_floats(words) -> NDArray[np.float32]:
    return (np.asarray(words, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def tile_major(matrix) -> NDArray[np.uint16]:
    """[rows, columns] -> [columns / 16][rows][16] BF16 words: one block's activations (``bf16.py:133-156``) and a
    whole weight matrix (``bf16.py:178-192``) are both this transform. Both axes pad with zeros to whole tiles."""
    matrix = np.asarray(matrix, dtype=np.float32)
    rows, columns = (-(-n // LANES) * LANES for n in matrix.shape)
    padded = np.zeros((rows, columns), np.float32)
    padded[: matrix.shape[0], : matrix.shape[1]] = matrix
    return to_words(padded).reshape(rows, -1, LANES).transpose(1, 0, 2).reshape(-1)


def from_tile_major(words, rows: int, columns: int) -> NDArray[np.float32]:
    """The inverse of :func:`tile_major` for whole tiles."""
    tiles = to_floats(np.asarray(words)[: rows * columns]).reshape(columns // LANES, rows, LANES)
    return tiles.transpose(1, 0, 2).reshape(rows, columns)


def bias_rows(bias) -> NDArray[np.uint16]:
    """[columns] -> [columns / 16][4][16]: each 16-value tile of the row four times (``bf16.py:159-175``)."""
    bias = np.asarray(bias, dtype=np.float32)
    if bias.ndim != 1 or bias.size % LANES:
        raise ValueError(f"Unable to lay out a bias of shape {bias.shape}. It must be one row of whole {LANES}-value "
                         f"tiles.")
    return np.repeat(to_words(bias).reshape(-1, 1, LANES), 4, axis=1).reshape(-1)


def norm_block(gamma, beta, scalars) -> NDArray[np.uint16]:
    """A LayerNorm constants block: gamma, beta, then each manifest scalar 64 times (``gpt2_inference.py:439-471``)."""
    parts = [np.asarray(gamma, np.float32), np.asarray(beta, np.float32)]
    parts += [np.full(64, s, np.float32) for s in scalars]
    return to_words(np.concatenate(parts))


def mask_tiles(*, keys: int, length: int, entering: float, stated=(), transposed: bool = True) -> NDArray[np.uint16]:
    """A decode step's constants (``bf16.py:195-225``): a tile of the entering maximum, a zero tile, one tile per
    stated constant, then one 16 x 16 mask tile per 16 keys, 0 for a key below `length` and -1e30 past it. The mask
    is the same for every query row, so with keys on the tile's rows (``transposed``) each row is one value."""
    head = [np.full(LANES * LANES, entering, np.float32), np.zeros(LANES * LANES, np.float32)]
    head += [np.full(LANES * LANES, c, np.float32) for c in stated]
    key_value = np.where(np.arange(keys) < length, 0.0, MASKED).astype(np.float32).reshape(-1, LANES)
    if transposed:
        tiles = np.repeat(key_value[:, :, None], LANES, axis=2)
    else:
        tiles = np.repeat(key_value[:, None, :], LANES, axis=1)
    return to_words(np.concatenate(head + [tiles.reshape(-1)]))


# ---------------------------------------------------------------------------------------------------------------
# Device memory
# ---------------------------------------------------------------------------------------------------------------

def _write(address: int, words: NDArray) -> None:
    data = np.ascontiguousarray(words).view(np.uint8).reshape(-1)
    region = rt.minitpuHostAlloc(data.size)
    region.view.view(np.uint8)[: data.size] = data
    rt.minitpuMemcpy(address, region, data.size, rt.MemcpyKind.HostToDevice)
    rt.minitpuHostReset()


def _read(address: int, nbytes: int) -> NDArray[np.uint8]:
    region = rt.minitpuHostAlloc(nbytes)
    rt.minitpuMemcpy(region, address, nbytes, rt.MemcpyKind.DeviceToHost)
    data = region.view.view(np.uint8)[:nbytes].copy()
    rt.minitpuHostReset()
    return data


@dataclass(frozen=True)
class Packed:
    """Packed activations in the arena: per 32-token block a zeroed tile, then [features / 16][32][16] BF16.

    ``rows(b, tile)`` addresses block b from feature tile `tile` on: with ``tile`` = 0 it is the operand a launch
    reads, and the first features / 16 tiles of a fused QKV block are its queries (an operand of their own)."""

    base: int
    tokens: int
    features: int

    @property
    def blocks(self) -> int:
        return self.tokens // BLOCK

    @property
    def stride(self) -> int:
        return CLEAR_BYTES + BLOCK * self.features * 2

    @property
    def nbytes(self) -> int:
        return self.blocks * self.stride

    def drain(self, block: int) -> int:
        return self.base + block * self.stride

    def rows(self, block: int, tile: int = 0) -> int:
        return self.drain(block) + CLEAR_BYTES + tile * BLOCK * LANES * 2


@dataclass(frozen=True)
class Resident:
    """A weight matrix [depth, columns] (tile-major), a bias (tile rows x4) or a LayerNorm constants block."""

    address: int
    depth: int
    columns: int


class Session:
    """Allocations through the runtime, all released by :meth:`close` (or on leaving a ``with`` block)."""

    def __init__(self) -> None:
        rt.minitpuSetDevice("minitpu")
        self._owned: list[int] = []

    def __enter__(self) -> Session:
        return self

    def __exit__(self, *_) -> None:
        self.close()

    def close(self) -> None:
        while self._owned:
            rt.minitpuFree(self._owned.pop())

    def malloc(self, nbytes: int) -> int:
        address = rt.minitpuMalloc(nbytes)
        self._owned.append(address)
        return address

    def put(self, words: NDArray) -> int:
        """Device copy of host words."""
        address = self.malloc(np.asarray(words).nbytes)
        _write(address, words)
        return address

    def packed(self, tokens: int, features: int) -> Packed:
        """A packed tensor whose clearing tiles (and rows) start at zero."""
        if tokens <= 0 or tokens % BLOCK or features % LANES:
            raise ValueError(f"Unable to hold [{tokens}, {features}] in the packed layout. Tokens must be a positive "
                             f"multiple of {BLOCK} and features a multiple of {LANES}.")
        tensor = Packed(0, tokens, features)
        tensor = Packed(self.malloc(tensor.nbytes), tokens, features)
        _write(tensor.base, np.zeros(tensor.nbytes, np.uint8))
        return tensor

    def rows_in(self, values, *, tensor: Packed | None = None) -> Packed:
        """Host rows [tokens, features] into a packed tensor (a new one unless given); tokens pad to whole blocks."""
        values = np.asarray(values, dtype=np.float32)
        tokens = -(-values.shape[0] // BLOCK) * BLOCK
        tensor = tensor or self.packed(tokens, values.shape[1])
        image = np.zeros((tensor.blocks, tensor.stride // 2), np.uint16)
        padded = np.zeros((tensor.tokens, tensor.features), np.float32)
        padded[: values.shape[0]] = values
        for b in range(tensor.blocks):
            image[b, CLEAR_BYTES // 2:] = tile_major(padded[b * BLOCK:(b + 1) * BLOCK])
        _write(tensor.base, image)
        return tensor

    @staticmethod
    def rows_out(tensor: Packed, *, blocks: range | None = None) -> NDArray[np.float32]:
        """Float32 rows of a packed tensor (all blocks, or the given ones)."""
        blocks = blocks if blocks is not None else range(tensor.blocks)
        data = _read(tensor.drain(blocks.start), len(blocks) * tensor.stride).view(np.uint16)
        per_block = data.reshape(len(blocks), tensor.stride // 2)[:, CLEAR_BYTES // 2:]
        return np.concatenate([from_tile_major(w, BLOCK, tensor.features) for w in per_block])

    def matrix(self, weights) -> Resident:
        weights = np.asarray(weights, dtype=np.float32)
        return Resident(self.put(tile_major(weights)), weights.shape[0], weights.shape[1])

    def bias(self, values) -> Resident:
        return Resident(self.put(bias_rows(values)), 1, int(np.asarray(values).size))

    def norm(self, gamma, beta, scalars) -> Resident:
        return Resident(self.put(norm_block(gamma, beta, scalars)), 1, int(np.asarray(gamma).size))


# ---------------------------------------------------------------------------------------------------------------
# Images
# ---------------------------------------------------------------------------------------------------------------

@dataclass(frozen=True)
class Image:
    address: int
    size: int
    entry: dict


class ImageSet:
    """Manifest lookup by kind and fields; each image (and causal constants block) staged once on first use."""

    def __init__(self, session: Session, directory: pathlib.Path = _images.DEFAULT_DIRECTORY) -> None:
        self.directory = _images.ensure_image_set(directory)
        self.manifest: dict[str, dict] = json.loads((self.directory / "manifest.json").read_text())
        self._session = session
        self._staged: dict[str, Image] = {}
        self._constants: dict[bytes, int] = {}

    def entries(self, kind: str) -> list[dict]:
        return [e for e in self.manifest.values() if e["kind"] == kind]

    def name_of(self, kind: str, **fields) -> str:
        for name, entry in self.manifest.items():
            if entry["kind"] == kind and all(entry.get(k) == v for k, v in fields.items()):
                return name
        stated = ", ".join(f"{k}={v}" for k, v in fields.items())
        raise ValueError(f"Unable to find a {kind} image with {stated} in {self.directory}.")

    def image_bytes(self, kind: str, **fields) -> bytes:
        return (self.directory / self.name_of(kind, **fields)).read_bytes()

    def get(self, kind: str, **fields) -> Image:
        name = self.name_of(kind, **fields)
        staged = self._staged.get(name)
        if staged is None:
            data = (self.directory / name).read_bytes()
            staged = Image(self._session.put(np.frombuffer(data, np.uint8)), len(data), self.manifest[name])
            self._staged[name] = staged
        return staged

    def causal_constants(self, entry: dict) -> int:
        data = (self.directory / entry["constants"]).read_bytes()
        address = self._constants.get(data)
        if address is None:
            address = self._session.put(np.frombuffer(data, np.uint8))
            self._constants[data] = address
        return address


Launch = tuple[Image, tuple[int, ...]]


def run(launches: list[Launch]) -> None:
    for image, args in launches:
        rt.minitpuLaunchKernel(image.address, image.size, args=list(args))


# ---------------------------------------------------------------------------------------------------------------
# Ops as launch lists
# ---------------------------------------------------------------------------------------------------------------

def gemm_launches(images: ImageSet, x: Packed, w: Resident, bias: Resident, out: Packed, *, activate: bool = False,
                  tile: int = 0) -> list[Launch]:
    """out = [GELU](x) W + bias, block by block; x's operand may start at a feature tile (a fused tensor's queries)."""
    image = images.get("gemm_bias", depth=w.depth, columns=w.columns, activate=activate)
    if out.features != w.columns or out.tokens != x.tokens:
        raise ValueError(f"Unable to write a [{x.tokens}, {w.columns}] product into [{out.tokens}, {out.features}].")
    return [(image, (x.rows(b, tile), w.address, out.drain(b), bias.address)) for b in range(x.blocks)]


def add_launches(images: ImageSet, left: Packed, right: Packed | Resident, out: Packed) -> list[Launch]:
    if isinstance(right, Resident):
        image = images.get("add_bias", features=left.features)
        return [(image, (left.rows(b), right.address, out.rows(b))) for b in range(left.blocks)]
    if (left.tokens, left.features) != (right.tokens, right.features):
        raise ValueError(f"Unable to add [{left.tokens}, {left.features}] and [{right.tokens}, {right.features}] "
                         f"tensors. Elementwise addition needs one shape.")
    image = images.get("add", features=left.features)
    return [(image, (left.rows(b), right.rows(b), out.rows(b))) for b in range(left.blocks)]


def norm_launches(images: ImageSet, x: Packed, constants: Resident, out: Packed,
                  blocks: range | None = None) -> list[Launch]:
    image = images.get("layernorm", features=x.features)
    return [(image, (x.rows(b), constants.address, out.rows(b))) for b in (blocks or range(x.blocks))]


def causal_launch(images: ImageSet, fused: Packed, heads: int) -> Launch:
    """Every head's causal attention over a fused QKV tensor in one launch, written over its queries."""
    image = images.get("attention", tokens=fused.tokens, heads=heads)
    return image, (images.causal_constants(image.entry), 0, fused.rows(0))


class PackedCache:
    """One layer's cached keys and values: a packed [capacity, 2 x width] tensor filled by the copy images."""

    def __init__(self, session: Session, images: ImageSet, capacity: int, width: int = WIDTH) -> None:
        self.tensor = session.packed(capacity, 2 * width)
        self.images = images
        self.width = width
        self.length = 0

    def _keys_tile(self) -> int:
        return self.width // LANES   # keys and values follow the queries' tiles in a fused block

    def fill_launches(self, fused: Packed, valid: int) -> list[Launch]:
        """Copies a prefill's whole blocks of keys and values after those held; `valid` of its tokens count."""
        if self.length % BLOCK or self.length + fused.tokens > self.tensor.tokens:
            raise ValueError(f"Unable to add {fused.tokens} tokens to a cache holding {self.length} of "
                             f"{self.tensor.tokens}. Prefills add whole blocks to a cache holding whole blocks.")
        rows = 2 * self.width // LANES * BLOCK
        image = self.images.get("copy", rows=rows, stride=2 * LANES)
        first = self.length // BLOCK
        launches = [(image, (fused.rows(b, self._keys_tile()), 0, self.tensor.rows(first + b)))
                    for b in range(fused.blocks)]
        self.length += valid
        return launches

    def push_launch(self, fused: Packed) -> Launch:
        """Copies row 0 of a decode block's keys and values into the next position."""
        if self.length >= self.tensor.tokens:
            raise ValueError(f"Unable to add a token to a cache holding all {self.tensor.tokens} it has room for.")
        image = self.images.get("copy", rows=2 * self.width // LANES, stride=BLOCK * LANES * 2)
        block, row = divmod(self.length, BLOCK)
        self.length += 1
        return image, (fused.rows(0, self._keys_tile()), 0, self.tensor.rows(block) + row * LANES * 2)


class DecodeConstants:
    """The decode images' constants blocks, one device block per key count, rewritten for each step's length."""

    def __init__(self, session: Session, images: ImageSet, heads: int) -> None:
        self.images, self.heads = images, heads
        self.session = session
        self._address: dict[int, int] = {}

    def launch(self, fused: Packed, cache: PackedCache) -> Launch:
        built = sorted(e["keys"] for e in self.images.entries("decode_attention") if e["heads"] == self.heads)
        keys = next((k for k in built if k >= cache.length), None)
        if cache.length < 1 or keys is None or keys > cache.tensor.tokens:
            raise ValueError(f"Unable to attend over {cache.length} cached tokens (room for {cache.tensor.tokens}) "
                             f"with decode images over {built} keys.")
        image = self.images.get("decode_attention", keys=keys, heads=self.heads)
        entry = image.entry
        words = mask_tiles(keys=keys, length=cache.length, entering=entry["entering"], stated=entry["stated"],
                           transposed=entry.get("transposed_masks", False))
        address = self._address.get(keys)
        if address is None:
            address = self._address[keys] = self.session.put(words)
        else:
            _write(address, words)
        return image, (address, cache.tensor.rows(0), fused.rows(0))


# ---------------------------------------------------------------------------------------------------------------
# The host product (the board's GEMM check path)
# ---------------------------------------------------------------------------------------------------------------

def block_product(activations, weights, *, activate: bool = False, bias=None) -> NDArray[np.float32]:
    """[tokens, depth] x [depth, columns] through the GEMM image on 32-token blocks (zero bias unless given)."""
    activations = np.asarray(activations, np.float32)
    weights = np.asarray(weights, np.float32)
    tokens, depth = activations.shape
    if depth != weights.shape[0]:
        raise ValueError(f"Unable to multiply [{tokens}, {depth}] by [{weights.shape[0]}, {weights.shape[1]}]. The "
                         f"inner dimensions must agree.")
    with Session() as session:
        images = ImageSet(session)
        x = session.rows_in(activations)
        w = session.matrix(weights)
        b = session.bias(np.zeros(weights.shape[1], np.float32) if bias is None else bias)
        out = session.packed(x.tokens, weights.shape[1])
        run(gemm_launches(images, x, w, b, out, activate=activate))
        return session.rows_out(out)[:tokens]


# ---------------------------------------------------------------------------------------------------------------
# The model
# ---------------------------------------------------------------------------------------------------------------

@dataclass
class _Workspace:
    """One padded token count's activations: hidden ping-pong pair, and each intermediate of a layer."""

    hidden: list[Packed]
    normed: Packed
    fused: Packed
    attended: Packed
    residual: Packed
    wide: Packed
    narrow: Packed


@dataclass
class _LayerWeights:
    ln1: Resident
    qkv: Resident
    qkv_bias: Resident
    proj: Resident
    proj_bias: Resident
    ln2: Resident
    fc: Resident
    fc_bias: Resident
    out: Resident
    out_bias: Resident


@dataclass
class PackedGPT2:
    """GPT-2 through the per-block images, every weight resident from construction.

    ``layers`` and ``shared`` use the reference's parameter names (``weights.py``); the query scale 1/sqrt(head) is
    folded into the QKV weights and bias at upload, as the reference does (``gpt2_inference.py:1153-1168``).
    """

    layers: list[dict]
    shared: dict
    heads: int = 12
    capacity: int = CONTEXT
    session: Session = field(default_factory=Session)

    def __post_init__(self) -> None:
        self.images = ImageSet(self.session)
        scalars = self.images.entries("layernorm")[0]["scalars"]
        width = self.shared["wte"].shape[1]
        scale = np.ones(3 * width, np.float32)
        scale[:width] = 1.0 / math.sqrt(width // self.heads)
        s = self.session
        self.weights = [_LayerWeights(
            ln1=s.norm(w["ln_1.g"], w["ln_1.b"], scalars),
            qkv=s.matrix(w["attn.qkv.w"] * scale), qkv_bias=s.bias(w["attn.qkv.b"] * scale),
            proj=s.matrix(w["attn.proj.w"]), proj_bias=s.bias(w["attn.proj.b"]),
            ln2=s.norm(w["ln_2.g"], w["ln_2.b"], scalars),
            fc=s.matrix(w["mlp.fc.w"]), fc_bias=s.bias(w["mlp.fc.b"]),
            out=s.matrix(w["mlp.proj.w"]), out_bias=s.bias(w["mlp.proj.b"])) for w in self.layers]
        self.final = s.norm(self.shared["ln_f.g"], self.shared["ln_f.b"], scalars)
        self.width = width
        self.caches: list[PackedCache] = []
        self.decode = DecodeConstants(s, self.images, self.heads)
        self._spaces: dict[int, _Workspace] = {}

    def close(self) -> None:
        self.session.close()

    def _space(self, tokens: int) -> _Workspace:
        space = self._spaces.get(tokens)
        if space is None:
            p, w = self.session.packed, self.width
            space = _Workspace(hidden=[p(tokens, w), p(tokens, w)], normed=p(tokens, w), fused=p(tokens, 3 * w),
                               attended=p(tokens, w), residual=p(tokens, w), wide=p(tokens, 4 * w),
                               narrow=p(tokens, w))
            self._spaces[tokens] = space
        return space

    def _layer(self, index: int, space: _Workspace, source: Packed,
               target: Packed) -> tuple[list[Launch], list[Launch]]:
        """One block's launches before its attention (LayerNorm, QKV) and after it (projection, residual, LayerNorm,
        MLP with the GELU on the second projection's input, residual), in the order of ``gpt2_inference.py:1133-1189``."""
        w, im = self.weights[index], self.images
        fused = space.fused
        return [*norm_launches(im, source, w.ln1, space.normed),
                *gemm_launches(im, space.normed, w.qkv, w.qkv_bias, fused)], [
            *gemm_launches(im, fused, w.proj, w.proj_bias, space.attended),
            *add_launches(im, source, space.attended, space.residual),
            *norm_launches(im, space.residual, w.ln2, space.normed),
            *gemm_launches(im, space.normed, w.fc, w.fc_bias, space.wide),
            *gemm_launches(im, space.wide, w.out, w.out_bias, space.narrow, activate=True),
            *add_launches(im, space.residual, space.narrow, target),
        ]

    def _forward(self, rows: NDArray[np.float32], valid: int, attend, observe: Observer | None) -> Packed:
        space = self._space(-(-rows.shape[0] // BLOCK) * BLOCK)
        source, target = space.hidden
        self.session.rows_in(rows, tensor=source)
        for index, cache in enumerate(self.caches):
            before, after = self._layer(index, space, source, target)
            run(before)
            run(attend(space.fused, cache))
            run(after)
            if observe is not None:
                observe(index, Session.rows_out(source)[:valid], Session.rows_out(target)[:valid])
            source, target = target, source
        return source

    def _embed(self, ids, start: int) -> NDArray[np.float32]:
        positions = start + np.arange(len(ids))
        return (self.shared["wte"][np.asarray(ids)] + self.shared["wpe"][positions]).astype(np.float32)

    def _last_row_logits(self, hidden: Packed, row: int) -> NDArray[np.float32]:
        """The final LayerNorm of the block holding `row` on the device, then the tied LM head on the host."""
        space = self._space(hidden.tokens)
        block = row // BLOCK
        run(norm_launches(self.images, hidden, self.final, space.normed, range(block, block + 1)))
        normed = Session.rows_out(space.normed, blocks=range(block, block + 1))[row % BLOCK]
        return normed @ self.shared["wte"].T

    def _prefill_rows(self, rows: NDArray[np.float32], valid: int, observe: Observer | None) -> Packed:
        """Hidden rows (whole blocks, `valid` of them real) through every layer, filling fresh caches."""
        if rows.shape[0] > self.capacity:
            raise ValueError(f"Unable to prefill {rows.shape[0]} rows into caches holding {self.capacity}.")
        if not self.caches:
            self.caches = [PackedCache(self.session, self.images, self.capacity, self.width) for _ in self.layers]
        for cache in self.caches:
            cache.length = 0

        def attend(fused: Packed, cache: PackedCache) -> list[Launch]:
            return [*cache.fill_launches(fused, valid), causal_launch(self.images, fused, self.heads)]

        return self._forward(rows, valid, attend, observe)

    def forward_rows(self, rows, *, observe: Observer | None = None) -> NDArray[np.float32]:
        """Given hidden rows [tokens, width] through every layer with causal attention (a prefill that starts from
        hidden states instead of token ids); returns the last layer's rows."""
        rows = np.asarray(rows, dtype=np.float32)
        tokens = rows.shape[0]
        padded = np.zeros((-(-tokens // BLOCK) * BLOCK, rows.shape[1]), np.float32)
        padded[:tokens] = rows
        return Session.rows_out(self._prefill_rows(padded, tokens, observe))[:tokens]

    def prefill(self, ids, *, observe: Observer | None = None) -> NDArray[np.float32]:
        """Fills fresh caches from a prompt; returns the next token's logits. The prompt pads with end-of-text
        tokens to whole blocks (causal attention keeps the padding out of the real rows)."""
        ids = np.asarray(ids, dtype=np.int64)
        tokens = len(ids)
        padded = -(-tokens // BLOCK) * BLOCK
        if tokens == 0:
            raise ValueError("Unable to prefill an empty prompt.")
        pad = min(END_OF_TEXT, self.shared["wte"].shape[0] - 1)   # any id: causal attention hides the padding
        rows = self._embed(np.concatenate([ids, np.full(padded - tokens, pad, np.int64)]), 0)
        return self._last_row_logits(self._prefill_rows(rows, tokens, observe), tokens - 1)

    def step(self, token: int, *, observe: Observer | None = None) -> NDArray[np.float32]:
        """One generated token through every layer (row 0 of a 32-row block); returns the next token's logits."""
        position = self.caches[0].length
        if position >= self.capacity:
            raise ValueError(f"Unable to decode past the caches' {self.capacity} positions.")
        rows = self._embed([token], position)

        def attend(fused: Packed, cache: PackedCache) -> list[Launch]:
            return [cache.push_launch(fused), self.decode.launch(fused, cache)]

        hidden = self._forward(rows, 1, attend, observe)
        return self._last_row_logits(hidden, 0)

    def generate(self, ids, new_tokens: int) -> list[int]:
        """Greedy continuation; stops early at end-of-text."""
        if len(ids) + new_tokens > self.capacity:
            raise ValueError(f"Unable to generate {new_tokens} tokens after {len(ids)}: the caches hold "
                             f"{self.capacity}.")
        out: list[int] = []
        logits = self.prefill(ids)
        while len(out) < new_tokens:
            out.append(int(np.argmax(logits)))
            if out[-1] == END_OF_TEXT or len(out) == new_tokens:
                break
            logits = self.step(out[-1])
        return out
