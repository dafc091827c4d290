"""The image set: one manifest entry per launchable tile op, with the reference's kinds and fields, and its image.

An "image" here is a 64-byte descriptor (``tempo_image`` in include/tempo_b200.h): magic, version, kind, the kind's
fields and a checksum. Staged in device memory and launched through ``runtime.minitpuLaunchKernel``, it selects the
B200 kernel the same way the reference's VLIW image selects its program; the layer drivers key images by their bytes
(board_package/gpt2_inference.py:1240-1259) and read the manifest by kind and fields
(gpt2_inference.py:1072-1108), so both behave unchanged.

The entries follow the reference's image builder (tools/board/build_images.py:24-58) and manifest writer
(mlir/lib/tempo/manifest.cpp:103-167): the four GPT-2 projections as ``gemm_bias`` with ``depth``, ``columns``,
``activate`` and ``drain_words``; ``add``/``add_bias`` with ``features``; ``layernorm`` with ``features``, ``rows`` and
``scalars``; ``attention`` with ``tokens``, ``heads`` and its ``constants`` file; ``decode_attention`` with ``keys``,
``heads``, ``entering``, ``stated`` and ``transposed_masks``; ``copy`` with ``rows`` and ``stride``; and ``halt``. The
B200 set adds causal attention for every multiple of 32 tokens up to 1024, so prefill pads to the next block rather
than being capped at 64 tokens.

    python -m tempo_compiler_b200.images [--output DIR]
"""

from __future__ import annotations

import argparse
import json
import pathlib
import struct

import numpy as np

from tempo_compiler_b200.lib import IMAGE_BYTES, IMAGE_MAGIC, KIND

DEFAULT_DIRECTORY = pathlib.Path(__file__).resolve().parent / "images" / "generated"

GEMMS = ((768, 2304, False), (768, 768, False), (768, 3072, False), (3072, 768, True))
ADDS = ((768, False), (768, True))
LAYERNORMS = (768,)
ATTENTION_TOKENS = tuple(range(32, 1025, 32))
DECODE_KEYS = (64, 256, 1024)
HEADS, HEAD = 12, 64
COPIES = ((3072, 32), (96, 1024))
LN_EPSILON = 9.999999747378752e-06  # float32(1e-5), as the manifest states it (manifest.json:44)
ENTERING_MAXIMUM = -1e30


def descriptor(kind: str, fields: tuple[int, ...] = (), scalars: tuple[float, float] = (0.0, 0.0)) -> bytes:
    """The 64-byte image descriptor of one entry."""
    words = [IMAGE_MAGIC, 1, KIND[kind], 0, *fields, *([0] * (8 - len(fields)))]
    head = struct.pack("<12I2f", *words, *scalars)
    checksum = sum(struct.unpack("<14I", head)) & 0xFFFFFFFF
    image = head + struct.pack("<2I", checksum, 0)
    assert len(image) == IMAGE_BYTES
    return image


def _bf16_words(values: np.ndarray) -> np.ndarray:
    bits = np.ascontiguousarray(values, dtype="<f4").view("<u4")
    return ((bits + np.uint32(0x7FFF) + ((bits >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype("<u2")


def causal_constants() -> bytes:
    """The block a causal attention image reads (mlir/lib/tempo/manifest.cpp:197-222): a tile of the entering maximum, a
    tile of zeros, then the diagonal mask tile laid out keys by queries (-1e30 where the key is past the query)."""
    key = np.arange(16)[:, None]
    query = np.arange(16)[None, :]
    tiles = [np.full((16, 16), ENTERING_MAXIMUM, np.float32), np.zeros((16, 16), np.float32),
             np.where(key > query, np.float32(ENTERING_MAXIMUM), np.float32(0.0))]
    return _bf16_words(np.concatenate(tiles)).tobytes()


def build_image_set() -> list[tuple[str, dict, bytes]]:
    """Every entry of the image set as (file name, manifest entry, image bytes), in manifest order."""
    entries: list[tuple[str, dict, bytes]] = []
    for depth, columns, activate in GEMMS:
        drain_words = 256 + columns * 32
        name = f"gemm_{depth}x{columns}{'_gelu' if activate else ''}_bias.bin"
        entry = {"kind": "gemm_bias", "depth": depth, "columns": columns, "activate": activate,
                 "drain_words": drain_words}
        entries.append((name, entry, descriptor("gemm_bias", (depth, columns, int(activate), drain_words))))
    for features, broadcast in ADDS:
        kind = "add_bias" if broadcast else "add"
        entries.append((f"{kind}_{features}.bin", {"kind": kind, "features": features}, descriptor(kind, (features,))))
    for features in LAYERNORMS:
        entry = {"kind": "layernorm", "features": features, "rows": ["gamma_pointer", "beta_pointer"],
                 "scalars": [1.0 / features, LN_EPSILON]}
        entries.append((f"layernorm_{features}.bin", entry,
                        descriptor("layernorm", (features,), (1.0 / features, LN_EPSILON))))
    for tokens in ATTENTION_TOKENS:
        entry = {"kind": "attention", "tokens": tokens, "heads": HEADS, "constants": f"attention_{tokens}_constants.bin"}
        entries.append((f"attention_{tokens}.bin", entry, descriptor("attention", (tokens, HEADS, HEAD))))
    for keys in DECODE_KEYS:
        entry = {"kind": "decode_attention", "keys": keys, "heads": HEADS, "entering": ENTERING_MAXIMUM, "stated": [],
                 "transposed_masks": True}
        entries.append((f"decode_attention_{keys}.bin", entry, descriptor("decode_attention", (keys, HEADS, HEAD, 0))))
    for rows, stride in COPIES:
        entries.append((f"copy_{rows}x{stride}.bin", {"kind": "copy", "rows": rows, "stride": stride},
                        descriptor("copy", (rows, stride))))
    entries.append(("halt.bin", {"kind": "halt"}, descriptor("halt")))
    return entries


def write_image_set(directory: pathlib.Path = DEFAULT_DIRECTORY) -> pathlib.Path:
    """Writes every image, the causal constants blocks and manifest.json into `directory`; returns it."""
    directory = pathlib.Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    manifest = {}
    constants = causal_constants()
    for name, entry, image in build_image_set():
        (directory / name).write_bytes(image)
        manifest[name] = entry
        if entry["kind"] == "attention":
            (directory / entry["constants"]).write_bytes(constants)
    (directory / "manifest.json").write_text(json.dumps(manifest, indent=2) + "\n")
    return directory


def ensure_image_set(directory: pathlib.Path = DEFAULT_DIRECTORY) -> pathlib.Path:
    """Returns the image directory, writing it first when its manifest is missing."""
    if not (pathlib.Path(directory) / "manifest.json").exists():
        write_image_set(directory)
    return pathlib.Path(directory)


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--output", default=str(DEFAULT_DIRECTORY))
    print(write_image_set(pathlib.Path(parser.parse_args().output)))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
