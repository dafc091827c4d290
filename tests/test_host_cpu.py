"""Host-side checks that need no GPU: the C ABI library loads and exports every declared symbol, the image set keeps
the reference's manifest kinds and fields, the drop-in packers agree with the oracle, and malformed runtime calls are
refused before any device work, with the reference's exception classes."""

from __future__ import annotations

import json
import os
import pathlib
import re
import struct

import numpy as np
import pytest

from oracle import bf16 as ob

ROOT = pathlib.Path(__file__).resolve().parents[1]


def test_library_exports_every_declared_symbol() -> None:
    from tempo_compiler_b200 import lib
    declared = set(re.findall(r"tempo_status\s+(tempo_\w+)\s*\(", (ROOT / "include" / "tempo_b200.h").read_text()))
    assert declared == set(lib.EXPORTED)
    library = lib.load()
    for name in declared:
        assert getattr(library, name) is not None


def test_binding_argument_types_follow_the_header() -> None:
    """Every declaration's parameters, in order, against the ctypes signature the binding passes: a pointer for a
    pointer and the same width and signedness for a scalar, so no argument is truncated or misread across the C ABI."""
    import ctypes

    from tempo_compiler_b200 import lib
    header = (ROOT / "include" / "tempo_b200.h").read_text()
    header = re.sub(r"/\*.*?\*/", "", header, flags=re.S)
    scalars = {"uint32_t": ctypes.c_uint32, "uint64_t": ctypes.c_uint64, "int32_t": ctypes.c_int32,
               "int64_t": ctypes.c_int64, "int": ctypes.c_int, "float": ctypes.c_float, "double": ctypes.c_double}
    declarations = re.findall(r"tempo_status\s+(tempo_\w+)\s*\(([^)]*)\)\s*;", header)
    assert {name for name, _ in declarations} == set(lib.EXPORTED)
    for name, params in declarations:
        params = " ".join(params.split())
        declared = [] if params in ("", "void") else [p.strip() for p in params.split(",")]
        bound = lib._SIGNATURES[name]
        assert len(declared) == len(bound), (name, declared, bound)
        for param, ctype in zip(declared, bound):
            if "*" in param:
                assert ctype in (ctypes.c_void_p, ctypes.c_char_p) or issubclass(ctype, ctypes._Pointer), (name, param)
            else:
                base = param.replace("const ", "").split()[0]
                assert scalars[base] is ctype, (name, param, ctype)


def test_status_codes_map_to_the_reference_exceptions() -> None:
    from tempo_compiler_b200 import lib
    for status, exc in ((lib.ERR_VALUE, ValueError), (lib.ERR_MEMORY, MemoryError), (lib.ERR_KEY, KeyError),
                        (lib.ERR_RUNTIME, RuntimeError), (lib.ERR_TIMEOUT, TimeoutError)):
        with pytest.raises(exc):
            lib.check(status)
    lib.check(lib.OK)


def test_launch_validation_needs_no_device() -> None:
    """Malformed launches are refused before the device is consulted (runtime/launch.py:67-120)."""
    from tempo_compiler_b200 import lib
    import ctypes
    args = (ctypes.c_int64 * 4)(0, 0, 0, 0)
    library = lib.load()
    assert library.tempo_launch(0x80000000, 0, args, 0, 1.0) == lib.ERR_VALUE
    assert library.tempo_launch(0x80000000, 24, args, 0, 1.0) == lib.ERR_VALUE
    assert library.tempo_launch(0x80000000, 65552, args, 0, 1.0) == lib.ERR_VALUE
    assert library.tempo_launch(0x80000010, 64, args, 0, 1.0) == lib.ERR_VALUE
    assert library.tempo_launch(0xFFFFFFF0, 64, args, 0, 1.0) == lib.ERR_VALUE
    assert library.tempo_launch(0x80000000, 64, args, 5, 1.0) == lib.ERR_VALUE
    bad = (ctypes.c_int64 * 1)(1 << 32)
    assert library.tempo_launch(0x80000000, 64, bad, 1, 1.0) == lib.ERR_VALUE
    negative = (ctypes.c_int64 * 1)(-1)
    assert library.tempo_launch(0x80000000, 64, negative, 1, 1.0) == lib.ERR_VALUE


def test_runtime_refuses_malformed_calls_before_the_device() -> None:
    from tempo_compiler_b200 import runtime
    with pytest.raises(ValueError, match="kind"):
        runtime.minitpuMemcpy(0, 0, 32, "Sideways")
    with pytest.raises(ValueError, match="positive"):
        runtime.minitpuMemcpy(0, 0, 0, runtime.MemcpyKind.HostToDevice)
    with pytest.raises(ValueError, match="positive"):
        runtime.minitpuMalloc(0)
    with pytest.raises(ValueError, match="non-negative"):
        runtime.minitpuLaunchKernel(-32, 64)
    with pytest.raises(ValueError, match="stream"):
        runtime.minitpuMemcpyAsync(0, 0, 32, runtime.MemcpyKind.HostToDevice, stream=1)


def test_image_set_keeps_the_reference_manifest_fields(tmp_path) -> None:
    from tempo_compiler_b200 import images
    directory = images.write_image_set(tmp_path)
    manifest = json.loads((directory / "manifest.json").read_text())
    # The reference's entries (board_package/images/manifest.json) are all present with identical fields.
    reference_entries = {
        "gemm_768x2304_bias.bin": {"kind": "gemm_bias", "depth": 768, "columns": 2304, "activate": False,
                                   "drain_words": 73984},
        "gemm_768x768_bias.bin": {"kind": "gemm_bias", "depth": 768, "columns": 768, "activate": False,
                                  "drain_words": 24832},
        "gemm_768x3072_bias.bin": {"kind": "gemm_bias", "depth": 768, "columns": 3072, "activate": False,
                                   "drain_words": 98560},
        "gemm_3072x768_gelu_bias.bin": {"kind": "gemm_bias", "depth": 3072, "columns": 768, "activate": True,
                                        "drain_words": 24832},
        "add_768.bin": {"kind": "add", "features": 768},
        "add_bias_768.bin": {"kind": "add_bias", "features": 768},
        "layernorm_768.bin": {"kind": "layernorm", "features": 768, "rows": ["gamma_pointer", "beta_pointer"],
                              "scalars": [0.0013020833333333333, 9.999999747378752e-06]},
        "attention_64.bin": {"kind": "attention", "tokens": 64, "heads": 12, "constants": "attention_64_constants.bin"},
        "decode_attention_64.bin": {"kind": "decode_attention", "keys": 64, "heads": 12, "entering": -1e30,
                                    "stated": [], "transposed_masks": True},
        "decode_attention_256.bin": {"kind": "decode_attention", "keys": 256, "heads": 12, "entering": -1e30,
                                     "stated": [], "transposed_masks": True},
        "decode_attention_1024.bin": {"kind": "decode_attention", "keys": 1024, "heads": 12, "entering": -1e30,
                                      "stated": [], "transposed_masks": True},
        "copy_3072x32.bin": {"kind": "copy", "rows": 3072, "stride": 32},
        "copy_96x1024.bin": {"kind": "copy", "rows": 96, "stride": 1024},
        "halt.bin": {"kind": "halt"},
    }
    for name, entry in reference_entries.items():
        assert manifest[name] == entry, name
    for name, entry in manifest.items():
        image = (directory / name).read_bytes()
        assert len(image) == 64 and len(image) % 16 == 0
        words = struct.unpack("<16I", image)
        assert words[0] == 0x49324254 and words[1] == 1
        assert words[14] == sum(words[:14]) & 0xFFFFFFFF
        if entry["kind"] == "attention":
            constants = np.frombuffer((directory / entry["constants"]).read_bytes(), dtype="<u2")
            np.testing.assert_array_equal(constants, ob.causal_constants_words())


def test_dropin_layouts_agree_with_the_oracle() -> None:
    """The drop-in driver's host layouts equal the oracle's restatement of the reference's packers."""
    from tempo_compiler_b200 import dropin
    rng = np.random.default_rng(9)
    act = rng.standard_normal((32, 40)).astype(np.float32)
    wts = rng.standard_normal((40, 24)).astype(np.float32)
    bias = rng.standard_normal(32).astype(np.float32)
    np.testing.assert_array_equal(dropin.tile_major(act), ob.pack_activations(act))
    np.testing.assert_array_equal(dropin.tile_major(wts), ob.pack_weights(wts))
    np.testing.assert_array_equal(dropin.bias_rows(bias), ob.pack_bias(bias))
    np.testing.assert_array_equal(dropin.to_words(act), ob.bf16_bits(act))
    for keys, length, stated, transposed in ((64, 49, (), True), (256, 200, (1.5,), True), (64, 1, (), False)):
        masks = ob.decode_mask_tiles(keys=keys, length=length)
        if transposed:
            masks = np.ascontiguousarray(masks.swapaxes(-1, -2))
        expected = ob.pack_attention_constants(initial_maximum=-1e30, constants=stated, masks=masks).reshape(-1)
        got = dropin.mask_tiles(keys=keys, length=length, entering=-1e30, stated=stated, transposed=transposed)
        np.testing.assert_array_equal(got, expected)
    words = dropin.tile_major(act)
    np.testing.assert_array_equal(dropin.from_tile_major(words, 32, 48)[:, :40], ob.bf16_grid(act))


def test_reference_drivers_import_against_the_runtime_shim() -> None:
    """The maintainer's binding: the reference's own drivers import with this runtime installed as ``runtime``.

    Only the import surface is checked here (no launch); it needs the reference's checkout, named by the environment
    variable TEMPO_REFERENCE_DIR, and is skipped without it."""
    import importlib
    import sys
    root = os.environ.get("TEMPO_REFERENCE_DIR")
    if not root or not (pathlib.Path(root) / "board_package").is_dir():
        pytest.skip("TEMPO_REFERENCE_DIR does not name the reference project's checkout")
    reference = pathlib.Path(root) / "board_package"
    from tempo_compiler_b200 import runtime
    saved = {name: sys.modules.get(name) for name in ("runtime", "gpt2_inference", "bf16", "tokenizer")}
    sys.modules["runtime"] = runtime
    sys.path.insert(0, str(reference))
    try:
        module = importlib.import_module("gpt2_inference")
        assert module.minitpuLaunchKernel is runtime.minitpuLaunchKernel
    finally:
        sys.path.remove(str(reference))
        for name, value in saved.items():
            if value is None:
                sys.modules.pop(name, None)
            else:
                sys.modules[name] = value


def test_weights_round_trip_through_the_reference_export_format(tmp_path) -> None:
    """Weights saved in the reference's npz export format (BF16 words, ``h.<layer>.`` prefixes) load back exactly."""
    from tempo_compiler_b200.weights import GPT2Shape, load_gpt2_npz, random_gpt2, save_gpt2_npz
    layers, shared = random_gpt2(4, GPT2Shape(layers=2, vocab=300, positions=64))
    path = tmp_path / "gpt2_weights.npz"
    save_gpt2_npz(path, layers, shared)
    loaded_layers, loaded_shared = load_gpt2_npz(path)
    assert len(loaded_layers) == 2
    for original, loaded in zip(layers, loaded_layers):
        assert set(original) == set(loaded)
        for name in original:
            np.testing.assert_array_equal(original[name], loaded[name])
    for name in shared:
        np.testing.assert_array_equal(shared[name], loaded_shared[name])


def test_gelu_constants_are_the_fit_and_meet_their_bound() -> None:
    """The coefficients compiled into gelu_erf (common.cuh) are those fit_gelu.py derives, and their float32
    evaluation stays within 1e-5 relative error of float64 erfc over every BF16 input with |x| <= 14."""
    import importlib.util
    csrc = pathlib.Path(__file__).resolve().parents[1] / "tempo_compiler_b200" / "csrc"
    spec = importlib.util.spec_from_file_location("fit_gelu", csrc / "fit_gelu.py")
    fit_gelu = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(fit_gelu)
    coeffs = fit_gelu.fit()
    body = (csrc / "common.cuh").read_text().split("float gelu_erf(float x)")[1].split("\n}\n")[0]
    compiled = [float(v) for v in re.findall(r"fmaf\(p, t, (-?[0-9.]+)f\)", body)]
    leading = float(re.search(r"float p = (-?[0-9.]+)f;", body).group(1))
    assert np.array_equal(np.float32([leading] + compiled), np.float32(coeffs[::-1]))
    x = fit_gelu.bf16_inputs()
    ref = fit_gelu.exact(x)
    keep = np.abs(ref / x) >= 2.0 ** -126
    rel = np.abs(fit_gelu.evaluate_float32(x, coeffs)[keep] - ref[keep]) / np.abs(ref[keep])
    assert rel.max() < 1e-5, rel.max()
