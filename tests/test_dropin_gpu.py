"""The reference's board checks (board_package/board_checks.py:557-576), ported onto the drop-in path: the layer
drivers in tempo_compiler_b200.gpt2 launch images through tempo_compiler_b200.runtime, i.e. through the C ABI, onto
the B200 kernels. Each check holds the device to the same host reference and bound the board check uses."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import bf16 as ob
from oracle import references as orf
from oracle.model import embed as host_embed
from oracle.model import final_norm, lm_head

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

PROMPT = (464, 3139, 286, 4881, 318)


@pytest.fixture(scope="module")
def g():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from tempo_compiler_b200 import gpt2
    return gpt2


def _layer_error(actual, expected, layer_input) -> float:
    """Error relative to the larger of the input's and output's norms (board_checks.py:521-530)."""
    scale = max(np.linalg.norm(layer_input), np.linalg.norm(expected))
    return float(np.linalg.norm(np.asarray(actual) - expected) / scale)


def _block_weights(model: int, seed: int) -> dict:
    rng = np.random.default_rng(seed)

    def normal(shape, scale):
        return ob.bf16_grid((rng.standard_normal(shape) * scale).astype(np.float32))

    ones = ob.bf16_grid(np.ones(model, dtype=np.float32))
    return {"ln_1.g": ones, "ln_1.b": normal((model,), 0.02), "attn.qkv.w": normal((model, 3 * model), 0.02),
            "attn.qkv.b": normal((3 * model,), 0.02), "attn.proj.w": normal((model, model), 0.02),
            "attn.proj.b": normal((model,), 0.02), "ln_2.g": ones.copy(), "ln_2.b": normal((model,), 0.02),
            "mlp.fc.w": normal((model, 4 * model), 0.02), "mlp.fc.b": normal((4 * model,), 0.02),
            "mlp.proj.w": normal((4 * model, model), 0.02), "mlp.proj.b": normal((model,), 0.02)}


def test_halt_launches_repeatedly(g) -> None:
    """check_halt (board_checks.py:76-109,172-183): stage the halt image at the aperture base and start it 3 times."""
    from tempo_compiler_b200 import runtime
    space = runtime.minitpuGetAddressSpace()
    image = g.halt_image()
    staging = runtime.minitpuHostAlloc(len(image))
    staging.view[: len(image) // 4] = np.frombuffer(image, dtype="<u4")
    runtime.minitpuMemcpy(dst=space.kernel_base, src=staging, nbytes=len(image), kind=runtime.MemcpyKind.HostToDevice)
    before = runtime.launches()
    for _ in range(3):
        runtime.minitpuLaunchKernel(kbin_addr=space.kernel_base, kbin_size=len(image))
    assert runtime.launches() == before + 3
    runtime.minitpuHostReset()


def test_copy_round_trip_is_exact(g) -> None:
    """check_copy_argument (board_checks.py:112-150,186-201): random words there and back, corruption-filled first."""
    from tempo_compiler_b200 import runtime
    words = np.random.default_rng(0).integers(0, 1 << 16, size=32 * 768, dtype=np.uint16)
    source = runtime.minitpuHostAlloc(words.nbytes)
    destination = runtime.minitpuHostAlloc(words.nbytes)
    source.view.view("<u2")[: words.size] = words
    address = runtime.minitpuMalloc(words.nbytes)
    try:
        runtime.minitpuMemcpy(dst=address, src=source, nbytes=words.nbytes, kind=runtime.MemcpyKind.HostToDevice)
        destination.view.view("<u2")[: words.size] = 0xBEEF
        runtime.minitpuMemcpy(dst=destination, src=address, nbytes=words.nbytes,
                              kind=runtime.MemcpyKind.DeviceToHost)
        np.testing.assert_array_equal(destination.view.view("<u2")[: words.size], words)
    finally:
        runtime.minitpuFree(address)
        runtime.minitpuHostReset()


def test_full_gemm_structured_exact_and_varying_within_one_percent(g) -> None:
    """check_full_gemm (board_checks.py:204-253) at [32,768] @ [768,3072]."""
    left, right = ob.build_operands(32, 768, 3072, kind="structured", seed=0)
    np.testing.assert_allclose(g.full_gemm(left, right), left @ right, rtol=0, atol=0)
    left, right = ob.build_operands(32, 768, 3072, kind="varying", seed=0)
    assert orf.relative_error(g.full_gemm(left, right), orf.gemm_f64(left, right)) < 0.01


def test_full_gemm_over_several_blocks_and_resident_weights(g) -> None:
    left, right = ob.build_operands(96, 768, 768, kind="varying", seed=4)
    d_w = g.upload_weights(right)
    try:
        assert orf.relative_error(g.full_gemm(left, d_w), orf.gemm_f64(left, right)) < 0.01
    finally:
        d_w.free()


def test_elementwise_add_and_bias_add_are_exact(g) -> None:
    """check_elementwise_add (board_checks.py:256-289)."""
    rng = np.random.default_rng(53)
    left = ob.bf16_grid(rng.standard_normal((32, 768)).astype(np.float32))
    right = ob.bf16_grid(rng.standard_normal((32, 768)).astype(np.float32))
    bias = ob.bf16_grid(rng.standard_normal(768).astype(np.float32))
    d_left, d_right, d_bias = g.upload_activations(left), g.upload_activations(right), g.upload_bias(bias)
    try:
        d_sum = g.add_resident(d_left, d_right)
        d_biased = g.add_bias_resident(d_left, d_bias)
        summed, biased = g.download_activations(d_sum), g.download_activations(d_biased)
        d_sum.free()
        d_biased.free()
    finally:
        d_left.free()
        d_right.free()
        d_bias.free()
    np.testing.assert_array_equal(summed, ob.bf16_grid(left + right))
    np.testing.assert_array_equal(biased, ob.bf16_grid(left + bias))


def test_decode_attention_all_heads_within_five_percent(g) -> None:
    """check_decode_attention (board_checks.py:292-332): 48 cached tokens plus the step's."""
    rng = np.random.default_rng(19)
    context, model = 48, 768
    tokens = 64
    prefill = ob.bf16_grid(rng.standard_normal((tokens, 3 * model)).astype(np.float32))
    step = ob.bf16_grid(rng.standard_normal((32, 3 * model)).astype(np.float32))
    d_prefill, d_step = g.upload_activations(prefill), g.upload_activations(step)
    cache = g.KVCache(capacity=tokens + 32, model=model)
    try:
        cache.extend(d_prefill, tokens=context)
        cache.append(d_step)
        actual = g.download_activations(g.decode_attention(d_step, cache, heads=12))[0]
    finally:
        cache.free()
        d_prefill.free()
        d_step.free()
    keys = np.concatenate([prefill[:context, model:2 * model], step[:1, model:2 * model]])
    values = np.concatenate([prefill[:context, 2 * model:], step[:1, 2 * model:]])
    expected = np.concatenate([orf.attention_f64(step[:1, h * 64:(h + 1) * 64], keys[:, h * 64:(h + 1) * 64],
                                                 values[:, h * 64:(h + 1) * 64]) for h in range(12)], axis=1)[0]
    assert orf.relative_error(actual[:model], expected) < 0.05


def test_layernorm_within_two_percent(g) -> None:
    """check_layernorm (board_checks.py:335-359)."""
    rng = np.random.default_rng(0)
    values = ob.bf16_grid((rng.standard_normal((32, 768)) * 2.0).astype(np.float32))
    gamma = ob.bf16_grid((1.0 + 0.1 * rng.standard_normal(768)).astype(np.float32))
    beta = ob.bf16_grid((0.1 * rng.standard_normal(768)).astype(np.float32))
    d_rows, d_constants = g.upload_activations(values), g.upload_layernorm_constants(gamma, beta)
    try:
        d_normed = g.layernorm_resident(d_rows, d_constants)
        actual = g.download_activations(d_normed)
        d_normed.free()
    finally:
        d_rows.free()
        from tempo_compiler_b200.runtime import minitpuFree
        minitpuFree(d_constants)
    assert orf.relative_error(actual, orf.layernorm_device(values, gamma, beta)) < 0.02


def test_kv_cache_holds_every_token_exactly(g) -> None:
    """check_kv_cache (board_checks.py:362-387)."""
    rng = np.random.default_rng(31)
    prefill = ob.bf16_grid(rng.standard_normal((64, 3 * 768)).astype(np.float32))
    step = ob.bf16_grid(rng.standard_normal((32, 3 * 768)).astype(np.float32))
    d_prefill, d_step = g.upload_activations(prefill), g.upload_activations(step)
    cache = g.KVCache(capacity=96, model=768)
    try:
        cache.extend(d_prefill)
        cache.append(d_step)
        held = g.download_activations(cache.tensor)[:cache.length]
    finally:
        cache.free()
        d_prefill.free()
        d_step.free()
    np.testing.assert_array_equal(held, np.concatenate([prefill[:, 768:], step[:1, 768:]]))


def test_transformer_block_within_five_percent(g) -> None:
    """check_transformer_block (board_checks.py:485-518): [64, 768], the board check's weights."""
    rng = np.random.default_rng(1)
    hidden = ob.bf16_grid((rng.standard_normal((64, 768)) * 0.5).astype(np.float32))
    weights = _block_weights(768, 2)
    actual = g.transformer_block(hidden=hidden, weights=weights)
    assert orf.relative_error(actual, orf.block_device(hidden, weights)) < 0.05
    assert orf.relative_error(actual, orf.block_exact(hidden, weights)) < 0.02


@pytest.fixture(scope="module")
def model():
    from tempo_compiler_b200.weights import random_gpt2
    return random_gpt2(7)


def test_gpt2_prefill_layers_within_five_percent(g, model) -> None:
    """check_gpt2_prefill (board_checks.py:390-423): every layer held to the reference on its own device input."""
    layers, shared = model
    tokens = len(PROMPT)
    errors: list[float] = []

    def compare(index, layer_input, layer_output):
        expected = orf.block_device(layer_input, layers[index])[:tokens]
        errors.append(_layer_error(layer_output[:tokens], expected, layer_input[:tokens]))

    _, caches = g.prefill(np.asarray(PROMPT), layers, shared, observe=compare)
    lengths = {cache.length for cache in caches}
    for cache in caches:
        cache.free()
    assert lengths == {tokens}
    assert max(errors) < 0.05, errors


def test_gpt2_decode_layers_and_greedy_tokens(g, model) -> None:
    """check_gpt2_decode (board_checks.py:426-482): one decode step, each layer within 5%, and the two greedy tokens
    equal the reference chain's (full recompute through the device-rounding references)."""
    layers, shared = model
    tokens = len(PROMPT)
    prompt_inputs: dict[int, np.ndarray] = {}
    errors: list[float] = []

    def remember(index, layer_input, _):
        prompt_inputs[index] = layer_input[:tokens]

    def compare(index, layer_input, layer_output):
        rows = np.concatenate([prompt_inputs[index], layer_input[None, :]])
        expected = orf.block_device(rows, layers[index])[-1]
        errors.append(_layer_error(layer_output, expected, layer_input))

    hidden, caches = g.prefill(np.asarray(PROMPT), layers, shared, observe=remember)
    try:
        first = int(np.argmax(g.next_token_logits(hidden[-1], shared)))
        second = int(np.argmax(g.next_token_logits(g.decode_step(first, layers, shared, caches, observe=compare),
                                                   shared)))
        lengths = {cache.length for cache in caches}
    finally:
        for cache in caches:
            cache.free()
    reference, margins = [], []
    for sequence in (PROMPT, (*PROMPT, first)):
        rows = host_embed(np.asarray(sequence), shared)
        for weights in layers:
            rows = orf.block_device(rows, weights)
        logits = lm_head(final_norm(rows[-1:], shared, "device")[0], shared, "device")
        top = np.sort(logits)[-2:]
        reference.append(int(np.argmax(logits)))
        margins.append(float(top[1] - top[0]))
    assert lengths == {tokens + 1}
    assert max(errors) < 0.05, errors
    assert [first, second] == reference, (reference, margins)


def test_runtime_error_classes(g) -> None:
    """The reference's exceptions for the same misuse (runtime/device.py:158-196, launch.py:67-141)."""
    from tempo_compiler_b200 import runtime
    with pytest.raises(KeyError):
        runtime.minitpuFree(0x8000_0040 + 12345 * 32)
    with pytest.raises(MemoryError):
        runtime.minitpuMalloc(1 << 40)
    space = runtime.minitpuGetAddressSpace()
    junk = runtime.minitpuHostAlloc(64)
    junk.view[:16] = np.arange(16, dtype=np.uint32)
    address = runtime.minitpuMalloc(64)
    try:
        runtime.minitpuMemcpy(address, junk, 64, runtime.MemcpyKind.HostToDevice)
        with pytest.raises(RuntimeError):
            runtime.minitpuLaunchKernel(address, 64)
        image = g.halt_image()
        with pytest.raises(ValueError):
            runtime.minitpuLaunchKernel(address + 16, 64)
        with pytest.raises(ValueError):
            runtime.minitpuLaunchKernel(space.kernel_base, len(image), args=[1, 2, 3, 4, 5])
        with pytest.raises(ValueError):
            runtime.minitpuLaunchKernel(space.kernel_base, len(image), args=[1 << 32])
        # an operand outside the arena is refused before the kernel runs
        add_image, _ = g._compiled_image(kind="add", features=768)
        staged = g._stage_image(add_image)
        with pytest.raises(ValueError, match="arena"):
            runtime.minitpuLaunchKernel(staged, len(add_image), args=[0x10, 0x10, 0x10])
    finally:
        runtime.minitpuFree(address)
        runtime.minitpuHostReset()
