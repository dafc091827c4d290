"""The reference's board checks (board_package/board_checks.py:557-576) on the drop-in path: images launched through
tempo_compiler_b200.runtime, i.e. through the C ABI, onto the B200 kernels, by the block driver in
tempo_compiler_b200.dropin. Each check holds the device to the host reference and bound its board check uses."""

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
def d():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from tempo_compiler_b200 import dropin
    return dropin


@pytest.fixture()
def session(d):
    with d.Session() as s:
        yield s, d.ImageSet(s)


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


def test_halt_launches_repeatedly(session) -> None:
    """check_halt (board_checks.py:76-109,172-183): stage the halt image at the aperture base and start it 3 times."""
    from tempo_compiler_b200 import runtime
    _, images = session
    space = runtime.minitpuGetAddressSpace()
    image = images.image_bytes("halt")
    staging = runtime.minitpuHostAlloc(len(image))
    staging.view[: len(image) // 4] = np.frombuffer(image, dtype="<u4")
    runtime.minitpuMemcpy(dst=space.kernel_base, src=staging, nbytes=len(image), kind=runtime.MemcpyKind.HostToDevice)
    before = runtime.launches()
    for _ in range(3):
        runtime.minitpuLaunchKernel(kbin_addr=space.kernel_base, kbin_size=len(image))
    assert runtime.launches() == before + 3
    runtime.minitpuHostReset()


def test_copy_round_trip_is_exact(d) -> None:
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


def test_block_product_structured_exact_and_varying_within_one_percent(d) -> None:
    """check_full_gemm (board_checks.py:204-253) at [32,768] @ [768,3072]."""
    left, right = ob.build_operands(32, 768, 3072, kind="structured", seed=0)
    np.testing.assert_allclose(d.block_product(left, right), left @ right, rtol=0, atol=0)
    left, right = ob.build_operands(32, 768, 3072, kind="varying", seed=0)
    assert orf.relative_error(d.block_product(left, right), orf.gemm_f64(left, right)) < 0.01


def test_block_product_over_several_blocks_with_bias_and_gelu(d) -> None:
    """Three blocks through the activating image (GELU of the input, bias added), against float64."""
    left, right = ob.build_operands(96, 3072, 768, kind="varying", seed=4)
    bias = ob.bf16_grid(np.random.default_rng(5).standard_normal(768).astype(np.float32) * 0.1)
    got = d.block_product(left, right, activate=True, bias=bias)
    assert orf.relative_error(got, orf.gemm_f64(left, right, bias=bias, activate=True)) < 0.01


def test_elementwise_add_and_bias_add_are_exact(d, session) -> None:
    """check_elementwise_add (board_checks.py:256-289)."""
    s, images = session
    rng = np.random.default_rng(53)
    left = ob.bf16_grid(rng.standard_normal((32, 768)).astype(np.float32))
    right = ob.bf16_grid(rng.standard_normal((32, 768)).astype(np.float32))
    bias = ob.bf16_grid(rng.standard_normal(768).astype(np.float32))
    d_left, d_right, d_bias = s.rows_in(left), s.rows_in(right), s.bias(bias)
    d_sum, d_biased = s.packed(32, 768), s.packed(32, 768)
    d.run(d.add_launches(images, d_left, d_right, d_sum) + d.add_launches(images, d_left, d_bias, d_biased))
    np.testing.assert_array_equal(s.rows_out(d_sum), ob.bf16_grid(left + right))
    np.testing.assert_array_equal(s.rows_out(d_biased), ob.bf16_grid(left + bias))


def test_decode_attention_all_heads_within_five_percent(d, session) -> None:
    """check_decode_attention (board_checks.py:292-332): 48 cached tokens plus the step's."""
    s, images = session
    rng = np.random.default_rng(19)
    context, model = 48, 768
    prefill = ob.bf16_grid(rng.standard_normal((64, 3 * model)).astype(np.float32))
    step = ob.bf16_grid(rng.standard_normal((32, 3 * model)).astype(np.float32))
    d_prefill, d_step = s.rows_in(prefill), s.rows_in(step)
    cache = d.PackedCache(s, images, capacity=96)
    constants = d.DecodeConstants(s, images, heads=12)
    d.run(cache.fill_launches(d_prefill, context))
    d.run([cache.push_launch(d_step)])
    d.run([constants.launch(d_step, cache)])
    actual = s.rows_out(d_step)[0]
    keys = np.concatenate([prefill[:context, model:2 * model], step[:1, model:2 * model]])
    values = np.concatenate([prefill[:context, 2 * model:], step[:1, 2 * model:]])
    expected = np.concatenate([orf.attention_f64(step[:1, h * 64:(h + 1) * 64], keys[:, h * 64:(h + 1) * 64],
                                                 values[:, h * 64:(h + 1) * 64]) for h in range(12)], axis=1)[0]
    assert cache.length == context + 1
    assert orf.relative_error(actual[:model], expected) < 0.05


def test_layernorm_within_two_percent(d, session) -> None:
    """check_layernorm (board_checks.py:335-359)."""
    s, images = session
    rng = np.random.default_rng(0)
    values = ob.bf16_grid((rng.standard_normal((32, 768)) * 2.0).astype(np.float32))
    gamma = ob.bf16_grid((1.0 + 0.1 * rng.standard_normal(768)).astype(np.float32))
    beta = ob.bf16_grid((0.1 * rng.standard_normal(768)).astype(np.float32))
    scalars = images.entries("layernorm")[0]["scalars"]
    d_rows, out = s.rows_in(values), s.packed(32, 768)
    d.run(d.norm_launches(images, d_rows, s.norm(gamma, beta, scalars), out))
    assert orf.relative_error(s.rows_out(out), orf.layernorm_device(values, gamma, beta)) < 0.02


def test_kv_cache_holds_every_token_exactly(d, session) -> None:
    """check_kv_cache (board_checks.py:362-387)."""
    s, images = session
    rng = np.random.default_rng(31)
    prefill = ob.bf16_grid(rng.standard_normal((64, 3 * 768)).astype(np.float32))
    step = ob.bf16_grid(rng.standard_normal((32, 3 * 768)).astype(np.float32))
    d_prefill, d_step = s.rows_in(prefill), s.rows_in(step)
    cache = d.PackedCache(s, images, capacity=96)
    d.run(cache.fill_launches(d_prefill, 64))
    d.run([cache.push_launch(d_step)])
    held = s.rows_out(cache.tensor)[:cache.length]
    np.testing.assert_array_equal(held, np.concatenate([prefill[:, 768:], step[:1, 768:]]))


def test_cache_refuses_a_prefill_past_its_room(d, session) -> None:
    s, images = session
    cache = d.PackedCache(s, images, capacity=64)
    fused = s.packed(96, 3 * 768)
    with pytest.raises(ValueError):
        cache.fill_launches(fused, 96)


@pytest.fixture(scope="module")
def model():
    from tempo_compiler_b200.weights import random_gpt2
    return random_gpt2(7)


def test_transformer_block_within_five_percent(d) -> None:
    """check_transformer_block (board_checks.py:485-518): [64, 768], the board check's weights, one layer's prefill."""
    rng = np.random.default_rng(1)
    hidden = ob.bf16_grid((rng.standard_normal((64, 768)) * 0.5).astype(np.float32))
    weights = _block_weights(768, 2)
    shared = {"wte": np.zeros((8, 768), np.float32), "wpe": np.zeros((64, 768), np.float32),
              "ln_f.g": np.ones(768, np.float32), "ln_f.b": np.zeros(768, np.float32)}
    net = d.PackedGPT2([weights], shared, capacity=64)
    try:
        actual = net.forward_rows(hidden)
        assert [cache.length for cache in net.caches] == [64]
    finally:
        net.close()
    assert orf.relative_error(actual, orf.block_device(hidden, weights)) < 0.05
    assert orf.relative_error(actual, orf.block_exact(hidden, weights)) < 0.02


def test_gpt2_prefill_layers_within_five_percent(d, model) -> None:
    """check_gpt2_prefill (board_checks.py:390-423): every layer held to the reference on its own device input."""
    layers, shared = model
    tokens = len(PROMPT)
    errors: list[float] = []

    def compare(index, layer_input, layer_output):
        expected = orf.block_device(layer_input, layers[index])
        errors.append(_layer_error(layer_output, expected, layer_input))

    net = d.PackedGPT2(layers, shared)
    try:
        net.prefill(np.asarray(PROMPT), observe=compare)
        lengths = {cache.length for cache in net.caches}
    finally:
        net.close()
    assert lengths == {tokens}
    assert len(errors) == len(layers)
    assert max(errors) < 0.05, errors


def test_gpt2_decode_layers_and_greedy_tokens(d, model) -> None:
    """check_gpt2_decode (board_checks.py:426-482): one decode step, each layer within 5%, and the two greedy tokens
    equal the reference chain's (full recompute through the device-rounding references)."""
    layers, shared = model
    tokens = len(PROMPT)
    prompt_inputs: dict[int, np.ndarray] = {}
    errors: list[float] = []

    def remember(index, layer_input, _):
        prompt_inputs[index] = layer_input

    def compare(index, layer_input, layer_output):
        rows = np.concatenate([prompt_inputs[index], layer_input])
        expected = orf.block_device(rows, layers[index])[-1]
        errors.append(_layer_error(layer_output[0], expected, layer_input[0]))

    net = d.PackedGPT2(layers, shared)
    try:
        first = int(np.argmax(net.prefill(np.asarray(PROMPT), observe=remember)))
        second = int(np.argmax(net.step(first, observe=compare)))
        lengths = {cache.length for cache in net.caches}
    finally:
        net.close()
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


def test_gpt2_generate_matches_step_by_step(d, model) -> None:
    """generate() is prefill plus greedy steps: eight tokens, the same as driving the steps by hand."""
    layers, shared = model
    net = d.PackedGPT2(layers, shared)
    try:
        tokens = net.generate(np.asarray(PROMPT), 8)
        by_hand = [int(np.argmax(net.prefill(np.asarray(PROMPT))))]
        while len(by_hand) < 8:
            by_hand.append(int(np.argmax(net.step(by_hand[-1]))))
    finally:
        net.close()
    assert tokens == by_hand


def test_runtime_error_classes(session) -> None:
    """The reference's exceptions for the same misuse (runtime/device.py:158-196, launch.py:67-141)."""
    from tempo_compiler_b200 import runtime
    _, images = session
    with pytest.raises(KeyError):
        runtime.minitpuFree(0x8000_0040 + 12345 * 32)
    with pytest.raises(MemoryError):
        runtime.minitpuMalloc(1 << 40)
    space = runtime.minitpuGetAddressSpace()
    halt = images.image_bytes("halt")
    junk = runtime.minitpuHostAlloc(64)
    junk.view[:16] = np.arange(16, dtype=np.uint32)
    address = runtime.minitpuMalloc(64)
    try:
        runtime.minitpuMemcpy(address, junk, 64, runtime.MemcpyKind.HostToDevice)
        with pytest.raises(RuntimeError):
            runtime.minitpuLaunchKernel(address, 64)
        with pytest.raises(ValueError):
            runtime.minitpuLaunchKernel(address + 16, 64)
        with pytest.raises(ValueError):
            runtime.minitpuLaunchKernel(space.kernel_base, len(halt), args=[1, 2, 3, 4, 5])
        with pytest.raises(ValueError):
            runtime.minitpuLaunchKernel(space.kernel_base, len(halt), args=[1 << 32])
        # an operand outside the arena is refused before the kernel runs
        add = images.get("add", features=768)
        with pytest.raises(ValueError, match="arena"):
            runtime.minitpuLaunchKernel(add.address, add.size, args=[0x10, 0x10, 0x10])
    finally:
        runtime.minitpuFree(address)
        runtime.minitpuHostReset()
