"""Per-op parity of the B200 kernels against the oracle, through the C ABI.

Tolerances are the reference's own: GEMM rel-Frobenius < 1e-2 vs float64 and exact on structured operands
(board_package/board_checks.py:227-248), add exact (:285-288), LayerNorm < 2% vs the device model (:335-359),
causal attention < 2% and decode < 2-3% vs float64 (tests/test_mlir_attention.py:227,246), KV copies exact.
"""

from __future__ import annotations

import math

import numpy as np
import pytest

from oracle import bf16 as ob
from oracle import references as orf

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def _device():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from tempo_compiler_b200 import lib
    lib.load()
    yield
    from tempo_compiler_b200 import ops
    torch.cuda.synchronize()
    assert ops.watchdog() == 0


def _words(array_u16: np.ndarray) -> "torch.Tensor":
    return torch.from_numpy(np.ascontiguousarray(array_u16).view(np.int16)).cuda()


def _host(tensor) -> np.ndarray:
    return tensor.cpu().numpy().view(np.uint16)


def _bf16(values) -> "torch.Tensor":
    return torch.from_numpy(np.ascontiguousarray(values, np.float32)).cuda().to(torch.bfloat16)


def _packed_block(rows: np.ndarray) -> np.ndarray:
    """A packed device block: 512-byte zero tile then [features/16][32][16] words."""
    return np.concatenate([np.zeros(256, np.uint16), ob.pack_activations(rows)])


# ------------------------------------------------------------------------------------------------------------
# add / add_bias / layernorm / copy on the packed layout
# ------------------------------------------------------------------------------------------------------------

@pytest.mark.parametrize("features", [128, 768, 2304, 3072])
@pytest.mark.parametrize("broadcast", [False, True])
def test_block_add_is_exact(features: int, broadcast: bool) -> None:
    from tempo_compiler_b200 import ops
    rng = np.random.default_rng(features + broadcast)
    left = ob.bf16_grid(rng.standard_normal((32, features)).astype(np.float32))
    right = ob.bf16_grid(rng.standard_normal(features if broadcast else (32, features)).astype(np.float32))
    d_left = _words(ob.pack_activations(left))
    d_right = _words(ob.pack_bias(right) if broadcast else ob.pack_activations(right))
    d_out = torch.zeros_like(d_left)
    ops.block_add(d_left, d_right, d_out, features, broadcast)
    got = ob.unpack_activations(_host(d_out), tokens=32, features=features)
    np.testing.assert_array_equal(got, ob.bf16_grid(left + right))


def test_block_layernorm_matches_device_model() -> None:
    from tempo_compiler_b200 import ops
    rng = np.random.default_rng(0)
    rows = ob.bf16_grid((rng.standard_normal((32, 768)) * 2.0).astype(np.float32))
    gamma = ob.bf16_grid((1.0 + 0.1 * rng.standard_normal(768)).astype(np.float32))
    beta = ob.bf16_grid((0.1 * rng.standard_normal(768)).astype(np.float32))
    constants = ob.bf16_bits(np.concatenate([gamma, beta, np.full(64, 1 / 768, np.float32),
                                             np.full(64, 9.999999747378752e-06, np.float32)]))
    d_rows = _words(ob.pack_activations(rows))
    d_out = torch.zeros_like(d_rows)
    ops.block_layernorm(d_rows, _words(constants), d_out, 768)
    got = ob.unpack_activations(_host(d_out), tokens=32, features=768)
    assert orf.relative_error(got, orf.layernorm_device(rows, gamma, beta)) < 0.02
    assert orf.relative_error(got, orf.layernorm_f64(rows, gamma, beta)) < 0.005


@pytest.mark.parametrize(("rows", "stride"), [(1, 32), (96, 1024), (129, 32), (300, 64), (3072, 32)])
def test_block_copy_moves_exactly_the_rows(rows: int, stride: int) -> None:
    from tempo_compiler_b200 import ops
    span = rows * stride
    source = np.random.default_rng(rows + stride).integers(0, 1 << 16, span // 2, dtype=np.uint16)
    d_src = _words(source)
    d_dst = torch.zeros_like(d_src)
    ops.block_copy(d_src.data_ptr(), d_dst.data_ptr(), rows, stride)
    got = _host(d_dst)
    moved = np.zeros(span // 2, dtype=bool)
    for row in range(rows):
        moved[row * stride // 2: row * stride // 2 + 16] = True
    np.testing.assert_array_equal(got[moved], source[moved])
    assert not got[~moved].any()


# ------------------------------------------------------------------------------------------------------------
# the packed per-block GEMM (tcgen05, swap-AB)
# ------------------------------------------------------------------------------------------------------------

def _run_block_gemm(left, right, bias, activate):
    from tempo_compiler_b200 import ops
    depth, columns = right.shape
    d_act = _words(ob.pack_activations(left))
    d_w = _words(ob.pack_weights(right))
    d_bias = _words(ob.pack_bias(bias)) if bias is not None else None
    d_drain = torch.zeros(256 + columns * 32, dtype=torch.int16, device="cuda")
    ops.block_gemm(d_act, d_w, d_drain, d_bias, depth, columns, activate)
    torch.cuda.synchronize()
    words = _host(d_drain)
    assert not words[:256].any(), "the clearing tile must stay zero"
    return ob.unpack_activations(words[256:], tokens=32, features=columns)


def test_block_gemm_structured_operands_are_exact() -> None:
    left, right = ob.build_operands(32, 768, 3072, kind="structured", seed=0)
    np.testing.assert_array_equal(_run_block_gemm(left, right, None, False), (left @ right).astype(np.float32))


@pytest.mark.parametrize(("depth", "columns"), [(768, 3072), (768, 768), (768, 2304), (3072, 768), (64, 16),
                                                (96, 48), (4128, 48)])
def test_block_gemm_varying_operands_within_one_percent(depth: int, columns: int) -> None:
    left, right = ob.build_operands(32, depth, columns, kind="varying", seed=0)
    error = orf.relative_error(_run_block_gemm(left, right, None, False), orf.gemm_f64(left, right))
    assert error < 0.01, error


@pytest.mark.parametrize(("depth", "columns", "activate"), [(768, 768, False), (3072, 768, True), (768, 3072, True)])
def test_block_gemm_folds_bias_and_gelu(depth: int, columns: int, activate: bool) -> None:
    left, right = ob.build_operands(32, depth, columns, kind="varying", seed=0)
    right = ob.bf16_grid(right * np.float32(0.02))
    bias = ob.bf16_grid(np.random.default_rng(1).standard_normal(columns).astype(np.float32))
    expected = orf.gemm_f64(left, right, bias=bias, activate=activate)
    error = orf.relative_error(_run_block_gemm(left, right, bias, activate), expected)
    assert error < 0.01, error


def test_block_gemm_deep_contraction_is_exact() -> None:
    """Sparse small-integer operands whose every partial sum BF16 holds: any dropped or repeated k-tile shows
    (tests/test_mlir_padding.py:208-221)."""
    rng = np.random.default_rng(3)
    depth, columns = 4112, 48
    left = ((rng.random((32, depth)) < 16 / depth) * rng.choice([1.0, 2.0], (32, depth))).astype(np.float32)
    right = rng.choice([-1.0, 0.5, 1.0], (depth, columns)).astype(np.float32)
    offsets = rng.integers(-4, 4, columns).astype(np.float32)
    np.testing.assert_array_equal(_run_block_gemm(left, right, offsets, False), left @ right + offsets)


# ------------------------------------------------------------------------------------------------------------
# the native row-major GEMM (tcgen05, persistent, double-buffered accumulators)
# ------------------------------------------------------------------------------------------------------------

@pytest.mark.parametrize(("m", "n", "k"), [(128, 256, 64), (1024, 2304, 768), (1000, 768, 768), (512, 3072, 768),
                                           (64, 768, 3072), (300, 200, 136), (4096, 768, 3072), (16000, 768, 768),
                                           # decode-sized shapes: full-K tiles of 16-128 columns at K <= 1024,
                                           (512, 2304, 768), (512, 768, 768), (64, 2304, 768), (200, 3072, 768),
                                           (384, 2304, 768), (256, 768, 768),
                                           # the cluster split-K path beyond (2, 4 and 8 splits)
                                           (33, 768, 3072), (512, 2304, 2048), (384, 768, 3072), (200, 768, 3072),
                                           (512, 768, 3072)])
@pytest.mark.parametrize("epilogue", ["plain", "bias", "gelu", "residual"])
def test_gemm_matches_fp32_reference(m: int, n: int, k: int, epilogue: str) -> None:
    from tempo_compiler_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(m * 7 + n + k)
    a = torch.randn((m, k), generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn((n, k), generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    bias = (torch.randn(n, generator=g, device="cuda") * 0.1).to(torch.bfloat16) if epilogue != "plain" else None
    residual = torch.randn((m, n), generator=g, device="cuda").to(torch.bfloat16) if epilogue == "residual" else None
    out = ops.gemm(a, w, bias=bias, residual=residual, gelu=epilogue == "gelu")
    ref = a.float() @ w.float().T
    if bias is not None:
        ref = ref + bias.float()
    if epilogue == "gelu":
        ref = torch.nn.functional.gelu(ref.to(torch.bfloat16).float())
    if residual is not None:
        ref = ref + residual.float()
    error = ((out.float() - ref).norm() / ref.norm()).item()
    assert error < 5e-3, error
    assert torch.isfinite(out.float()).all()


@pytest.mark.parametrize("m_extra", [0, 60000])
def test_gemm_gelu_on_every_bf16_input(m_extra: int) -> None:
    """GELU's input is the BF16-rounded sum, so every finite BF16 value with |x| <= 14 (the rows of A, times an
    identity weight) covers all its inputs; beyond 14 GELU(x) is x or a value flushed to zero. Against float64
    erfc: correctly rounded for all but a handful, never more than one BF16 step off. m_extra pads M with zero rows
    so the prefill kernels run it too."""
    from tempo_compiler_b200 import ops
    bits = (torch.arange(1 << 16, dtype=torch.int32) << 16).view(torch.float32)
    x = bits[torch.isfinite(bits) & (bits.abs() <= 14) & (bits.abs() >= 1e-30)]
    cols = 128
    rows = (x.numel() + cols - 1) // cols
    a = torch.zeros(rows * cols + m_extra * cols)
    a[:x.numel()] = x
    a = a.view(-1, cols).to(torch.bfloat16).cuda()
    eye = torch.eye(cols, dtype=torch.bfloat16, device="cuda")
    out = ops.gemm(a, eye, gelu=True).flatten()[:x.numel()].cpu()
    xd = x.double()
    exact = 0.5 * xd * torch.special.erfc(-xd / math.sqrt(2.0))
    want = exact.to(torch.bfloat16)
    normal = (exact / xd).abs() >= 2.0 ** -126  # Phi(x) below the smallest normal float flushes to zero
    assert (out[~normal].float().abs() <= x[~normal].abs() * 2.0 ** -126).all()
    as_int = lambda t: t.view(torch.int16).int()
    steps = (as_int(out) - as_int(want)).abs()[normal]
    assert steps.max().item() <= 1, float(x[normal][steps.argmax()])
    assert (steps > 0).sum().item() <= 16, (steps > 0).sum().item()


@pytest.mark.parametrize("m", [1, 3, 8])
def test_gemm_norm_has_the_bits_of_layernorm_then_gemm(m: int) -> None:
    """tempo_gemm_norm against tempo_layernorm followed by the same projection: QKV with the cache store, FC with
    GELU, and the LM head's argmax partials -- identical outputs, caches and partials."""
    from tempo_compiler_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(m + 100)
    x = (torch.randn((m, 768), generator=g, device="cuda") * 3 + 0.5).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(768, generator=g, device="cuda")).to(torch.bfloat16)
    beta = (0.1 * torch.randn(768, generator=g, device="cuda")).to(torch.bfloat16)
    ln = ops.layernorm(x, gamma, beta, epsilon=1e-5)
    # QKV + bias + cache store at positions
    w = (torch.randn((2304, 768), generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    b = (torch.randn(2304, generator=g, device="cuda") * 0.1).to(torch.bfloat16)
    positions = torch.arange(m, dtype=torch.int32, device="cuda") * 5 + 3
    caches = [torch.zeros((m, 12, 64, 64), dtype=torch.bfloat16, device="cuda") for _ in range(4)]
    want = torch.empty((m, 2304), dtype=torch.bfloat16, device="cuda")
    ops.gemm_qkv(ln, w, b, want, caches[0], caches[1], positions=positions)
    got = ops.gemm_norm(x, gamma, beta, w, epsilon=1e-5, bias=b, k_cache=caches[2], v_cache=caches[3],
                        positions=positions)
    assert torch.equal(got, want)
    assert torch.equal(caches[2], caches[0]) and torch.equal(caches[3], caches[1])
    assert caches[2].abs().sum() > 0
    # FC + bias + GELU
    w = (torch.randn((3072, 768), generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    b = (torch.randn(3072, generator=g, device="cuda") * 0.1).to(torch.bfloat16)
    assert torch.equal(ops.gemm_norm(x, gamma, beta, w, epsilon=1e-5, bias=b, gelu=True),
                       ops.gemm(ln, w, bias=b, gelu=True))
    # LM head argmax partials
    wte = (torch.randn((50257, 768), generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    tiles = (50257 + 255) // 256
    parts = [torch.empty((m, tiles), dtype=dt, device="cuda") for dt in (torch.float32, torch.int32) * 2]
    ops.gemm_argmax(ln, wte, parts[0], parts[1])
    ops.gemm_norm(x, gamma, beta, wte, epsilon=1e-5, part_val=parts[2], part_idx=parts[3])
    assert torch.equal(parts[0], parts[2]) and torch.equal(parts[1], parts[3])


def test_gemm_norm_refuses_more_than_8_rows() -> None:
    from tempo_compiler_b200 import ops
    x = torch.zeros((9, 768), dtype=torch.bfloat16, device="cuda")
    ones = torch.ones(768, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        ops.gemm_norm(x, ones, ones, torch.zeros((64, 768), dtype=torch.bfloat16, device="cuda"))


def test_stream_read_folds_every_word() -> None:
    """The calibration read touches every word of a source of whole groups: the XOR of its sink words is the XOR of
    all source words."""
    import ctypes
    from tempo_compiler_b200 import lib, ops
    threads = ctypes.c_uint32()
    lib.call("tempo_stream_read_threads", ctypes.byref(threads))
    words = threads.value * 8 * 3
    src = torch.randint(-2**31, 2**31 - 1, (words * 4,), dtype=torch.int32, device="cuda")
    sink = ops.stream_read(src)
    torch.cuda.synchronize()
    fold = lambda t: np.bitwise_xor.reduce(t.cpu().numpy().view(np.uint32).reshape(-1, 4), axis=0)  # noqa: E731
    np.testing.assert_array_equal(fold(sink), fold(src))


@pytest.mark.parametrize("m", [1, 2, 3, 5, 8])
@pytest.mark.parametrize(("n", "k"), [(2304, 768), (768, 3072), (200, 136)])
@pytest.mark.parametrize("epilogue", ["bias", "gelu", "residual"])
def test_gemv_path_for_few_rows_matches_fp32(m: int, n: int, k: int, epilogue: str) -> None:
    """At most 8 rows take the weight-streaming GEMV kernel; same epilogues, same tolerance."""
    from tempo_compiler_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(m * 131 + n + k)
    a = torch.randn((m, k), generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn((n, k), generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    bias = (torch.randn(n, generator=g, device="cuda") * 0.1).to(torch.bfloat16)
    residual = torch.randn((m, n), generator=g, device="cuda").to(torch.bfloat16) if epilogue == "residual" else None
    out = ops.gemm(a, w, bias=bias, residual=residual, gelu=epilogue == "gelu")
    ref = a.float() @ w.float().T + bias.float()
    if epilogue == "gelu":
        ref = torch.nn.functional.gelu(ref.to(torch.bfloat16).float())
    if residual is not None:
        ref = ref + residual.float()
    error = ((out.float() - ref).norm() / ref.norm()).item()
    assert error < 5e-3, error


@pytest.mark.parametrize("m", [1, 3, 8, 200])
def test_gemm_argmax_small_and_large_batches(m: int) -> None:
    from tempo_compiler_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(17 + m)
    a = torch.randn((m, 768), generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn((50257, 768), generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    tiles = (50257 + 255) // 256
    part_val = torch.empty((m, tiles), dtype=torch.float32, device="cuda")
    part_idx = torch.empty((m, tiles), dtype=torch.int32, device="cuda")
    ids = torch.empty(m, dtype=torch.int32, device="cuda")
    ops.gemm_argmax(a, w, part_val, part_idx)
    ops.argmax_finish(part_val, part_idx, ids)
    logits = a.float() @ w.float().T
    top2 = logits.topk(2, dim=1).values
    clear = (top2[:, 0] - top2[:, 1]) > 1e-3
    assert torch.equal(ids[clear], logits.argmax(dim=1).to(torch.int32)[clear])


@pytest.mark.parametrize(("seqs", "tokens", "decode"), [(3, 40, False), (2, 1000, False), (5, 1, True),
                                                         (64, 1, True), (300, 1, True)])
def test_gemm_qkv_writes_keys_and_values_into_the_cache(seqs: int, tokens: int, decode: bool) -> None:
    """The fused KV write: every row's key and value columns land in the cache exactly as the product computed them,
    rows past the capacity are skipped, and nothing else in the cache is touched."""
    from tempo_compiler_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(seqs + tokens)
    rows = seqs * tokens
    capacity = 48 if not decode else 16
    a = torch.randn((rows, 768), generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn((2304, 768), generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    bias = (torch.randn(2304, generator=g, device="cuda") * 0.1).to(torch.bfloat16)
    kc = torch.full((seqs, 12, max(capacity, tokens), 64), 7.0, dtype=torch.bfloat16, device="cuda")
    vc = torch.full_like(kc, 7.0)
    capacity = kc.shape[2]
    out = torch.empty((rows, 2304), dtype=torch.bfloat16, device="cuda")
    positions = None
    if decode:
        positions = torch.randint(0, capacity + 3, (seqs,), generator=g, device="cuda", dtype=torch.int32)
        ops.gemm_qkv(a, w, bias, out, kc, vc, positions=positions)
    else:
        ops.gemm_qkv(a, w, bias, out, kc, vc, tokens_per_seq=tokens)
    reference = ops.gemm(a, w, bias=bias)
    assert torch.equal(out, reference)
    expected_k = torch.full_like(kc, 7.0)
    expected_v = torch.full_like(vc, 7.0)
    for r in range(rows):
        s, p = (r, int(positions[r])) if decode else (r // tokens, r % tokens)
        if p >= capacity:
            continue
        expected_k[s, :, p] = reference[r, 768:1536].view(12, 64)
        expected_v[s, :, p] = reference[r, 1536:].view(12, 64)
    assert torch.equal(kc, expected_k)
    assert torch.equal(vc, expected_v)


@pytest.mark.parametrize(("m", "n", "k", "epilogue"), [(20000, 3072, 768, "gelu"), (20000, 2304, 768, "bias"),
                                                      (25700, 768, 3072, "residual"), (19000, 3000, 768, "plain")])
def test_pair_gemm_matches_fp32_reference(m: int, n: int, k: int, epilogue: str) -> None:
    """Prefill-sized products (256 x 256 tiles on CTA pairs), ragged M and N included."""
    from tempo_compiler_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    a = torch.randn((m, k), generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn((n, k), generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    bias = (torch.randn(n, generator=g, device="cuda") * 0.1).to(torch.bfloat16) if epilogue != "plain" else None
    residual = torch.randn((m, n), generator=g, device="cuda").to(torch.bfloat16) if epilogue == "residual" else None
    out = ops.gemm(a, w, bias=bias, residual=residual, gelu=epilogue == "gelu")
    ref = a.float() @ w.float().T
    if bias is not None:
        ref += bias.float()
    if epilogue == "gelu":
        ref = torch.nn.functional.gelu(ref.to(torch.bfloat16).float())
    if residual is not None:
        ref += residual.float()
    error = ((out.float() - ref).norm() / ref.norm()).item()
    assert error < 5e-3, error
    assert torch.isfinite(out).all()
    assert ops.watchdog() == 0


def test_pair_gemm_qkv_prefill_cache_store() -> None:
    """The prefill QKV projection of 20 x 1024 tokens on CTA pairs stores every key and value into the caches."""
    from tempo_compiler_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(11)
    seqs, tokens = 20, 1024
    a = torch.randn((seqs * tokens, 768), generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn((2304, 768), generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    bias = (torch.randn(2304, generator=g, device="cuda") * 0.1).to(torch.bfloat16)
    kc = torch.zeros((seqs, 12, tokens, 64), dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    out = torch.empty((seqs * tokens, 2304), dtype=torch.bfloat16, device="cuda")
    ops.gemm_qkv(a, w, bias, out, kc, vc, tokens_per_seq=tokens)
    ref = a.float() @ w.float().T + bias.float()
    assert ((out.float() - ref).norm() / ref.norm()).item() < 5e-3
    assert torch.equal(kc, out[:, 768:1536].reshape(seqs, tokens, 12, 64).transpose(1, 2))
    assert torch.equal(vc, out[:, 1536:].reshape(seqs, tokens, 12, 64).transpose(1, 2))


@pytest.mark.parametrize(("m", "n", "gelu"), [(3, 2304, False), (64, 2304, False), (64, 3072, True),
                                               (128, 3072, True), (200, 2304, False), (512, 3072, True)])
def test_gemm_ln_matches_layernorm_then_gemm(m: int, n: int, gelu: bool) -> None:
    """LayerNorm folded into the projection: against torch fp32 LayerNorm -> BF16 -> matmul (+ bias, GELU), with
    non-trivial gamma / beta and rows whose mean is far from zero (the in-kernel statistics are centred)."""
    from tempo_compiler_b200 import ops
    from tempo_compiler_b200.engine import fold_layernorm
    g = torch.Generator(device="cuda").manual_seed(m + n)
    x = (torch.randn((m, 768), generator=g, device="cuda") * 3.0
         + torch.randn((m, 1), generator=g, device="cuda") * 40.0).to(torch.bfloat16)
    gamma = (1.0 + 0.2 * torch.randn(768, generator=g, device="cuda")).to(torch.bfloat16)
    beta = (0.1 * torch.randn(768, generator=g, device="cuda")).to(torch.bfloat16)
    w = (torch.randn((n, 768), generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    bias = (torch.randn(n, generator=g, device="cuda") * 0.1).to(torch.bfloat16)
    folded, colsum, bias_folded = fold_layernorm(gamma, beta, w, bias)
    out = ops.gemm_ln(x, folded, colsum, bias_folded, epsilon=1e-5, gelu=gelu)
    ln = torch.nn.functional.layer_norm(x.float(), (768,), gamma.float(), beta.float(), 1e-5).to(torch.bfloat16)
    ref = ln.float() @ w.float().T + bias.float()
    if gelu:
        ref = torch.nn.functional.gelu(ref.to(torch.bfloat16).float())
    error = ((out.float() - ref).norm() / ref.norm()).item()
    assert error < 1e-2, error
    assert ops.watchdog() == 0


def test_gemm_ln_refuses_more_tiles_than_sms() -> None:
    """The folded LayerNorm runs one output tile per CTA; a product needing more is refused, not mis-computed."""
    from tempo_compiler_b200 import ops
    from tempo_compiler_b200.engine import fold_layernorm
    x = torch.zeros((8192, 768), dtype=torch.bfloat16, device="cuda")
    w = torch.zeros((3072, 768), dtype=torch.bfloat16, device="cuda")
    one = torch.ones(768, dtype=torch.bfloat16, device="cuda")
    folded, colsum, bias_folded = fold_layernorm(one, one * 0, w, None)
    with pytest.raises(ValueError, match="one 128-row tile per SM"):
        ops.gemm_ln(x, folded, colsum, bias_folded)


def test_gemm_ln_stores_keys_and_values() -> None:
    """The folded QKV projection with the decode cache store: the caches receive exactly its key and value columns."""
    from tempo_compiler_b200 import ops
    from tempo_compiler_b200.engine import fold_layernorm
    g = torch.Generator(device="cuda").manual_seed(77)
    seqs, capacity = 40, 20
    x = torch.randn((seqs, 768), generator=g, device="cuda").to(torch.bfloat16)
    gamma = (1.0 + 0.1 * torch.randn(768, generator=g, device="cuda")).to(torch.bfloat16)
    beta = (0.1 * torch.randn(768, generator=g, device="cuda")).to(torch.bfloat16)
    w = (torch.randn((2304, 768), generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    folded, colsum, bias_folded = fold_layernorm(gamma, beta, w, None)
    kc = torch.full((seqs, 12, capacity, 64), 7.0, dtype=torch.bfloat16, device="cuda")
    vc = torch.full_like(kc, 7.0)
    positions = torch.randint(0, capacity + 3, (seqs,), generator=g, device="cuda", dtype=torch.int32)
    out = ops.gemm_ln(x, folded, colsum, bias_folded, k_cache=kc, v_cache=vc, positions=positions)
    expected_k, expected_v = torch.full_like(kc, 7.0), torch.full_like(vc, 7.0)
    for r in range(seqs):
        p = int(positions[r])
        if p < capacity:
            expected_k[r, :, p] = out[r, 768:1536].view(12, 64)
            expected_v[r, :, p] = out[r, 1536:].view(12, 64)
    assert torch.equal(kc, expected_k)
    assert torch.equal(vc, expected_v)


def test_gemm_argmax_matches_torch() -> None:
    from tempo_compiler_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(5)
    a = torch.randn((200, 768), generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn((50257, 768), generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    tiles = (50257 + 255) // 256
    part_val = torch.empty((200, tiles), dtype=torch.float32, device="cuda")
    part_idx = torch.empty((200, tiles), dtype=torch.int32, device="cuda")
    ids = torch.empty(200, dtype=torch.int32, device="cuda")
    ops.gemm_argmax(a, w, part_val, part_idx)
    ops.argmax_finish(part_val, part_idx, ids)
    logits = a.float() @ w.float().T
    expected = logits.argmax(dim=1).to(torch.int32)
    top2 = logits.topk(2, dim=1).values
    clear = (top2[:, 0] - top2[:, 1]) > 1e-3
    assert torch.equal(ids[clear], expected[clear])
    assert clear.float().mean().item() > 0.9


# ------------------------------------------------------------------------------------------------------------
# attention
# ------------------------------------------------------------------------------------------------------------

def _fused_packed(fused: np.ndarray) -> np.ndarray:
    """A packed fused QKV tensor: per 32-token block a zero tile and its [144][32][16] tiles."""
    blocks = [_packed_block(fused[b * 32:(b + 1) * 32]) for b in range(fused.shape[0] // 32)]
    return np.concatenate(blocks)


def _unpack_fused(words: np.ndarray, tokens: int, features: int) -> np.ndarray:
    per = 256 + 32 * features
    return np.concatenate([ob.unpack_activations(words[b * per + 256:(b + 1) * per], tokens=32, features=features)
                           for b in range(tokens // 32)])


@pytest.mark.parametrize("tokens", [32, 64, 160, 256, 1024])
def test_block_causal_attention_within_two_percent(tokens: int) -> None:
    from tempo_compiler_b200 import ops
    rng = np.random.default_rng(tokens)
    fused = ob.bf16_grid(rng.standard_normal((tokens, 3 * 768)).astype(np.float32))
    fused[:, :768] = ob.bf16_grid(fused[:, :768] / 8.0)  # the queries arrive scaled by 1/sqrt(64)
    d_fused = _words(_fused_packed(fused))
    constants = _words(ob.causal_constants_words())
    ops.block_attention(constants, d_fused.data_ptr() + 512, tokens, 12)
    got = _unpack_fused(_host(d_fused), tokens, 3 * 768)
    np.testing.assert_array_equal(got[:, 768:], fused[:, 768:])  # keys and values untouched
    for h in range(12):
        cols = slice(h * 64, (h + 1) * 64)
        expected = orf.causal_attention_f64(fused[:, cols], fused[:, 768:][:, cols], fused[:, 1536:][:, cols])
        error = orf.relative_error(got[:, cols], expected)
        assert error < 0.02, (h, error)


@pytest.mark.parametrize(("seqs", "tokens"), [(1, 64), (2, 200), (3, 128), (1, 1024), (4, 384),
                                             (4, 1024),    # 384 (query tile, head, sequence) items: more than two per SM
                                             (24, 1000)])  # 2304 items over several waves, a ragged last query tile
def test_native_prefill_attention_matches_fp32(seqs: int, tokens: int) -> None:
    from tempo_compiler_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(seqs * 1000 + tokens)
    qkv = torch.randn((seqs * tokens, 3 * 768), generator=g, device="cuda").to(torch.bfloat16)
    qkv[:, :768] = (qkv[:, :768].float() / 8.0).to(torch.bfloat16)
    out = ops.attention_prefill(qkv, seqs, tokens, 12)
    q = qkv[:, :768].float().view(seqs, tokens, 12, 64).transpose(1, 2)
    k = qkv[:, 768:1536].float().view(seqs, tokens, 12, 64).transpose(1, 2)
    v = qkv[:, 1536:].float().view(seqs, tokens, 12, 64).transpose(1, 2)
    ref = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True, scale=1.0)
    ref = ref.transpose(1, 2).reshape(seqs * tokens, 768)
    error = ((out.float() - ref).norm() / ref.norm()).item()
    assert error < 0.01, error
    # every row and head, not only the norm: a wrong row would hide in the norm-wise figure
    row_error = ((out.float() - ref).abs().amax(dim=1) / ref.abs().amax(dim=1)).max().item()
    assert row_error < 0.05, row_error


@pytest.mark.parametrize(("keys", "length"), [(64, 1), (64, 49), (256, 200), (1024, 1024)])
def test_block_decode_attention_matches_float64(keys: int, length: int) -> None:
    from tempo_compiler_b200 import ops
    rng = np.random.default_rng(keys + length)
    fused = ob.bf16_grid(rng.standard_normal((32, 3 * 768)).astype(np.float32))
    cache = ob.bf16_grid(rng.standard_normal((keys, 2 * 768)).astype(np.float32))
    masks = ob.decode_mask_tiles(keys=keys, length=length)
    constants = ob.pack_attention_constants(initial_maximum=-1e30, constants=(),
                                            masks=np.ascontiguousarray(masks.swapaxes(-1, -2))).reshape(-1)
    d_fused = _words(_fused_packed(fused))
    d_cache = _words(_fused_packed_cache(cache))
    ops.block_decode_attention(_words(constants), d_cache.data_ptr() + 512, d_fused.data_ptr() + 512, keys, 12)
    got = _unpack_fused(_host(d_fused), 32, 3 * 768)
    expected = np.concatenate([orf.attention_f64(fused[:1, h * 64:(h + 1) * 64], cache[:length, h * 64:(h + 1) * 64],
                                                 cache[:length, 768 + h * 64:768 + (h + 1) * 64])
                               for h in range(12)], axis=1)[0]
    assert orf.relative_error(got[0, :768], expected) < (0.03 if keys > 256 else 0.02)
    np.testing.assert_array_equal(got[16:], fused[16:])  # only the first 16 query rows are written


def _fused_packed_cache(cache: np.ndarray) -> np.ndarray:
    return np.concatenate([_packed_block(cache[b * 32:(b + 1) * 32]) for b in range(cache.shape[0] // 32)])


@pytest.mark.parametrize(("seqs", "capacity", "lengths"), [
    (3, 64, (1, 33, 64)),               # one CTA per (sequence, head)
    (2, 1152, (1024, 1100)),            # eight CTAs per (sequence, head), the last one's key range empty
    (4, 512, (0, 1, 200, 512)),         # four per pair: empty, single-key and ragged lengths
    (90, 256, tuple(range(1, 91))),     # two per pair, every length 1..90
    (1, 383, (129,)),                   # four per pair of 64-key chunks, the last two empty
    (2, 383, (383, 200)),               # four per pair, a full and a ragged cache
])
def test_native_decode_attention_matches_fp32(seqs: int, capacity: int, lengths) -> None:
    from tempo_compiler_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(capacity)
    qkv = torch.randn((seqs, 3 * 768), generator=g, device="cuda").to(torch.bfloat16)
    kc = torch.randn((seqs, 12, capacity, 64), generator=g, device="cuda").to(torch.bfloat16)
    vc = torch.randn((seqs, 12, capacity, 64), generator=g, device="cuda").to(torch.bfloat16)
    lens = torch.tensor(lengths, dtype=torch.int32, device="cuda")
    out = ops.decode_attention(qkv, kc, vc, lens)
    for s, length in enumerate(lengths):
        if length == 0:
            assert not out[s].float().abs().any(), "an empty cache attends to nothing"
            continue
        q = qkv[s, :768].float().view(12, 1, 64)
        scores = q @ kc[s, :, :length].float().transpose(1, 2)
        ref = (scores.softmax(-1) @ vc[s, :, :length].float()).reshape(768)
        error = ((out[s].float() - ref).norm() / ref.norm()).item()
        assert error < 0.01, (s, error)


# ------------------------------------------------------------------------------------------------------------
# native LayerNorm, embedding, KV store
# ------------------------------------------------------------------------------------------------------------

def test_native_layernorm_matches_float64() -> None:
    from tempo_compiler_b200 import ops
    rng = np.random.default_rng(2)
    rows = ob.bf16_grid((rng.standard_normal((1000, 768)) * 2.0 + 0.5).astype(np.float32))
    gamma = ob.bf16_grid((1.0 + 0.1 * rng.standard_normal(768)).astype(np.float32))
    beta = ob.bf16_grid((0.1 * rng.standard_normal(768)).astype(np.float32))
    out = ops.layernorm(_bf16(rows), _bf16(gamma), _bf16(beta))
    assert orf.relative_error(out.float().cpu().numpy(), orf.layernorm_f64(rows, gamma, beta)) < 0.005


def test_embed_and_kv_store_are_exact() -> None:
    from tempo_compiler_b200 import ops
    rng = np.random.default_rng(4)
    wte = ob.bf16_grid((rng.standard_normal((1000, 768)) * 0.02).astype(np.float32))
    wpe = ob.bf16_grid((rng.standard_normal((64, 768)) * 0.02).astype(np.float32))
    ids = rng.integers(0, 1000, 40).astype(np.int32)
    pos = rng.integers(0, 64, 40).astype(np.int32)
    x = ops.embed(torch.from_numpy(ids).cuda(), torch.from_numpy(pos).cuda(), _bf16(wte), _bf16(wpe))
    np.testing.assert_array_equal(x.float().cpu().numpy(), ob.bf16_grid(wte[ids] + wpe[pos]))
    qkv = torch.randn((40, 2304), device="cuda").to(torch.bfloat16)
    kc = torch.zeros((4, 12, 16, 64), dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    seq_of = torch.arange(40, dtype=torch.int32, device="cuda") % 4
    pos_of = torch.arange(40, dtype=torch.int32, device="cuda") // 4
    ops.kv_store(qkv, kc, vc, seq_of, pos_of)
    for r in range(40):
        s, p = r % 4, r // 4
        assert torch.equal(kc[s, :, p].reshape(768), qkv[r, 768:1536])
        assert torch.equal(vc[s, :, p].reshape(768), qkv[r, 1536:])
