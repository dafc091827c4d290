"""Row statistics partials and the LayerNorm folded on them (tempo_gemm_rowstats, tempo_gemm_ln_rowstats,
tempo_row_stats): the residual projections write (mean, M2) of every 16-column chunk of the BF16 rows they store, and
the next projection combines them instead of a LayerNorm launch.

* gemm_rowstats stores the bits tempo_gemm stores (same kernels) and partials equal to float64 statistics of those
  stored rows, on every kernel the dispatch can pick: narrow full-K tiles, split-K over 2-8 CTAs, the row-major
  kernels and the CTA pair, a ragged N, GELU.
* row_stats matches float64 on its own.
* gemm_ln_rowstats against torch fp32 LayerNorm -> BF16 -> matmul (+ bias, GELU), rows with a large mean, on the
  split-K and narrow-tile paths, with the decode cache store; and against tempo_gemm_ln (statistics in the kernel).
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    yield
    from tempo_compiler_b200 import ops
    torch.cuda.synchronize()
    assert ops.watchdog() == 0


def _stats_f64(rows: torch.Tensor) -> np.ndarray:
    """(mean, M2) of each 16-column chunk, in float64."""
    x = rows.float().cpu().numpy().astype(np.float64)
    chunks = x.reshape(x.shape[0], -1, 16)
    mean = chunks.mean(axis=2)
    m2 = ((chunks - mean[:, :, None]) ** 2).sum(axis=2)
    return np.stack([mean, m2], axis=2)


def _check_stats(got: torch.Tensor, rows: torch.Tensor) -> None:
    want = _stats_f64(rows)
    got = got.cpu().numpy().astype(np.float64)
    scale = np.abs(rows.float().cpu().numpy()).reshape(want.shape[0], -1, 16).max(axis=2) + 1e-30
    # FP32 sums of 16 values: a few units of 2^-24 of the chunk's scale
    assert np.all(np.abs(got[:, :, 0] - want[:, :, 0]) <= 2e-6 * scale), "chunk means"
    assert np.all(np.abs(got[:, :, 1] - want[:, :, 1]) <= 2e-5 * 16 * scale * scale), "chunk M2"


@pytest.mark.parametrize(("m", "n", "k", "epilogue"), [
    (512, 768, 768, "residual"),     # split-K, 4 CTAs of 128 columns (the 512-row out-projection)
    (512, 768, 3072, "residual"),    # split-K over K = 3072 (the second MLP projection)
    (64, 768, 768, "residual"),      # narrow 16-column full-K tiles
    (64, 768, 3072, "residual"),     # split-K, 8 CTAs of 64 columns
    (33, 768, 3072, "bias"),
    (5, 768, 768, "residual"),       # a handful of rows: the tensor-core path (the GEMV has no statistics)
    (300, 784, 768, "residual"),     # N = 49 chunks: a ragged last tile
    (512, 3072, 768, "gelu"),
    (4096, 768, 768, "residual"),    # 128-column row-major tiles, TMA-store epilogue
    (32768, 768, 768, "residual"),   # the CTA pair
])
def test_gemm_rowstats_stores_the_gemm_and_its_statistics(m: int, n: int, k: int, epilogue: str) -> None:
    from tempo_compiler_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(m + 3 * n + k)
    a = torch.randn((m, k), generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn((n, k), generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    bias = (torch.randn(n, generator=g, device="cuda") * 0.1).to(torch.bfloat16)
    residual = (torch.randn((m, n), generator=g, device="cuda") * 2.0).to(torch.bfloat16) \
        if epilogue == "residual" else None
    stats = torch.full((m, n // 16, 2), float("nan"), dtype=torch.float32, device="cuda")
    out = ops.gemm_rowstats(a, w, stats, bias=bias, residual=residual, gelu=epilogue == "gelu")
    if m > 8:
        plain = ops.gemm(a, w, bias=bias, residual=residual, gelu=epilogue == "gelu")
        assert torch.equal(out, plain), "the statistics changed what the kernel stores"
    _check_stats(stats, out)


def test_row_stats_matches_float64() -> None:
    from tempo_compiler_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(4)
    x = (torch.randn((1000, 768), generator=g, device="cuda") * 5 + 30).to(torch.bfloat16)
    stats = torch.empty((1000, 48, 2), dtype=torch.float32, device="cuda")
    ops.row_stats(x, stats)
    _check_stats(stats, x)


def _layernorm_inputs(m: int, n: int, seed: int):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = (torch.randn((m, 768), generator=g, device="cuda") * 3.0
         + torch.randn((m, 1), generator=g, device="cuda") * 40.0).to(torch.bfloat16)
    gamma = (1.0 + 0.2 * torch.randn(768, generator=g, device="cuda")).to(torch.bfloat16)
    beta = (0.1 * torch.randn(768, generator=g, device="cuda")).to(torch.bfloat16)
    w = (torch.randn((n, 768), generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    bias = (torch.randn(n, generator=g, device="cuda") * 0.1).to(torch.bfloat16)
    return x, gamma, beta, w, bias


@pytest.mark.parametrize(("m", "n", "gelu"), [(512, 2304, False), (512, 3072, True), (64, 2304, False),
                                              (64, 3072, True), (200, 2304, False), (9, 3072, True)])
def test_gemm_ln_rowstats_matches_layernorm_then_gemm(m: int, n: int, gelu: bool) -> None:
    from tempo_compiler_b200 import ops
    from tempo_compiler_b200.engine import fold_layernorm
    x, gamma, beta, w, bias = _layernorm_inputs(m, n, m + n)
    folded, colsum, bias_folded = fold_layernorm(gamma, beta, w, bias)
    stats = torch.empty((m, 48, 2), dtype=torch.float32, device="cuda")
    ops.row_stats(x, stats)
    out = ops.gemm_ln_rowstats(x, folded, colsum, bias_folded, stats, epsilon=1e-5, gelu=gelu)
    ln = torch.nn.functional.layer_norm(x.float(), (768,), gamma.float(), beta.float(), 1e-5).to(torch.bfloat16)
    ref = ln.float() @ w.float().T + bias.float()
    if gelu:
        ref = torch.nn.functional.gelu(ref.to(torch.bfloat16).float())
    error = ((out.float() - ref).norm() / ref.norm()).item()
    assert error < 1e-2, error
    # the statistics computed in the kernel give nearly the same numbers
    inner = ops.gemm_ln(x, folded, colsum, bias_folded, epsilon=1e-5, gelu=gelu)
    assert ((out.float() - inner.float()).norm() / inner.float().norm()).item() < 2e-3


def test_gemm_ln_rowstats_stores_keys_and_values() -> None:
    from tempo_compiler_b200 import ops
    from tempo_compiler_b200.engine import fold_layernorm
    seqs, capacity = 300, 20
    x, gamma, beta, w, _ = _layernorm_inputs(seqs, 2304, 77)
    folded, colsum, bias_folded = fold_layernorm(gamma, beta, w, None)
    stats = torch.empty((seqs, 48, 2), dtype=torch.float32, device="cuda")
    ops.row_stats(x, stats)
    kc = torch.full((seqs, 12, capacity, 64), 7.0, dtype=torch.bfloat16, device="cuda")
    vc = torch.full_like(kc, 7.0)
    g = torch.Generator(device="cuda").manual_seed(5)
    positions = torch.randint(0, capacity + 3, (seqs,), generator=g, device="cuda", dtype=torch.int32)
    out = ops.gemm_ln_rowstats(x, folded, colsum, bias_folded, stats, k_cache=kc, v_cache=vc, positions=positions)
    expected_k, expected_v = torch.full_like(kc, 7.0), torch.full_like(vc, 7.0)
    for r in range(seqs):
        p = int(positions[r])
        if p < capacity:
            expected_k[r, :, p] = out[r, 768:1536].view(12, 64)
            expected_v[r, :, p] = out[r, 1536:].view(12, 64)
    assert torch.equal(kc, expected_k)
    assert torch.equal(vc, expected_v)


def test_limits_are_checked() -> None:
    from tempo_compiler_b200 import ops
    a = torch.zeros((64, 768), dtype=torch.bfloat16, device="cuda")
    w = torch.zeros((200, 768), dtype=torch.bfloat16, device="cuda")  # N not a multiple of 16
    stats = torch.zeros((64, 13, 2), dtype=torch.float32, device="cuda")
    with pytest.raises(ValueError):
        ops.gemm_rowstats(a, w, stats)
    with pytest.raises(ValueError):
        ops.gemm_rowstats(a, torch.zeros((768, 768), dtype=torch.bfloat16, device="cuda"), stats)  # too few floats
