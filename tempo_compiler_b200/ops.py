"""torch-tensor wrappers over the native C-ABI entry points (section 3 of include/tempo_b200.h).

torch supplies device memory and the current CUDA stream; every op passes raw pointers and sizes to
libtempo_b200.so, whose kernels do the work. Nothing here computes on its own, and nothing falls back: a CPU tensor,
a wrong dtype or a missing library raises.
"""

from __future__ import annotations

import ctypes

import torch

from tempo_compiler_b200 import lib as _lib


_LAUNCHES = [0]


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _launch(name: str, *args) -> None:
    """Calls one kernel-launching entry point of the library (one kernel per call) and counts it."""
    _LAUNCHES[0] += 1
    _lib.call(name, *args)


def reset_launch_count() -> None:
    _LAUNCHES[0] = 0


def launch_count() -> int:
    """Kernel launches issued through this module since the last reset (graph replays are not counted)."""
    return _LAUNCHES[0]


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _check(t: torch.Tensor, dtype: torch.dtype, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor: the B200 kernels have no CPU path")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def gemm(a: torch.Tensor, w_t: torch.Tensor, *, bias: torch.Tensor | None = None,
         residual: torch.Tensor | None = None, gelu: bool = False, out: torch.Tensor | None = None) -> torch.Tensor:
    """out[M, N] = epilogue(a[M, K] @ w_t[N, K]^T): + bias, exact-erf GELU (of the BF16-rounded sum), + residual."""
    _check(a, torch.bfloat16, "a")
    _check(w_t, torch.bfloat16, "w_t")
    m, k = a.shape
    n = w_t.shape[0]
    if w_t.shape[1] != k:
        raise ValueError(f"inner dimensions differ: a {tuple(a.shape)}, w_t {tuple(w_t.shape)}")
    if out is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=a.device)
    _check(out, torch.bfloat16, "out")
    if bias is not None:
        _check(bias, torch.bfloat16, "bias")
    if residual is not None:
        _check(residual, torch.bfloat16, "residual")
    flags = _lib.GEMM_GELU if gelu else 0
    _launch("tempo_gemm", a.data_ptr(), k, w_t.data_ptr(), k, _ptr(bias), _ptr(residual), n, out.data_ptr(), n, m, n,
              k, flags, None, None, _stream())
    return out


def gemm_qkv(a: torch.Tensor, w_t: torch.Tensor, bias: torch.Tensor, out: torch.Tensor, k_cache: torch.Tensor,
             v_cache: torch.Tensor, *, tokens_per_seq: int = 0, positions: torch.Tensor | None = None) -> torch.Tensor:
    """The QKV projection (+ bias) into `out`, its key and value columns also stored into the [seq][head][pos][64]
    caches: row r is sequence r // tokens_per_seq at r % tokens_per_seq, or sequence r at positions[r]."""
    _check(a, torch.bfloat16, "a")
    _check(w_t, torch.bfloat16, "w_t")
    _check(out, torch.bfloat16, "out")
    m, k = a.shape
    seqs, heads, capacity, head = k_cache.shape
    _launch("tempo_gemm_qkv", a.data_ptr(), k, w_t.data_ptr(), k, bias.data_ptr(), out.data_ptr(), out.shape[1], m, k,
            k_cache.data_ptr(), v_cache.data_ptr(), seqs, heads, head, capacity, tokens_per_seq, _ptr(positions),
            _stream())
    return out


def gemm_ln(x: torch.Tensor, w_folded: torch.Tensor, colsum: torch.Tensor, bias_folded: torch.Tensor, *,
            epsilon: float = 1e-5, gelu: bool = False, out: torch.Tensor | None = None,
            k_cache: torch.Tensor | None = None, v_cache: torch.Tensor | None = None,
            positions: torch.Tensor | None = None) -> torch.Tensor:
    """out = epilogue(LayerNorm(x) @ W + b) with the LayerNorm folded into the weights: w_folded[N, K] = (gamma * W)^T
    in BF16, colsum[N] = its FP32 row sums, bias_folded[N] = b + beta @ W in FP32; the row statistics are computed in
    the kernel. With the caches (and positions) the key and value columns are also stored, as in gemm_qkv decode."""
    _check(x, torch.bfloat16, "x")
    _check(w_folded, torch.bfloat16, "w_folded")
    _check(colsum, torch.float32, "colsum")
    _check(bias_folded, torch.float32, "bias_folded")
    m, k = x.shape
    n = w_folded.shape[0]
    if w_folded.shape[1] != k:
        raise ValueError(f"inner dimensions differ: x {tuple(x.shape)}, w_folded {tuple(w_folded.shape)}")
    if out is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=x.device)
    _check(out, torch.bfloat16, "out")
    seqs = heads = head = capacity = 0
    if k_cache is not None:
        seqs, heads, capacity, head = k_cache.shape
    _launch("tempo_gemm_ln", x.data_ptr(), k, w_folded.data_ptr(), k, colsum.data_ptr(), bias_folded.data_ptr(),
            float(epsilon), out.data_ptr(), out.shape[1], m, n, k, _lib.GEMM_GELU if gelu else 0, _ptr(k_cache),
            _ptr(v_cache), seqs, heads, head, capacity, _ptr(positions), _stream())
    return out


def gemm_rowstats(a: torch.Tensor, w_t: torch.Tensor, row_stats: torch.Tensor, *, bias: torch.Tensor | None = None,
                  residual: torch.Tensor | None = None, gelu: bool = False,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """gemm that also writes the statistics partials of its BF16 output rows into row_stats [M, N / 16, 2] (FP32
    mean and M2 of each 16-column chunk), for the folded LayerNorm of the projection that reads those rows next."""
    _check(a, torch.bfloat16, "a")
    _check(w_t, torch.bfloat16, "w_t")
    _check(row_stats, torch.float32, "row_stats")
    m, k = a.shape
    n = w_t.shape[0]
    if w_t.shape[1] != k:
        raise ValueError(f"inner dimensions differ: a {tuple(a.shape)}, w_t {tuple(w_t.shape)}")
    if row_stats.numel() < m * n // 8:
        raise ValueError(f"row_stats holds {row_stats.numel()} floats, {m * n // 8} needed")
    if out is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=a.device)
    _check(out, torch.bfloat16, "out")
    _launch("tempo_gemm_rowstats", a.data_ptr(), k, w_t.data_ptr(), k, _ptr(bias), _ptr(residual), n, out.data_ptr(),
            n, m, n, k, _lib.GEMM_GELU if gelu else 0, row_stats.data_ptr(), _stream())
    return out


def gemm_ln_rowstats(x: torch.Tensor, w_folded: torch.Tensor, colsum: torch.Tensor, bias_folded: torch.Tensor,
                     row_stats: torch.Tensor, *, epsilon: float = 1e-5, gelu: bool = False,
                     out: torch.Tensor | None = None, k_cache: torch.Tensor | None = None,
                     v_cache: torch.Tensor | None = None, positions: torch.Tensor | None = None) -> torch.Tensor:
    """gemm_ln with the rows' statistics combined from row_stats [M, K / 16, 2] (gemm_rowstats' or row_stats'
    partials of x) instead of computed in the kernel."""
    _check(x, torch.bfloat16, "x")
    _check(w_folded, torch.bfloat16, "w_folded")
    _check(colsum, torch.float32, "colsum")
    _check(bias_folded, torch.float32, "bias_folded")
    _check(row_stats, torch.float32, "row_stats")
    m, k = x.shape
    n = w_folded.shape[0]
    if w_folded.shape[1] != k:
        raise ValueError(f"inner dimensions differ: x {tuple(x.shape)}, w_folded {tuple(w_folded.shape)}")
    if row_stats.numel() < m * k // 8:
        raise ValueError(f"row_stats holds {row_stats.numel()} floats, {m * k // 8} needed")
    if out is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=x.device)
    _check(out, torch.bfloat16, "out")
    seqs = heads = head = capacity = 0
    if k_cache is not None:
        seqs, heads, capacity, head = k_cache.shape
    _launch("tempo_gemm_ln_rowstats", x.data_ptr(), k, w_folded.data_ptr(), k, colsum.data_ptr(),
            bias_folded.data_ptr(), float(epsilon), row_stats.data_ptr(), out.data_ptr(), out.shape[1], m, n, k,
            _lib.GEMM_GELU if gelu else 0, _ptr(k_cache), _ptr(v_cache), seqs, heads, head, capacity,
            _ptr(positions), _stream())
    return out


def row_stats(x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """The statistics partials of x's rows ([M, K / 16, 2] FP32 into `out`), as gemm_rowstats writes them."""
    _check(x, torch.bfloat16, "x")
    _check(out, torch.float32, "out")
    m, k = x.shape
    if out.numel() < m * k // 8:
        raise ValueError(f"out holds {out.numel()} floats, {m * k // 8} needed")
    _launch("tempo_row_stats", x.data_ptr(), x.stride(0), m, k, out.data_ptr(), _stream())
    return out


def gemm_norm(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, w_t: torch.Tensor, *, epsilon: float = 1e-5,
              bias: torch.Tensor | None = None, gelu: bool = False, out: torch.Tensor | None = None,
              k_cache: torch.Tensor | None = None, v_cache: torch.Tensor | None = None,
              positions: torch.Tensor | None = None, part_val: torch.Tensor | None = None,
              part_idx: torch.Tensor | None = None) -> torch.Tensor | None:
    """LayerNorm(x) then the projection, one launch for at most 8 rows: the bits of layernorm() followed by gemm()
    (gemm_qkv with the caches and positions; gemm_argmax with the partial buffers, returning None)."""
    _check(x, torch.bfloat16, "x")
    _check(w_t, torch.bfloat16, "w_t")
    m, k = x.shape
    n = w_t.shape[0]
    if w_t.shape[1] != k:
        raise ValueError(f"inner dimensions differ: x {tuple(x.shape)}, w_t {tuple(w_t.shape)}")
    argmax = part_val is not None
    if not argmax and out is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=x.device)
    heads = head = capacity = 0
    if k_cache is not None:
        _, heads, capacity, head = k_cache.shape
    flags = _lib.GEMM_ARGMAX if argmax else (_lib.GEMM_GELU if gelu else 0)
    _launch("tempo_gemm_norm", x.data_ptr(), x.stride(0), gamma.data_ptr(), beta.data_ptr(), float(epsilon),
            w_t.data_ptr(), w_t.stride(0), _ptr(bias), _ptr(out), out.stride(0) if out is not None else n, m, n, k,
            flags, _ptr(part_val), _ptr(part_idx), _ptr(k_cache), _ptr(v_cache), heads, head, capacity,
            _ptr(positions), _stream())
    return None if argmax else out


def gemm_argmax(a: torch.Tensor, w_t: torch.Tensor, part_val: torch.Tensor, part_idx: torch.Tensor) -> None:
    """Per-row (max, first argmax) of a @ w_t^T over each 256-column tile into the partial buffers [M, ceil(N/256)]."""
    _check(a, torch.bfloat16, "a")
    _check(w_t, torch.bfloat16, "w_t")
    m, k = a.shape
    n = w_t.shape[0]
    _launch("tempo_gemm", a.data_ptr(), k, w_t.data_ptr(), k, None, None, n, None, n, m, n, k, _lib.GEMM_ARGMAX,
              part_val.data_ptr(), part_idx.data_ptr(), _stream())


def decode_step_workspace_bytes(rows: int, width: int, heads: int, vocab: int) -> int:
    size = ctypes.c_uint64()
    _lib.call("tempo_decode_step_workspace", rows, width, heads, vocab, ctypes.byref(size))
    return int(size.value)


def decode_step(args: "_lib.DecodeStepArgs") -> None:
    """One persistent decode step (tempo_decode_step) with prepared arguments, on the current stream."""
    _launch("tempo_decode_step", ctypes.byref(args), _stream())


def argmax_finish(part_val: torch.Tensor, part_idx: torch.Tensor, ids: torch.Tensor, *,
                  tokens_out: torch.Tensor | None = None, positions: torch.Tensor | None = None,
                  index_offset: int = 0, advance: int = 0) -> None:
    """ids = per-row argmax; tokens_out[r, positions[r] + index_offset] = ids[r]; positions += advance."""
    rows, tiles = part_val.shape
    stride = tokens_out.shape[1] if tokens_out is not None else 0
    _launch("tempo_argmax_finish", part_val.data_ptr(), part_idx.data_ptr(), rows, tiles, ids.data_ptr(),
              _ptr(tokens_out), stride, _ptr(positions), index_offset, advance, _stream())


def layernorm(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, *, epsilon: float = 1e-5,
              out: torch.Tensor | None = None, rows: int | None = None, row_stride: int | None = None) -> torch.Tensor:
    """LayerNorm of `rows` rows of x read `row_stride` elements apart (default: every row of a contiguous x)."""
    if not x.is_cuda or x.dtype != torch.bfloat16:
        raise ValueError("x must be a CUDA bfloat16 tensor")
    features = x.shape[-1]
    rows = x.numel() // features if rows is None else rows
    row_stride = features if row_stride is None else row_stride
    if out is None:
        out = torch.empty((rows, features), dtype=torch.bfloat16, device=x.device)
    _launch("tempo_layernorm", x.data_ptr(), row_stride, gamma.data_ptr(), beta.data_ptr(), out.data_ptr(), rows,
              features, float(epsilon), _stream())
    return out


def embed(ids: torch.Tensor, positions: torch.Tensor, wte: torch.Tensor, wpe: torch.Tensor, *,
          out: torch.Tensor | None = None) -> torch.Tensor:
    _check(ids, torch.int32, "ids")
    _check(positions, torch.int32, "positions")
    rows, width = ids.numel(), wte.shape[1]
    if out is None:
        out = torch.empty((rows, width), dtype=torch.bfloat16, device=wte.device)
    _launch("tempo_embed", ids.data_ptr(), positions.data_ptr(), wte.data_ptr(), wpe.data_ptr(), out.data_ptr(), rows,
              width, wte.shape[0], wpe.shape[0], _stream())
    return out


def attention_prefill(qkv: torch.Tensor, seqs: int, tokens: int, heads: int, *,
                      out: torch.Tensor | None = None) -> torch.Tensor:
    _check(qkv, torch.bfloat16, "qkv")
    width = qkv.shape[1] // 3
    if out is None:
        out = torch.empty((seqs * tokens, width), dtype=torch.bfloat16, device=qkv.device)
    _launch("tempo_attention_prefill", qkv.data_ptr(), out.data_ptr(), seqs, tokens, heads, width // heads, _stream())
    return out


def kv_store(qkv: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, seq_of: torch.Tensor,
             pos_of: torch.Tensor) -> None:
    seqs, heads, capacity, head = k_cache.shape
    _launch("tempo_kv_store", qkv.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), seq_of.data_ptr(),
              pos_of.data_ptr(), seq_of.numel(), seqs, heads, head, capacity, _stream())


def decode_attention(qkv: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, lengths: torch.Tensor, *,
                     length_offset: int = 0, out: torch.Tensor | None = None) -> torch.Tensor:
    seqs, heads, capacity, head = k_cache.shape
    if out is None:
        out = torch.empty((seqs, heads * head), dtype=torch.bfloat16, device=qkv.device)
    _launch("tempo_decode_attention", qkv.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), lengths.data_ptr(),
              length_offset, out.data_ptr(), seqs, heads, head, capacity, _stream())
    return out


# ---- the packed per-block ops on raw device tensors (uint16 words) ----

def block_gemm(activations: torch.Tensor, weights: torch.Tensor, drain: torch.Tensor, bias: torch.Tensor | None,
               depth: int, columns: int, activate: bool) -> None:
    _launch("tempo_block_gemm", activations.data_ptr(), weights.data_ptr(), drain.data_ptr(), _ptr(bias), depth,
              columns, int(activate), _stream())


def block_add(left: torch.Tensor, right: torch.Tensor, out: torch.Tensor, features: int, broadcast: bool) -> None:
    _launch("tempo_block_add", left.data_ptr(), right.data_ptr(), out.data_ptr(), features, int(broadcast), _stream())


def block_layernorm(rows: torch.Tensor, constants: torch.Tensor, out: torch.Tensor, features: int) -> None:
    _launch("tempo_block_layernorm", rows.data_ptr(), constants.data_ptr(), out.data_ptr(), features, _stream())


def block_attention(constants: torch.Tensor, fused_operand: int, tokens: int, heads: int) -> None:
    _launch("tempo_block_attention", constants.data_ptr(), fused_operand, tokens, heads, 64, _stream())


def block_decode_attention(constants: torch.Tensor, cache_operand: int, fused_operand: int, keys: int, heads: int,
                           stated: int = 0) -> None:
    _launch("tempo_block_decode_attention", constants.data_ptr(), cache_operand, fused_operand, keys, heads, 64,
              stated, _stream())


def block_copy(source: int, destination: int, rows: int, stride: int) -> None:
    _launch("tempo_block_copy", source, destination, rows, stride, _stream())


def watchdog() -> int:
    """Reads and clears the kernels' bounded-wait watchdog (0 = no wait expired)."""
    import ctypes
    code = ctypes.c_int32()
    _lib.call("tempo_watchdog", ctypes.byref(code))
    return int(code.value)


def stream_read(src: torch.Tensor, sink: torch.Tensor | None = None) -> torch.Tensor:
    """Calibration: streams `src` (a contiguous device tensor) once through the HBM read path; returns the sink the
    kernel folds it into. Its rate is the read ceiling of the bandwidth-bound kernels."""
    if not src.is_contiguous():
        raise ValueError("stream_read needs a contiguous source")
    threads = ctypes.c_uint32()
    _lib.call("tempo_stream_read_threads", ctypes.byref(threads))
    if sink is None:
        sink = torch.empty(threads.value * 16, dtype=torch.uint8, device=src.device)
    elif sink.numel() * sink.element_size() < threads.value * 16:
        raise ValueError("stream_read sink too small")
    _launch("tempo_stream_read", src.data_ptr(), src.numel() * src.element_size(), sink.data_ptr(), _stream())
    return sink

