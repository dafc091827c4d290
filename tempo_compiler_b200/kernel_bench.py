"""Per-kernel microbenchmarks: one kernel of the library on synthetic inputs of a chosen size, timed with CUDA events.

It allocates only that kernel's operands, so a profiler capture of it stays small:

    python -m tempo_compiler_b200.kernel_bench gemm --m 65536 --n 3072 --k 768 --epilogue gelu
    python -m tempo_compiler_b200.kernel_bench decode_attention --seqs 64 --capacity 1152
    python -m tempo_compiler_b200.kernel_bench prefill_attention --seqs 8 --tokens 1024
    python -m tempo_compiler_b200.kernel_bench layernorm --rows 65536
    python -m tempo_compiler_b200.kernel_bench block_gemm --depth 768 --columns 3072
    python -m tempo_compiler_b200.kernel_bench stream_read --gib 2

Prints one JSON line: the launch time and the achieved rate against the algorithmic work.
"""

from __future__ import annotations

import argparse
import json

import torch

from tempo_compiler_b200 import lib, ops


def _time(fn, repeats: int, warmup: int) -> float:
    """Mean device time of one call: the `repeats` calls are captured into one CUDA graph and replayed, so host launch
    cost (which exceeds the run time of the small decode kernels) does not enter the measurement."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(repeats):
            fn()
    graph.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    graph.replay()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / repeats


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("kernel", choices=["gemm", "decode_attention", "prefill_attention", "layernorm", "block_gemm",
                                           "stream_read"])
    parser.add_argument("--gib", type=float, default=2.0, help="stream_read: GiB read per launch")
    parser.add_argument("--m", type=int, default=65536)
    parser.add_argument("--n", type=int, default=3072)
    parser.add_argument("--k", type=int, default=768)
    parser.add_argument("--epilogue", choices=["plain", "bias", "gelu", "residual", "ln", "ln_gelu"], default="gelu",
                        help="ln / ln_gelu: the LayerNorm folded in on row statistics partials (gemm_ln_rowstats)")
    parser.add_argument("--seqs", type=int, default=64)
    parser.add_argument("--capacity", type=int, default=1152)
    parser.add_argument("--length", type=int, default=None, help="decode: cached keys per sequence (default capacity)")
    parser.add_argument("--tokens", type=int, default=1024)
    parser.add_argument("--rows", type=int, default=65536)
    parser.add_argument("--depth", type=int, default=768)
    parser.add_argument("--columns", type=int, default=3072)
    parser.add_argument("--repeats", type=int, default=10)
    parser.add_argument("--warmup", type=int, default=3)
    args = parser.parse_args()
    lib.load()
    torch.manual_seed(0)
    dev = "cuda"
    bf = torch.bfloat16
    result: dict = {"kernel": args.kernel}

    if args.kernel == "gemm" and args.epilogue.startswith("ln"):
        from tempo_compiler_b200.engine import fold_layernorm
        x = torch.randn((args.m, args.k), device=dev).to(bf)
        w = (torch.randn((args.n, args.k), device=dev) * 0.05).to(bf)
        gamma = torch.ones(args.k, device=dev, dtype=bf)
        beta = torch.zeros(args.k, device=dev, dtype=bf)
        folded, colsum, bias_folded = fold_layernorm(gamma, beta, w, None)
        stats = torch.empty((args.m, args.k // 16, 2), dtype=torch.float32, device=dev)
        ops.row_stats(x, stats)
        out = torch.empty((args.m, args.n), device=dev, dtype=bf)
        ms = _time(lambda: ops.gemm_ln_rowstats(x, folded, colsum, bias_folded, stats, gelu=args.epilogue == "ln_gelu",
                                                out=out), args.repeats, args.warmup)
        flops = 2.0 * args.m * args.n * args.k
        result.update(m=args.m, n=args.n, k=args.k, epilogue=args.epilogue, ms=ms, tflops=flops / ms / 1e9)
    elif args.kernel == "gemm":
        a = torch.randn((args.m, args.k), device=dev).to(bf)
        w = (torch.randn((args.n, args.k), device=dev) * 0.05).to(bf)
        bias = (torch.randn(args.n, device=dev) * 0.1).to(bf) if args.epilogue != "plain" else None
        residual = torch.randn((args.m, args.n), device=dev).to(bf) if args.epilogue == "residual" else None
        out = torch.empty((args.m, args.n), device=dev, dtype=bf)
        ms = _time(lambda: ops.gemm(a, w, bias=bias, residual=residual, gelu=args.epilogue == "gelu", out=out),
                   args.repeats, args.warmup)
        flops = 2.0 * args.m * args.n * args.k
        result.update(m=args.m, n=args.n, k=args.k, epilogue=args.epilogue, ms=ms, tflops=flops / ms / 1e9)
    elif args.kernel == "decode_attention":
        qkv = torch.randn((args.seqs, 3 * 768), device=dev).to(bf)
        kc = torch.randn((args.seqs, 12, args.capacity, 64), device=dev).to(bf)
        vc = torch.randn_like(kc)
        length = args.capacity if args.length is None else args.length
        lengths = torch.full((args.seqs,), length, dtype=torch.int32, device=dev)
        out = torch.empty((args.seqs, 768), device=dev, dtype=bf)
        ms = _time(lambda: ops.decode_attention(qkv, kc, vc, lengths, out=out), args.repeats, args.warmup)
        nbytes = args.seqs * 12 * length * 64 * 2 * 2 + args.seqs * 3 * 768 * 2 + args.seqs * 768 * 2
        result.update(seqs=args.seqs, capacity=args.capacity, length=length, ms=ms,
                      bytes=nbytes, gbs=nbytes / ms / 1e6)
    elif args.kernel == "prefill_attention":
        rows = args.seqs * args.tokens
        qkv = torch.randn((rows, 3 * 768), device=dev).to(bf)
        out = torch.empty((rows, 768), device=dev, dtype=bf)
        ms = _time(lambda: ops.attention_prefill(qkv, args.seqs, args.tokens, 12, out=out), args.repeats, args.warmup)
        flops = args.seqs * 12 * 4.0 * 64 * args.tokens * (args.tokens + 1) / 2
        result.update(seqs=args.seqs, tokens=args.tokens, ms=ms, tflops=flops / ms / 1e9)
    elif args.kernel == "layernorm":
        x = torch.randn((args.rows, 768), device=dev).to(bf)
        g = torch.ones(768, device=dev, dtype=bf)
        b = torch.zeros(768, device=dev, dtype=bf)
        out = torch.empty_like(x)
        ms = _time(lambda: ops.layernorm(x, g, b, out=out), args.repeats, args.warmup)
        nbytes = 2 * args.rows * 768 * 2
        result.update(rows=args.rows, ms=ms, bytes=nbytes, gbs=nbytes / ms / 1e6)
    elif args.kernel == "stream_read":
        nbytes = int(args.gib * (1 << 30)) // 16 * 16
        src = torch.empty(nbytes, dtype=torch.uint8, device=dev).random_(0, 255)
        sink = ops.stream_read(src)
        ms = _time(lambda: ops.stream_read(src, sink), args.repeats, args.warmup)
        result.update(bytes=nbytes, ms=ms, gbs=nbytes / ms / 1e6)
    else:
        acts = torch.randint(-2000, 2000, (args.depth * 32,), dtype=torch.int16, device=dev)
        weights = torch.randint(-2000, 2000, (args.depth * args.columns,), dtype=torch.int16, device=dev)
        bias = torch.zeros(args.columns * 4, dtype=torch.int16, device=dev)
        drain = torch.zeros(256 + args.columns * 32, dtype=torch.int16, device=dev)
        ms = _time(lambda: ops.block_gemm(acts, weights, drain, bias, args.depth, args.columns, False), args.repeats,
                   args.warmup)
        nbytes = 2 * (32 * args.depth + args.depth * args.columns + 32 * args.columns) + 8 * args.columns
        result.update(depth=args.depth, columns=args.columns, ms=ms, bytes=nbytes, gbs=nbytes / ms / 1e6)
    result["watchdog"] = ops.watchdog()
    print(json.dumps(result), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
