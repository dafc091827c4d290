#!/usr/bin/env python3
"""GPT-2 small batched prefill + greedy-decode throughput on B200, one process per GPU.

Workload (the batched throughput configuration): 512 independent sequences, each a 1024-token prefill followed by
128 greedy decode steps, seeded uniform token ids and random-init weights ~N(0, 0.02). Sequences are sharded
contiguously over the ranks (strong scaling: the job is fixed, each rank takes 512/N sequences); no collective is on
the data path, the process group only times (barrier, max over ranks). One step = the whole job once.

    python bench.py [--gpus N --steps K --warmup W]                      # the B200 arm
    python bench.py --impl reference [--steps K --warmup W]              # the reference's CPU path (oracle port)

Prints one JSON line on rank 0.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

METRIC = "GPT-2-small prefill+decode tok/s at 1/2/4/8 B200; GEMM % of bf16 TC peak"
ROOT = os.path.dirname(os.path.abspath(__file__))
PEAKS_FILE = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def parse() -> argparse.Namespace:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=3)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["b200", "reference"], default="b200")
    p.add_argument("--sequences", type=int, default=512)
    p.add_argument("--prompt", type=int, default=1024)
    p.add_argument("--decode", type=int, default=128)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--cpu-prompt", type=int, default=None,
                   help="prompt of the bounded CPU sample (default: the workload's prompt)")
    p.add_argument("--cpu-decode", type=int, default=8, help="decode steps timed per CPU sample")
    p.add_argument("--cpu-literal-steps", type=int, default=1,
                   help="decode steps also timed the reference's literal way (the whole sequence recomputed)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-graph", action="store_true", help="eager decode instead of the captured CUDA graph")
    p.add_argument("--fold-layernorms", choices=["auto", "on", "off"], default="auto",
                   help="decode with the LayerNorms folded into the projections (default: the engine's choice)")
    p.add_argument("--fuse-small-norms", choices=["auto", "on", "off"], default="auto",
                   help="decode groups of at most 8 sequences normalise inside their projections (default: the "
                        "engine's choice)")
    p.add_argument("--persistent-decode", choices=["auto", "on", "off"], default="auto",
                   help="decode steps of at most 8 sequences as one persistent kernel (default: the engine's choice)")
    p.add_argument("--decode-groups", type=int, default=None,
                   help="independent sequence groups per decode step, one CUDA stream each (default: the engine's)")
    return p.parse_args()


def peaks() -> tuple[dict, str]:
    try:
        with open(PEAKS_FILE) as f:
            return json.load(f), "measured"
    except OSError:
        return dict(FALLBACK_PEAKS), "fallback"


def workload(args) -> dict:
    return {"workload": (f"batched GPT-2 small: {args.sequences} sequences x ({args.prompt}-token prefill + "
                         f"{args.decode} greedy decode steps)"),
            "sequences": args.sequences, "prompt_tokens": args.prompt, "decode_steps": args.decode,
            "parallelism": f"sequences sharded over {args.gpus} GPU(s), no collective on the data path",
            "l2": "inputs larger than L2 (170 MB weights + the KV cache, 21.7 GB at 512 sequences)",
            "positions": max(1024, args.prompt + args.decode),
            "positions_note": ("GPT-2 small learns 1024 positions; sequences of prompt + decode tokens past that use "
                               "a longer learned table, drawn like the other weights")}


# ---------------------------------------------------------------------------------------------------------------
# CPU side: the reference's own host path (the oracle's restatement of board_package/references.py)
# ---------------------------------------------------------------------------------------------------------------

def blas_threads() -> int:
    try:
        from threadpoolctl import threadpool_info
        counts = [info.get("num_threads", 1) for info in threadpool_info() if info.get("user_api") == "blas"]
        return max(counts) if counts else 1
    except Exception:  # noqa: BLE001
        return 1


def all_host_threads() -> None:
    """Lets the BLAS pool use every core this process may run on (torchrun starts each rank with
    OMP_NUM_THREADS=1; the reference arm runs on rank 0 alone)."""
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(limits=len(os.sched_getaffinity(0)), user_api="blas")
    except Exception:  # noqa: BLE001
        pass


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def model(args):
    """The workload's random-init GPT-2 small. Its sequences reach prompt + decode positions; past GPT-2's 1024
    learned positions the table grows, drawn like the rest (its first 1024 rows are the 1024-row table's)."""
    from tempo_compiler_b200.weights import GPT2Shape, random_gpt2
    return random_gpt2(args.seed, GPT2Shape(positions=max(1024, args.prompt + args.decode)))


class CpuSample:
    """The reference's host path on one sequence of the workload's shape, on this machine's cores.

    The reference's host references (board_package/references.py, restated by the oracle in device mode: BF16
    accumulation, table GELU) run the prompt once; decode steps then run through the KV-cached restatement of the
    same references (oracle.model.CachedChain), each sample from a copy of the post-prefill state, so every sample
    decodes the positions right after the prompt. A sequence's time is extrapolated: the prefill plus `decode`
    times the mean step. The reference's own decode check recomputes the whole sequence for each token
    (board_package/board_checks.py:467-474); `literal_steps` such steps are timed beside it."""

    def __init__(self, args, layers, shared) -> None:
        import copy
        from oracle.model import CachedChain, forward_logits
        from tempo_compiler_b200.weights import random_token_ids
        self.args = args
        self.prompt = args.prompt if args.cpu_prompt is None else args.cpu_prompt
        self.ids = [int(t) for t in random_token_ids(args.seed + 1000, self.prompt)]
        chain = CachedChain(layers, shared, mode="device")
        started = time.perf_counter()
        logits = chain.prefill(self.ids)
        self.prefill_s = time.perf_counter() - started
        self.first = int(np.argmax(logits))
        self.state = chain
        self._copy = copy.deepcopy
        self.step_seconds: list[float] = []
        self.literal_s = None
        if args.cpu_literal_steps > 0:
            started = time.perf_counter()
            for k in range(args.cpu_literal_steps):
                forward_logits(self.ids + [self.first] * (k + 1), layers, shared, mode="device")
            self.literal_s = (time.perf_counter() - started) / args.cpu_literal_steps

    def decode_sample(self) -> float:
        """Times `cpu_decode` greedy steps after the prompt; returns their seconds."""
        chain = self._copy(self.state)
        token = self.first
        started = time.perf_counter()
        for _ in range(self.args.cpu_decode):
            token = int(np.argmax(chain.step(token)))
        seconds = time.perf_counter() - started
        self.step_seconds.append(seconds / max(1, self.args.cpu_decode))
        return seconds

    def per_sequence_s(self) -> float:
        mean_step = sum(self.step_seconds) / len(self.step_seconds) if self.step_seconds else 0.0
        return self.prefill_s + self.args.decode * mean_step

    def value(self) -> float:
        return (self.prompt + self.args.decode) / self.per_sequence_s()

    def record(self) -> dict:
        mean_step = sum(self.step_seconds) / len(self.step_seconds) if self.step_seconds else 0.0
        threads = blas_threads()
        out = {"value": self.value(), "unit": "tok/s", "cores": threads, "kind": "port",
               "host_cpus": os.cpu_count(), "cpu_model": cpu_model(), "blas_threads": threads,
               "prefill_s": self.prefill_s, "decode_step_s": mean_step,
               "sample": (f"KV-cached restatement (extrapolated per sequence): 1 sequence of the workload's shape, a "
                          f"{self.prompt}-token prefill timed once ({self.prefill_s:.1f} s) plus {self.args.decode} "
                          f"decode steps extrapolated from {len(self.step_seconds)} x {self.args.cpu_decode} timed "
                          f"steps (mean {mean_step * 1000:.0f} ms, positions {self.prompt}-"
                          f"{self.prompt + self.args.cpu_decode - 1}); the reference's host references "
                          f"(board_package/references.py semantics: BF16 accumulation, table GELU) restated in numpy")}
        if self.literal_s is not None:
            out["literal_full_recompute_s_per_token"] = self.literal_s
            out["literal_full_recompute_tok_s"] = 1.0 / self.literal_s
            out["sample"] += (f"; the reference's literal decode (whole sequence recomputed per token, "
                              f"board_checks.py:467-474) measured at {self.literal_s:.1f} s per token at "
                              f"{self.prompt + 1} tokens")
        return out


def reference_arm(args) -> int:
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    all_host_threads()
    layers, shared = model(args)
    sample = CpuSample(args, layers, shared)
    for _ in range(args.warmup):
        sample.decode_sample()
    sample.step_seconds.clear()
    seconds = sum(sample.decode_sample() for _ in range(args.steps))
    record = sample.record()
    value = record["value"]
    line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 * seconds / max(1, args.steps), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16 storage, float64/BF16-rounded arithmetic",
            "data": "synthetic (seeded uniform token ids, random-init weights ~N(0,0.02))", "config": workload(args),
            "impl": "reference", "cpu_baseline": record,
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------------------------------------------
# Clock sampling during the timed region
# ---------------------------------------------------------------------------------------------------------------

class Clocks:
    """nvidia-smi sampling of the job's GPUs every 100 ms. Each sample carries nvidia-smi's own timestamp, so only the
    samples taken inside the timed region count, whatever the pipe's buffering."""
    QUERY = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, indices: list[int]) -> None:
        self.indices = indices
        self.proc = None
        self.lines: list[str] = []
        self.thread = None
        self.t_start = self.t_end = 0.0

    def start(self) -> "Clocks":
        """Starts the sampler and waits (up to 10 s) for its first sample, so the timed region is covered."""
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", ",".join(str(i) for i in self.indices)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
            return self
        deadline = time.time() + 10.0
        while not self.lines and time.time() < deadline and self.proc.poll() is None:
            time.sleep(0.02)
        return self

    def _read(self) -> None:
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def mark_start(self) -> None:
        self.t_start = time.time()

    def mark_end(self) -> None:
        self.t_end = time.time()

    @staticmethod
    def _stamp(text: str) -> float | None:
        try:
            return datetime.datetime.strptime(text, "%Y/%m/%d %H:%M:%S.%f").timestamp()
        except ValueError:
            return None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        time.sleep(0.25)  # the sample that closes the region
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=2)
        return self.summarize(self.lines, self.t_start, self.t_end, len(self.indices))

    @classmethod
    def summarize(cls, lines: list[str], t_start: float, t_end: float, gpus: int) -> dict | None:
        """Median SM clock, maximum clock and the throttle reasons of the samples stamped inside [t_start, t_end]
        (50 ms of slack either side); with none inside (a region shorter than the interval), the first sample of
        each GPU after t_start."""
        rows = []
        for line in lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            stamp = cls._stamp(parts[0])
            try:
                rows.append((stamp, float(parts[2]), float(parts[3]), parts[6:10]))
            except ValueError:
                continue
        inside = [r for r in rows if r[0] is not None and t_start - 0.05 <= r[0] <= t_end + 0.05]
        used = inside or [r for r in rows if r[0] is not None and r[0] >= t_start][:gpus]
        if not used:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = {name for r in used for name, value in zip(names, r[3]) if value.lower() == "active"}
        return {"sm_mhz": statistics.median(r[1] for r in used), "sm_max_mhz": max(r[2] for r in used),
                "reasons": sorted(reasons), "samples": len(used), "gpus": gpus, "in_timed_region": bool(inside)}


def _job_gpu_indices(world: int) -> list[int]:
    """nvidia-smi indices of local ranks 0 .. world - 1 (one rank per GPU on one node)."""
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    if visible:
        ids = [v.strip() for v in visible.split(",") if v.strip()]
        if all(v.isdigit() for v in ids) and len(ids) >= world:
            return [int(v) for v in ids[:world]]
    return list(range(world))


# ---------------------------------------------------------------------------------------------------------------
# The B200 arm
# ---------------------------------------------------------------------------------------------------------------

def b200_arm(args) -> int:
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        args.gpus = world
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=device)

    def barrier():
        if world > 1:
            dist.barrier()

    from tempo_compiler_b200 import lib, ops
    from tempo_compiler_b200.engine import Engine
    from tempo_compiler_b200.sharding import gather_tokens, shard
    from tempo_compiler_b200.sharding import max_over_ranks as _max_over_ranks
    from tempo_compiler_b200.weights import random_token_ids

    def max_over_ranks(value: float) -> float:
        return _max_over_ranks(value, device)

    lib.load()
    layers, shared = model(args)
    first, per_rank = shard(args.sequences, world, rank)
    if per_rank == 0:
        raise SystemExit(f"{args.sequences} sequences leave rank {rank} of {world} without work")
    ids = np.stack([random_token_ids(args.seed + 1000 + s, args.prompt) for s in range(first, first + per_rank)])
    ids = ids.astype(np.int32)
    engine = Engine(layers, shared, batch=per_rank, prompt=args.prompt, capacity=args.prompt + args.decode,
                    device=device, decode_groups=args.decode_groups,
                    fold_layernorms=None if args.fold_layernorms == "auto" else args.fold_layernorms == "on",
                    fuse_small_norms=None if args.fuse_small_norms == "auto" else args.fuse_small_norms == "on",
                    persistent_decode=None if args.persistent_decode == "auto" else args.persistent_decode == "on")
    ids_dev = torch.from_numpy(ids).to(device)
    graph = not args.no_graph

    # launch count of one step, from an eager run (the graph replays the same kernels)
    ops.reset_launch_count()
    engine.run(ids_dev, args.decode, graph=False)
    torch.cuda.synchronize()
    launches_per_step = ops.launch_count()

    for _ in range(args.warmup):
        engine.run(ids_dev, args.decode, graph=graph)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()

    stream = torch.cuda.current_stream(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = Clocks(_job_gpu_indices(world)).start() if rank == 0 else None
    barrier()
    torch.cuda.synchronize()
    if clocks is not None:
        clocks.mark_start()
    start.record(stream)
    for _ in range(args.steps):
        engine.run(ids_dev, args.decode, graph=graph)
    end.record(stream)
    torch.cuda.synchronize()
    if clocks is not None:
        clocks.mark_end()
    timed_tokens = engine.tokens.cpu().numpy().copy()
    barrier()
    clock_info = clocks.stop() if clocks is not None else None
    ms = max_over_ranks(start.elapsed_time(end))
    tokens_per_step = args.sequences * (args.prompt + args.decode)
    value = tokens_per_step * args.steps / (ms / 1000.0)

    # end to end through the public call: host prompts in (pinned), host tokens out. One untimed call first: the
    # engine allocates its pinned staging buffers on the first call and keeps them.
    engine.generate(ids, args.decode, graph=graph)
    e2e_start, e2e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    e2e_start.record(stream)
    first_tokens = None
    for _ in range(args.steps):
        tokens = engine.generate(ids, args.decode, graph=graph)
        if first_tokens is None:
            first_tokens = tokens.copy()
    e2e_end.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e2e_start.elapsed_time(e2e_end))
    e2e_value = tokens_per_step * args.steps / (e2e_ms / 1000.0)
    h2d = args.sequences * args.prompt * 4
    d2h = args.sequences * (args.decode + 1) * 4

    # phase split and per-kernel rooflines, timed with CUDA events on the launching stream
    measured, source = peaks()
    prefill_ms = _time(lambda: engine.prefill(ids_dev, graph=graph), stream, 2)
    decode_ms = _time(lambda: engine.decode(args.decode, graph=graph), stream, 1) if args.decode else 0.0
    roof = _decode_attention_roofline(engine, stream, measured, source)
    gemm_roof = _gemm_roofline(engine, stream, measured, source)
    watchdog = int(max_over_ranks(float(ops.watchdog())))
    # the same job repeated gives the same tokens: the device-timed run, the first and the last end-to-end run
    runs = [gather_tokens(torch.from_numpy(np.ascontiguousarray(t)), args.sequences, device)
            for t in (timed_tokens, first_tokens, tokens)]
    all_tokens = runs[-1]

    line = None
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (seeded uniform token ids, random-init weights ~N(0,0.02))",
                "config": {**workload(args), "decode_groups_per_gpu": len(engine.decode_groups),
                           "layernorms_folded_in_decode": engine.fold_layernorms,
                           "layernorms_inside_small_decode_projections": engine.fuse_small_norms,
                           "persistent_decode_step": engine.persistent_decode},
                "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
                "gpu_launches": launches_per_step * args.steps * world,
                "clocks": clock_info, "roofline": roof, "gemm_roofline": gemm_roof,
                "phases_ms_rank0": {"prefill": prefill_ms, "decode": decode_ms,
                                    "decode_ms_per_step": decode_ms / max(1, args.decode)},
                "decode_graph": graph, "watchdog": watchdog,
                "tokens_checksum": int(all_tokens.to(torch.int64).sum().item()),
                "tokens_checksums_of_repeats": [int(r.to(torch.int64).sum().item()) for r in runs],
                "tokens_repeat_identical": all(bool(torch.equal(r, runs[0])) for r in runs)}
        if world == 1 and not args.no_cpu_baseline:
            sample = CpuSample(args, layers, shared)
            sample.decode_sample()
            line["cpu_baseline"] = sample.record()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)
    return 0


def _time(fn, stream, repeats: int) -> float:
    import torch
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(repeats):
        fn()
    end.record(stream)
    torch.cuda.synchronize()
    return start.elapsed_time(end) / repeats


# DRAM traffic of decode attention per algorithmic byte, from one ncu capture of 64 sequences x 12 heads x 1152 keys:
# 226.6 MB read + 3.5 MB written for 226.9 MB of cached keys, values, queries and outputs.
DECODE_TRAFFIC_PER_BYTE = (226.6e6 + 3.5e6) / 226.885632e6


def _decode_attention_roofline(engine, stream, measured, source) -> dict:
    """Decode attention over the full caches (every sequence at `capacity` keys): algorithmic bytes are each cached
    key and value read once plus the query read and the output written."""
    import torch
    from tempo_compiler_b200 import ops
    layer = len(engine.layers) // 2
    lengths = torch.full((engine.batch,), engine.capacity, dtype=torch.int32, device=engine.device)
    fn = lambda: ops.decode_attention(engine.dqkv, engine.k_cache[layer], engine.v_cache[layer], lengths,  # noqa
                                      out=engine.dattn)
    fn()
    ms = _time(fn, stream, 20)
    heads, head = engine.shape.heads, engine.shape.head
    algorithmic = engine.batch * heads * engine.capacity * head * 2 * 2 + engine.batch * 3 * heads * head * 2 + \
        engine.batch * heads * head * 2
    achieved = algorithmic / (ms / 1000.0) / 1e9
    peak = float(measured["hbm_gbs"])
    # the streaming-read ceiling of this GPU, measured beside it: 2 GiB read once per launch by the calibration kernel
    src = torch.empty(2 << 30, dtype=torch.uint8, device=engine.device)
    sink = ops.stream_read(src)
    read_ms = _time(lambda: ops.stream_read(src, sink), stream, 10)
    read_gbs = (2 << 30) / (read_ms / 1000.0) / 1e9
    del src, sink
    return {"kernel": "decode_attention_kernel", "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
            "frac": achieved / peak, "read_ceiling_gbs": read_gbs, "frac_of_read_ceiling": achieved / read_gbs, "traffic": algorithmic * DECODE_TRAFFIC_PER_BYTE,
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one 64-sequence launch, scaled to "
                              "this launch by its algorithmic bytes (each key and value is read once at any size)",
            "algorithmic_bytes_per_launch": algorithmic,
            "launch_ms": ms, "peak_source": f"{source} ({PEAKS_FILE if source == 'measured' else 'fallback'})"}


def _gemm_roofline(engine, stream, measured, source) -> dict:
    """The prefill FC projection: M = sequences x prompt, N = 3072, K = 768, bias + exact-erf GELU epilogue."""
    import torch
    from tempo_compiler_b200 import ops
    lw = engine.layers[0]
    fn = lambda: ops.gemm(engine.ln, lw.w_fc, bias=lw.b_fc, gelu=True, out=engine.h)  # noqa: E731
    fn()
    ms = _time(fn, stream, 5)
    m, k = engine.ln.shape
    n = lw.w_fc.shape[0]
    achieved = 2.0 * m * n * k / (ms / 1000.0) / 1e12
    peak = float(measured["bf16_tflops"])
    # the library's choice at this size: CTA pairs on 256 x 256 tiles once there are four tiles per pair of SMs
    sms = torch.cuda.get_device_properties(engine.device).multi_processor_count
    pair = -(-m // 256) * -(-n // 256) >= 4 * (sms // 2)
    name = "gemm_pair_kernel" if pair else "gemm_rowmajor_kernel"
    return {"kernel": "%s (prefill FC, M=%d N=%d K=%d)" % (name, m, n, k), "bound": "tensor",
            "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak, "launch_ms": ms,
            "peak_source": f"{source} burst cuBLAS bf16"}


def main() -> int:
    args = parse()
    if args.impl == "reference":
        return reference_arm(args)
    return b200_arm(args)


if __name__ == "__main__":
    sys.exit(main())
