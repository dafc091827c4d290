"""The B200-native GPT-2 engine: resident weights, batched prefill and greedy decode, one CUDA graph per decode step.

The op order is the reference's layer (``_run_layer``, board_package/gpt2_inference.py:1133-1189) and the model chain
its ``generate`` runs (:941-978): embed -> 12 x [LN1, QKV + bias, causal attention, proj + bias + residual, LN2,
FC + bias + GELU, proj + bias + residual] -> final LN on the last token -> tied LM head -> greedy argmax. What changes
is the B200 layout of the same math:

* weights are uploaded once, transposed to [out, in] (K-major for the tensor cores), with the 1/sqrt(head) query
  scale folded into the QKV weights and bias as the reference does (:1153-1168);
* activations are row-major [tokens, features] for the whole batch, so each projection is one GEMM over every
  token of every sequence (M = sequences x tokens) instead of one launch per 32-token block;
* the bias, the exact-erf GELU (applied to the FC output, which the reference applies while staging the next GEMM's
  input) and the residual add are fused into the GEMM epilogue, so the add images vanish;
* keys and values are stored once per token into a [seq][head][position][64] cache, which decode attention streams;
* the LM head's argmax is fused into its GEMM epilogue, so the 50257-wide logits never reach HBM;
* with at most 8 sequences per decode group each LayerNorm runs inside the projection after it (``gemm_norm``, the
  same bits as the separate kernels), two launches fewer per layer;
* the decode step (embedding, 12 layers, LM head, argmax, position advance) is captured once as a CUDA graph and
  replayed, its varying state (ids, positions) living in device buffers.

Every kernel is libtempo_b200.so's (through ``tempo_compiler_b200.ops``); torch only provides memory and streams.
Sequences in one batch share one prompt length.
"""

from __future__ import annotations

import dataclasses
import math
from dataclasses import dataclass

import numpy as np
import torch

from tempo_compiler_b200 import ops
from tempo_compiler_b200.weights import GPT2_SMALL, GPT2Shape

LN_EPSILON = 1e-5


def _bf16(array: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(array, dtype=np.float32)).to(device).to(torch.bfloat16)


def fold_layernorm(gamma: torch.Tensor, beta: torch.Tensor, w_t: torch.Tensor, bias: torch.Tensor | None
                   ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """The operands of gemm_ln for LayerNorm(gamma, beta) followed by x @ W + bias (w_t = W^T, [N, K] BF16): the folded
    BF16 weights (gamma scaling W's rows), their FP32 column sums and the FP32 folded bias b + beta @ W. Computed once
    per weight set, in float64 on the device (weight preparation, not the decode path)."""
    w64 = w_t.double()
    folded = (w64 * gamma.double()[None, :]).to(torch.bfloat16).contiguous()
    colsum = folded.double().sum(dim=1).float().contiguous()
    b = w64 @ beta.double()
    if bias is not None:
        b = b + bias.double()
    return folded, colsum, b.float().contiguous()


@dataclass
class LayerWeights:
    ln1_g: torch.Tensor
    ln1_b: torch.Tensor
    w_qkv: torch.Tensor   # [3W, W], query rows scaled by 1/sqrt(head)
    b_qkv: torch.Tensor
    w_proj: torch.Tensor  # [W, W]
    b_proj: torch.Tensor
    ln2_g: torch.Tensor
    ln2_b: torch.Tensor
    w_fc: torch.Tensor    # [4W, W]
    b_fc: torch.Tensor
    w_out: torch.Tensor   # [W, 4W]
    b_out: torch.Tensor
    # decode with the LayerNorms folded into the QKV and FC projections (fold_layernorm's operands)
    qkv_folded: tuple[torch.Tensor, torch.Tensor, torch.Tensor] | None = None
    fc_folded: tuple[torch.Tensor, torch.Tensor, torch.Tensor] | None = None


class Engine:
    """Batched GPT-2 greedy generation on one GPU.

    Args:
        layers, shared: weights as ``tempo_compiler_b200.weights.random_gpt2`` (or the reference's loader) returns them.
        batch: sequences per batch.
        prompt: tokens per prompt (every sequence of a batch has the same length).
        capacity: cache positions per sequence (prompt + decode steps).
        device: the CUDA device.
        fold_layernorms: decode folds each block's two LayerNorms into the QKV and FC projections
            (``ops.gemm_ln_rowstats``): the out-projection and the second MLP projection also write the statistics
            partials of the rows they store (``ops.gemm_rowstats``) and the projection after each combines them, so
            a layer runs five kernels instead of seven. Needs more than 8 sequences (8 or fewer rows take the
            CUDA-core path, which normalises inside its projections anyway). Default on for more than 8 sequences:
            measured side by side on a B200, 64 sequences 653,000-655,000 tokens/s folded against 632,000-633,000
            (decode step 781-795 us against 827-831), 512 sequences within the run-to-run spread.
        decode_groups: the decode step splits the batch into this many groups of sequences, each on its own CUDA
            stream (default 1). The groups are independent, so one group's bandwidth-bound attention may overlap
            another's projections; on a B200 the extra, smaller launches cost more than the overlap gains (512
            sequences: 453 ms of decode with one group, 483 with two, 519 with four), hence the default.
        fuse_small_norms: decode groups of at most 8 sequences compute each LayerNorm inside the projection that
            follows it (``ops.gemm_norm``, the same bits as the separate kernels): five kernels per layer instead of
            seven, and the final LayerNorm inside the LM head. Default on.
        persistent_decode: a decode step of at most 8 sequences (one group) runs as one persistent kernel
            (``ops.decode_step``: one CTA per SM, grid-wide barriers between the phases) instead of five kernels per
            layer; the tokens are the same bits. Default off: measured on a B200 (128-token prompt, 256 steps), a
            step takes 293 / 341 / 706 us persistent against 279 / 308 / 690 us kernel-per-op at 1 / 2 / 8
            sequences. A grid barrier costs 1.36 us, about what a dependent launch's boundary costs, and the step
            has 61 dependent phases either way.
    """

    def __init__(self, layers: list[dict], shared: dict, *, batch: int, prompt: int, capacity: int,
                 shape: GPT2Shape = GPT2_SMALL, device: str | torch.device = "cuda",
                 decode_groups: int | None = None, fold_layernorms: bool | None = None,
                 fuse_small_norms: bool | None = None, persistent_decode: bool | None = None) -> None:
        if not torch.cuda.is_available():
            raise RuntimeError("the B200 engine needs a CUDA device; there is no CPU path")
        self.device = torch.device(device)
        # the vocabulary and the learned position table are whatever the weights hold
        shape = dataclasses.replace(shape, layers=len(layers), vocab=int(shared["wte"].shape[0]),
                                    positions=int(shared["wpe"].shape[0]))
        self.shape = shape
        self.batch, self.prompt, self.capacity = batch, prompt, capacity
        if not 0 < prompt <= capacity <= shape.positions:
            raise ValueError(f"prompt {prompt} and capacity {capacity} must satisfy 0 < prompt <= capacity <= "
                             f"{shape.positions}, the model's learned positions")
        width, heads = shape.width, shape.heads
        scale = np.ones(3 * width, dtype=np.float32)
        scale[:width] = 1.0 / math.sqrt(width // heads)
        self.layers: list[LayerWeights] = []
        for w in layers:
            self.layers.append(LayerWeights(
                ln1_g=_bf16(w["ln_1.g"], self.device), ln1_b=_bf16(w["ln_1.b"], self.device),
                w_qkv=_bf16((w["attn.qkv.w"] * scale).T, self.device), b_qkv=_bf16(w["attn.qkv.b"] * scale, self.device),
                w_proj=_bf16(w["attn.proj.w"].T, self.device), b_proj=_bf16(w["attn.proj.b"], self.device),
                ln2_g=_bf16(w["ln_2.g"], self.device), ln2_b=_bf16(w["ln_2.b"], self.device),
                w_fc=_bf16(w["mlp.fc.w"].T, self.device), b_fc=_bf16(w["mlp.fc.b"], self.device),
                w_out=_bf16(w["mlp.proj.w"].T, self.device), b_out=_bf16(w["mlp.proj.b"], self.device)))
        self.wte = _bf16(shared["wte"], self.device)   # also the LM head's [vocab, W] operand
        self.wpe = _bf16(shared["wpe"], self.device)
        self.lnf_g = _bf16(shared["ln_f.g"], self.device)
        self.lnf_b = _bf16(shared["ln_f.b"], self.device)
        self.fold_layernorms = (batch > 8) if fold_layernorms is None else (fold_layernorms and batch > 8)
        # decode groups of at most 8 sequences normalise inside their projections (tempo_gemm_norm: same bits, two
        # launches fewer per layer and one fewer per step)
        self.fuse_small_norms = True if fuse_small_norms is None else fuse_small_norms
        if self.fold_layernorms:
            for lw in self.layers:
                lw.qkv_folded = fold_layernorm(lw.ln1_g, lw.ln1_b, lw.w_qkv, lw.b_qkv)
                lw.fc_folded = fold_layernorm(lw.ln2_g, lw.ln2_b, lw.w_fc, lw.b_fc)
        n_layers = len(layers)
        cache_shape = (batch, heads, capacity, shape.head)
        self.k_cache = [torch.empty(cache_shape, dtype=torch.bfloat16, device=self.device) for _ in range(n_layers)]
        self.v_cache = [torch.empty(cache_shape, dtype=torch.bfloat16, device=self.device) for _ in range(n_layers)]
        rows = batch * prompt
        bf = dict(dtype=torch.bfloat16, device=self.device)
        i32 = dict(dtype=torch.int32, device=self.device)
        # prefill activations (all sequences at once)
        self.x = torch.empty((rows, width), **bf)
        self.ln = torch.empty((rows, width), **bf)
        self.qkv = torch.empty((rows, 3 * width), **bf)
        self.attn = torch.empty((rows, width), **bf)
        self.h = torch.empty((rows, shape.ffn), **bf)
        self.prompt_ids = torch.empty(rows, **i32)
        self.prompt_pos = torch.arange(prompt, **i32).repeat(batch)
        self.prompt_seq = torch.arange(batch, **i32).repeat_interleave(prompt)
        # decode state
        self.dx = torch.empty((batch, width), **bf)
        self.dln = torch.empty((batch, width), **bf)
        self.dqkv = torch.empty((batch, 3 * width), **bf)
        self.dattn = torch.empty((batch, width), **bf)
        self.dh = torch.empty((batch, shape.ffn), **bf)
        # the folded LayerNorms' row statistics partials (mean, M2 of each 16 columns), before attention and before
        # the MLP
        self.dstats1 = torch.empty((batch, width // 16, 2), dtype=torch.float32, device=self.device)
        self.dstats2 = torch.empty((batch, width // 16, 2), dtype=torch.float32, device=self.device)
        self.ids = torch.zeros(batch, **i32)
        self.positions = torch.zeros(batch, **i32)
        self.seq_index = torch.arange(batch, **i32)
        self.tiles = (shape.vocab + 255) // 256
        self.part_val = torch.empty((batch, self.tiles), dtype=torch.float32, device=self.device)
        self.part_idx = torch.empty((batch, self.tiles), **i32)
        self.tokens: torch.Tensor | None = None
        self._graph: torch.cuda.CUDAGraph | None = None
        self._prefill_graph: torch.cuda.CUDAGraph | None = None
        # generate()'s pinned host staging for the prompts and the tokens, kept between calls
        self._pinned_ids: torch.Tensor | None = None
        self._pinned_tokens: torch.Tensor | None = None
        self._graph_steps = 0
        groups = 1 if decode_groups is None else decode_groups
        if not 1 <= groups <= batch:
            raise ValueError(f"decode_groups must be in [1, {batch}], got {groups}")
        bounds = [batch * g // groups for g in range(groups + 1)]
        self.decode_groups = [(bounds[g], bounds[g + 1]) for g in range(groups)]
        self._side_streams = [torch.cuda.Stream(device=self.device) for _ in range(groups - 1)]
        applies = batch <= 8 and groups == 1 and not self.fold_layernorms and len(layers) <= 16
        self.persistent_decode = bool(persistent_decode) and applies
        self._step_args = None
        self._step_layers = None
        if self.persistent_decode:
            size = ops.decode_step_workspace_bytes(batch, width, heads, shape.vocab)
            self._step_workspace = torch.zeros(size, dtype=torch.uint8, device=self.device)

    # ---- prefill ---------------------------------------------------------------------------------------------

    def _layer(self, lw: LayerWeights, index: int, x, ln, qkv, attn, h, *, decode: bool,
               seqs: slice = slice(None)) -> None:
        if decode and self.fold_layernorms:
            self._folded_decode_layer(lw, index, x, qkv, attn, h, seqs)
            return
        if decode and self._fused_norms(x):
            self._normalising_decode_layer(lw, index, x, qkv, attn, h, seqs)
            return
        ops.layernorm(x, lw.ln1_g, lw.ln1_b, epsilon=LN_EPSILON, out=ln)
        # the projection's epilogue also writes this step's keys and values into the layer's cache
        k_cache, v_cache = self.k_cache[index][seqs], self.v_cache[index][seqs]
        if decode:
            positions = self.positions[seqs]
            ops.gemm_qkv(ln, lw.w_qkv, lw.b_qkv, qkv, k_cache, v_cache, positions=positions)
            ops.decode_attention(qkv, k_cache, v_cache, positions, length_offset=1, out=attn)
        else:
            ops.gemm_qkv(ln, lw.w_qkv, lw.b_qkv, qkv, k_cache, v_cache, tokens_per_seq=self.prompt)
            ops.attention_prefill(qkv, self.batch, self.prompt, self.shape.heads, out=attn)
        ops.gemm(attn, lw.w_proj, bias=lw.b_proj, residual=x, out=x)
        ops.layernorm(x, lw.ln2_g, lw.ln2_b, epsilon=LN_EPSILON, out=ln)
        ops.gemm(ln, lw.w_fc, bias=lw.b_fc, gelu=True, out=h)
        ops.gemm(h, lw.w_out, bias=lw.b_out, residual=x, out=x)

    def _fused_norms(self, x) -> bool:
        return self.fuse_small_norms and x.shape[0] <= 8

    def _normalising_decode_layer(self, lw: LayerWeights, index: int, x, qkv, attn, h, seqs: slice) -> None:
        """One decode block of at most 8 sequences, each LayerNorm computed inside the projection after it."""
        k_cache, v_cache = self.k_cache[index][seqs], self.v_cache[index][seqs]
        positions = self.positions[seqs]
        ops.gemm_norm(x, lw.ln1_g, lw.ln1_b, lw.w_qkv, epsilon=LN_EPSILON, bias=lw.b_qkv, out=qkv, k_cache=k_cache,
                      v_cache=v_cache, positions=positions)
        ops.decode_attention(qkv, k_cache, v_cache, positions, length_offset=1, out=attn)
        ops.gemm(attn, lw.w_proj, bias=lw.b_proj, residual=x, out=x)
        ops.gemm_norm(x, lw.ln2_g, lw.ln2_b, lw.w_fc, epsilon=LN_EPSILON, bias=lw.b_fc, gelu=True, out=h)
        ops.gemm(h, lw.w_out, bias=lw.b_out, residual=x, out=x)

    def _folded_decode_layer(self, lw: LayerWeights, index: int, x, qkv, attn, h, seqs: slice) -> None:
        """One decode block with both LayerNorms folded into the projections after them: each residual projection
        also writes the statistics partials of the rows it stores, and the next projection combines them."""
        k_cache, v_cache = self.k_cache[index][seqs], self.v_cache[index][seqs]
        positions = self.positions[seqs]
        stats1, stats2 = self.dstats1[seqs], self.dstats2[seqs]
        w, cs, bf = lw.qkv_folded
        ops.gemm_ln_rowstats(x, w, cs, bf, stats1, epsilon=LN_EPSILON, out=qkv, k_cache=k_cache, v_cache=v_cache,
                             positions=positions)
        ops.decode_attention(qkv, k_cache, v_cache, positions, length_offset=1, out=attn)
        ops.gemm_rowstats(attn, lw.w_proj, stats2, bias=lw.b_proj, residual=x, out=x)
        w, cs, bf = lw.fc_folded
        ops.gemm_ln_rowstats(x, w, cs, bf, stats2, epsilon=LN_EPSILON, gelu=True, out=h)
        ops.gemm_rowstats(h, lw.w_out, stats1, bias=lw.b_out, residual=x, out=x)

    def prefill(self, token_ids: torch.Tensor, *, graph: bool = False) -> None:
        """Runs the prompts ([batch, prompt] int32 on the device) through every layer, filling the caches, and writes
        the first generated token of each sequence into ``self.tokens[:, 0]``. With `graph` the layers run as one
        replay of a CUDA graph captured on first use (the host then issues one launch instead of about a hundred)."""
        self.prompt_ids.copy_(token_ids.reshape(-1))
        self._prefill_loaded(graph)

    def _prefill_loaded(self, graph: bool) -> None:
        """prefill() on the prompts already in ``self.prompt_ids``."""
        if graph:
            self._capture_prefill()
            self._prefill_graph.replay()
        else:
            self._prefill_body()

    def _capture_prefill(self) -> None:
        if self._prefill_graph is not None:
            return
        stream = torch.cuda.Stream(device=self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(stream):
            self._prefill_body()  # warm-up (the replay that follows recomputes the same state from the same prompts)
        torch.cuda.current_stream(self.device).wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self._prefill_body()
        self._prefill_graph = graph

    def _prefill_body(self) -> None:
        ops.embed(self.prompt_ids, self.prompt_pos, self.wte, self.wpe, out=self.x)
        for index, lw in enumerate(self.layers):
            self._layer(lw, index, self.x, self.ln, self.qkv, self.attn, self.h, decode=False)
        # final LayerNorm on each sequence's last token only, then the LM head with its argmax fused
        last = self.x[self.prompt - 1:]
        ops.layernorm(last, self.lnf_g, self.lnf_b, epsilon=LN_EPSILON, out=self.dln, rows=self.batch,
                      row_stride=self.prompt * self.shape.width)
        self.positions.fill_(self.prompt)
        self._head(index_offset=-self.prompt, advance=0)

    def _head(self, *, index_offset: int, advance: int, seqs: slice = slice(None)) -> None:
        ops.gemm_argmax(self.dln[seqs], self.wte, self.part_val[seqs], self.part_idx[seqs])
        ops.argmax_finish(self.part_val[seqs], self.part_idx[seqs], self.ids[seqs], tokens_out=self.tokens[seqs],
                          positions=self.positions[seqs], index_offset=index_offset, advance=advance)

    # ---- decode ----------------------------------------------------------------------------------------------

    def _persistent_args(self):
        """The persistent decode step's arguments (device pointers of this engine's tensors), rebuilt when the token
        buffer changes."""
        from tempo_compiler_b200 import lib
        key = (self.tokens.data_ptr(), self.tokens.shape[1])
        if self._step_args is not None and self._step_key == key:
            return self._step_args
        layers = (lib.DecodeLayer * len(self.layers))()
        for i, lw in enumerate(self.layers):
            layers[i] = lib.DecodeLayer(
                lw.ln1_g.data_ptr(), lw.ln1_b.data_ptr(), lw.w_qkv.data_ptr(), lw.b_qkv.data_ptr(),
                lw.w_proj.data_ptr(), lw.b_proj.data_ptr(), lw.ln2_g.data_ptr(), lw.ln2_b.data_ptr(),
                lw.w_fc.data_ptr(), lw.b_fc.data_ptr(), lw.w_out.data_ptr(), lw.b_out.data_ptr(),
                self.k_cache[i].data_ptr(), self.v_cache[i].data_ptr())
        args = lib.DecodeStepArgs(
            len(self.layers), self.batch, self.shape.width, self.shape.heads, self.shape.vocab, self.shape.positions,
            self.capacity, LN_EPSILON, layers, self.wte.data_ptr(), self.wpe.data_ptr(), self.lnf_g.data_ptr(),
            self.lnf_b.data_ptr(), self.ids.data_ptr(), self.positions.data_ptr(), self.tokens.data_ptr(),
            self.tokens.shape[1], 1 - self.prompt, self._step_workspace.data_ptr(), self._step_workspace.numel())
        self._step_layers, self._step_args, self._step_key = layers, args, key
        return args

    def _decode_group(self, seqs: slice) -> None:
        """One decode step of the sequences in `seqs` on the current stream."""
        if self.persistent_decode:
            ops.decode_step(self._persistent_args())
            return
        dx, dln, dqkv, dattn, dh = (t[seqs] for t in (self.dx, self.dln, self.dqkv, self.dattn, self.dh))
        ops.embed(self.ids[seqs], self.positions[seqs], self.wte, self.wpe, out=dx)
        if self.fold_layernorms:
            ops.row_stats(dx, self.dstats1[seqs])
        for index, lw in enumerate(self.layers):
            self._layer(lw, index, dx, dln, dqkv, dattn, dh, decode=True, seqs=seqs)
        # the token decoded at position p is generated token p - prompt + 1
        if self._fused_norms(dx):
            ops.gemm_norm(dx, self.lnf_g, self.lnf_b, self.wte, epsilon=LN_EPSILON, part_val=self.part_val[seqs],
                          part_idx=self.part_idx[seqs])
            ops.argmax_finish(self.part_val[seqs], self.part_idx[seqs], self.ids[seqs], tokens_out=self.tokens[seqs],
                              positions=self.positions[seqs], index_offset=1 - self.prompt, advance=1)
            return
        ops.layernorm(dx, self.lnf_g, self.lnf_b, epsilon=LN_EPSILON, out=dln)
        self._head(index_offset=1 - self.prompt, advance=1, seqs=seqs)

    def _decode_step(self) -> None:
        main = torch.cuda.current_stream(self.device)
        # fork every side stream before any group's work is queued, then join them all
        for side in self._side_streams:
            side.wait_stream(main)
        for g, (s0, s1) in enumerate(self.decode_groups):
            with torch.cuda.stream(main if g == 0 else self._side_streams[g - 1]):
                self._decode_group(slice(s0, s1))
        for side in self._side_streams:
            main.wait_stream(side)

    def _capture(self) -> None:
        if self._graph is not None:
            return
        saved_ids, saved_pos = self.ids.clone(), self.positions.clone()
        saved_tokens = self.tokens.clone()
        stream = torch.cuda.Stream(device=self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(stream):
            self._decode_step()  # warm-up: kernel attributes and tensor-map encoders set up before capture
        torch.cuda.current_stream(self.device).wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self._decode_step()
        self._graph = graph
        # the warm-up and the capture advanced state: restore it
        self.ids.copy_(saved_ids)
        self.positions.copy_(saved_pos)
        self.tokens.copy_(saved_tokens)

    def decode(self, steps: int, *, graph: bool = True) -> None:
        """Runs `steps` greedy decode steps, each consuming the last generated token."""
        if steps <= 0:
            return
        if graph:
            self._capture()
            for _ in range(steps):
                self._graph.replay()
        else:
            for _ in range(steps):
                self._decode_step()

    # ---- public API ------------------------------------------------------------------------------------------

    def run(self, token_ids: torch.Tensor, steps: int, *, graph: bool = True) -> torch.Tensor:
        """Prefill plus `steps` decode steps on device-resident prompts; returns [batch, steps + 1] int32 tokens."""
        if token_ids.shape != (self.batch, self.prompt):
            raise ValueError(f"expected prompts of shape {(self.batch, self.prompt)}, got {tuple(token_ids.shape)}")
        self.prompt_ids.copy_(token_ids.reshape(-1))
        return self._run_loaded(steps, graph)

    def _run_loaded(self, steps: int, graph: bool) -> torch.Tensor:
        if self.prompt + steps > self.capacity:
            raise ValueError(f"{self.prompt} prompt tokens + {steps} steps exceed the cache capacity {self.capacity}")
        if self.tokens is None or self.tokens.shape[1] != steps + 1:
            self.tokens = torch.zeros((self.batch, steps + 1), dtype=torch.int32, device=self.device)
            self._graph = None
            self._prefill_graph = None  # both graphs write into the token buffer
        self._prefill_loaded(graph)
        self.decode(steps, graph=graph)
        return self.tokens

    def generate(self, token_ids: np.ndarray, steps: int, *, graph: bool = True) -> np.ndarray:
        """The end-to-end call: host prompts in, host tokens out ([batch, steps + 1]). The prompts go through a pinned
        staging buffer straight into the engine's prompt buffer and the tokens come back through another; both
        buffers are kept between calls (each call ends synchronised, so the next may refill them)."""
        ids = np.asarray(token_ids)
        if ids.shape != (self.batch, self.prompt):
            raise ValueError(f"expected prompts of shape {(self.batch, self.prompt)}, got {tuple(ids.shape)}")
        if self._pinned_ids is None:
            self._pinned_ids = torch.empty((self.batch, self.prompt), dtype=torch.int32, pin_memory=True)
        np.copyto(self._pinned_ids.numpy(), ids, casting="same_kind")
        self.prompt_ids.view(self.batch, self.prompt).copy_(self._pinned_ids, non_blocking=True)
        tokens = self._run_loaded(steps, graph)
        if self._pinned_tokens is None or self._pinned_tokens.shape != tokens.shape:
            self._pinned_tokens = torch.empty(tokens.shape, dtype=torch.int32, pin_memory=True)
        self._pinned_tokens.copy_(tokens, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return self._pinned_tokens.numpy().copy()
