#!/usr/bin/env python3
"""Generates the golden vectors that pin the oracle to the reference's own host references.

Run in the build container, where the reference is importable from /root/reference (read-only). It imports the
reference's ``board_package/bf16.py``, ``references.py``, ``gpt2_inference.py`` (for ``embed`` and ``lm_head``) and
``board_checks.py`` (for ``_block_weights``), runs them on seeded inputs, and writes ``oracle_golden.npz`` beside this
script. The GPU box never reads the reference; it only reads the committed ``.npz``.

    python tests/golden/make_golden.py [--reference /root/reference]
"""

from __future__ import annotations

import argparse
import hashlib
import pathlib
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parents[1]


def sha(array) -> str:
    return hashlib.sha256(np.ascontiguousarray(array).tobytes()).hexdigest()


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", default="/root/reference")
    args = parser.parse_args()
    sys.path.insert(0, str(pathlib.Path(args.reference) / "board_package"))
    sys.path.insert(0, str(ROOT))

    import bf16 as rb  # the reference's module
    import references as rr
    import gpt2_inference as gi
    import board_checks as bc
    from tempo_compiler_b200.weights import GPT2Shape, random_gpt2

    out: dict[str, np.ndarray] = {}
    rng = np.random.default_rng(2024)

    # 1. BF16 rounding: specials, ties and random values.
    specials = np.array([0.0, -0.0, 1.0, -1.0, 1.00390625, 1.005859375, 1.0078125, 65504.0, 3.0e38, -3.0e38,
                         1e-40, -1e-40, 1.17549435e-38, np.inf, -np.inf, 2.0 ** -133], dtype=np.float32)
    ties = (np.arange(1, 513, dtype=np.uint32) << 16 | np.uint32(0x8000)).view(np.float32)
    rand = np.concatenate([rng.standard_normal(4096).astype(np.float32) * 10.0 ** rng.integers(-20, 20, 4096)])
    rne_in = np.concatenate([specials, ties, rand.astype(np.float32)])
    out["rne_in"] = rne_in
    out["rne_out"] = rb.as_bf16_words(values=rne_in.copy())

    # 2. The GELU ROM and the table GELU over every BF16 word.
    out["gelu_table"] = rb._gelu_table()
    every = np.arange(1 << 16, dtype=np.uint32)
    lut = rb.gelu_lut_reference(words=every)
    assert int(lut.max()) < (1 << 16)
    out["gelu_lut_all"] = lut.astype(np.uint16)

    # 3. Packers, with padding on every padded axis.
    act = rng.standard_normal((32, 40)).astype(np.float32)
    wts = rng.standard_normal((40, 24)).astype(np.float32)
    bias = rng.standard_normal(24).astype(np.float32)
    out["pack_act_in"], out["pack_act_out"] = act, rb.pack_activations(activations=act)
    out["pack_wts_in"], out["pack_wts_out"] = wts, rb.pack_weights(weights=wts)
    out["pack_bias_in"], out["pack_bias_out"] = bias, rb.pack_bias(bias=bias)
    masks = rb.decode_mask_tiles(keys=64, length=49)
    out["decode_consts_64_49"] = rb.pack_attention_constants(
        initial_maximum=-1e30, constants=(), masks=np.ascontiguousarray(masks.swapaxes(-1, -2))).reshape(-1)
    out["decode_consts_256_200_plain"] = rb.pack_attention_constants(
        initial_maximum=-1e30, constants=(1.5,), masks=rb.decode_mask_tiles(keys=256, length=200)).reshape(-1)

    # 4. LayerNorm on the board check's operands (board_checks.py:337-340).
    lrng = np.random.default_rng(0)
    rows = rb._on_bf16_grid(values=(lrng.standard_normal((32, 768)) * 2.0).astype(np.float32))
    gamma = rb._on_bf16_grid(values=(1.0 + 0.1 * lrng.standard_normal(768)).astype(np.float32))
    beta = rb._on_bf16_grid(values=(0.1 * lrng.standard_normal(768)).astype(np.float32))
    out["ln_inputs_sha"] = np.array([sha(rows), sha(gamma), sha(beta)])
    out["ln_out"] = rb.as_bf16_words(values=rr.layernorm_reference(rows=rows, gamma=gamma, beta=beta))

    # 5. Softmax and the device product.
    scores = (rng.standard_normal((16, 64)) * 3.0).astype(np.float32)
    out["softmax_in"], out["softmax_out"] = scores, rr.softmax_reference(scores=scores)
    left = rb._on_bf16_grid(values=rng.standard_normal((32, 96)).astype(np.float32))
    right = rb._on_bf16_grid(values=(rng.standard_normal((96, 48)) * 0.1).astype(np.float32))
    out["dp_left"], out["dp_right"] = left, right
    out["dp_out"] = rb.as_bf16_words(values=rr._device_product(left, right))

    # 6. Attention: the device model (causal), the tile-wise BF16 model and the float64 check.
    q = rb._on_bf16_grid(values=rng.standard_normal((64, 64)).astype(np.float32))
    k = rb._on_bf16_grid(values=rng.standard_normal((64, 64)).astype(np.float32))
    v = rb._on_bf16_grid(values=rng.standard_normal((64, 64)).astype(np.float32))
    out["att_q"], out["att_k"], out["att_v"] = q, k, v
    out["att_device_causal"] = rr.attention_reference(query=q, key=k, value=v, causal=True)
    dmask = rb.decode_mask_tiles(keys=64, length=49)[0].transpose(1, 0, 2).reshape(16, 64)
    out["att_tiles_masked"] = rb.attention_bf16_reference(q[:16] / 8.0, k, v, initial_maximum=-1e30, mask=dmask)
    out["att_f64_masked"] = rb.attention_reference(q[:16] / 8.0, k, v, mask=dmask)

    # 7. One transformer block on the board check's weights (board_checks.py:501-508) over 32 tokens.
    brng = np.random.default_rng(1)
    hidden = rb._on_bf16_grid(values=(brng.standard_normal((32, 768)) * 0.5).astype(np.float32))
    weights = bc._block_weights(model=768, seed=2)
    out["block_hidden_sha"] = np.array([sha(hidden)])
    out["block_out"] = rb.as_bf16_words(values=rr.transformer_block_reference(hidden=hidden, weights=weights))
    out["block_weights_sha"] = np.array([name + ":" + sha(value) for name, value in weights.items()])

    # 8. Operand builders (hashes: the arrays are large and regenerated from their seeds).
    sl, sr = rb.build_operands(32, 768, 3072, kind="structured", seed=0)
    vl, vr = rb.build_operands(32, 768, 3072, kind="varying", seed=0)
    out["operands_sha"] = np.array([sha(sl), sha(sr), sha(vl), sha(vr)])

    # 9. A small random GPT-2 (two layers, the full vocabulary) through the reference chain: two greedy tokens as
    #    board_checks.check_gpt2_decode computes its reference (board_checks.py:467-474).
    shape = GPT2Shape(layers=2)
    layers, shared = random_gpt2(7, shape)
    prompt = (464, 3139, 286, 4881, 318)
    tokens, tops = [], []
    for sequence in (prompt, None):
        sequence = prompt if sequence is not None else (*prompt, tokens[0])
        rows_ = gi.embed(np.asarray(sequence), shared)
        for w in layers:
            rows_ = rr.transformer_block_reference(hidden=rows_, weights=w)
        normalised = rr.layernorm_reference(rows=rows_[-1:], gamma=shared["ln_f.g"], beta=shared["ln_f.b"])[0]
        logits = gi.lm_head(normalised, shared)
        tokens.append(int(np.argmax(logits)))
        tops.append(np.sort(logits)[-5:][::-1].astype(np.float32))
    out["gpt2_small2_prompt"] = np.asarray(prompt, dtype=np.int64)
    out["gpt2_small2_tokens"] = np.asarray(tokens, dtype=np.int64)
    out["gpt2_small2_top5"] = np.stack(tops)

    np.savez_compressed(HERE / "oracle_golden.npz", **out)
    size = (HERE / "oracle_golden.npz").stat().st_size
    print(f"wrote {HERE / 'oracle_golden.npz'} ({size / 1024:.0f} KiB, {len(out)} arrays); greedy tokens {tokens}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
