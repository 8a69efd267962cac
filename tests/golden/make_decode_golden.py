#!/usr/bin/env python3
"""Regenerates the decode-step fixtures in tests/golden/ from the reference itself
(oracle/_ref/libefref.so, built from the reference's own sources by oracle/Makefile).

Two small Llama-architecture models (D=64, 4 query / 2 KV heads of 16, F=128, V=96,
2 layers, max_position 64), random BF16 weights from edgeforge_b200.synthetic, are
quantized by the reference's quantize_model:
  * decode_tiny_uniform.efq: the "auto" policy (uniform: Q4_0 layers, Q8_0 lm_head,
    BF16 embedding);
  * decode_tiny_mixed.efq: explicit overrides putting layer 0's k_proj and layer 1's
    up_proj in Q8_0, so q/k/v and gate/up mix storage types.
A third model, decode_tiny_tied.efq (seed 6), ties lm_head to the BF16 embedding; its
logits and greedy tokens are in decode_tiny_tied.npz. For the first two, decode_tiny.npz holds a seeded 7-token prompt, 8 forced continuation ids, the
reference decoder's teacher-forced logits (scalar and AVX2 backends; the logits after
the last prompt token and after each forced id but the last) and the reference's own
greedy tokens (8 steps, argmax of its logits).

    python tests/golden/make_decode_golden.py
"""
from __future__ import annotations

import json
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from edgeforge_b200 import synthetic  # noqa: E402
from oracle.oracle import Reference  # noqa: E402

MAX_SEQ = 64
MIXED = "model.layers.0.self_attn.k_proj.weight=q8_0,model.layers.1.mlp.up_proj.weight=q8_0"


def teacher_forced(dec, prompt, forced, vocab, avx2):
    dec.reset()
    out, pos = [], 0
    for i, t in enumerate(prompt):
        lg = dec.forward(int(t), pos, vocab, avx2=avx2, logits=i + 1 == len(prompt))
        pos += 1
    out.append(lg)
    for t in forced[:-1]:
        out.append(dec.forward(int(t), pos, vocab, avx2=avx2))
        pos += 1
    return np.stack(out)


def greedy(dec, prompt, steps, vocab):
    """generate_greedy (src/model.cpp:278-304) with eos disabled."""
    dec.reset()
    pos = 0
    for i, t in enumerate(prompt):
        lg = dec.forward(int(t), pos, vocab, logits=i + 1 == len(prompt))
        pos += 1
    toks = []
    for step in range(steps):
        tok = int(np.argmax(lg))  # first maximum, as kern::argmax
        toks.append(tok)
        if step + 1 == steps:
            break
        lg = dec.forward(tok, pos, vocab)
        pos += 1
    return np.array(toks, np.int32)


def main() -> int:
    ref = Reference()
    cfg = synthetic.tiny_config(max_pos=MAX_SEQ)
    V = cfg["vocab_size"]
    rng = np.random.default_rng(11)
    prompt = rng.integers(0, V, 7).astype(np.int32)
    forced = rng.integers(0, V, 8).astype(np.int32)
    out = {"prompt": prompt, "forced": forced}
    with tempfile.TemporaryDirectory() as td:
        src = synthetic.write_checkpoint(Path(td) / "ckpt", cfg, seed=5)
        for tag, overrides in (("uniform", ""), ("mixed", MIXED)):
            efq = HERE / f"decode_tiny_{tag}.efq"
            ref.quantize_model(src, efq, policy="auto", overrides=overrides, threads=1)
            dec = ref.decoder(efq, MAX_SEQ, threads=1)
            out[f"{tag}_scalar"] = teacher_forced(dec, prompt, forced, V, avx2=False)
            if ref.avx2:
                out[f"{tag}_avx2"] = teacher_forced(dec, prompt, forced, V, avx2=True)
            out[f"{tag}_greedy"] = greedy(dec, prompt, 8, V)
            out[f"{tag}_bytes_per_token"] = np.array(dec.bytes_per_token(), np.uint64)
            dec.close()
        # tied embeddings: lm_head is the BF16 embedding itself (src/model.cpp:88, 273)
        tcfg = dict(cfg, tie_word_embeddings=True)
        tsrc = synthetic.write_checkpoint(Path(td) / "ckpt_tied", tcfg, seed=6)
        efq = HERE / "decode_tiny_tied.efq"
        ref.quantize_model(tsrc, efq, policy="auto", threads=1)
        dec = ref.decoder(efq, MAX_SEQ, threads=1)
        tied = {"prompt": prompt, "forced": forced,
                "tied_scalar": teacher_forced(dec, prompt, forced, V, avx2=False),
                "tied_greedy": greedy(dec, prompt, 8, V)}
        if ref.avx2:
            tied["tied_avx2"] = teacher_forced(dec, prompt, forced, V, avx2=True)
        dec.close()
    np.savez_compressed(HERE / "decode_tiny.npz", **out)
    np.savez_compressed(HERE / "decode_tiny_tied.npz", **tied)
    man_path = HERE / "manifest.json"
    man = json.loads(man_path.read_text()) if man_path.exists() else {"files": {}}
    man["files"]["decode_tiny_uniform.efq"] = "tiny Llama model, reference quantize_model policy auto (uniform)"
    man["files"]["decode_tiny_mixed.efq"] = "same weights, overrides " + MIXED
    man["files"]["decode_tiny_tied.efq"] = "tiny Llama model with tied embeddings (BF16 lm_head), policy auto"
    man["files"]["decode_tiny_tied.npz"] = "reference decoder teacher-forced logits and greedy tokens of the tied model"
    man["files"]["decode_tiny.npz"] = ("prompt/forced ids; reference decoder teacher-forced logits (scalar, AVX2) "
                                       "and greedy tokens for both models (make_decode_golden.py)")
    man_path.write_text(json.dumps(man, indent=1) + "\n")
    print("wrote decode_tiny_{uniform,mixed,tied}.efq, decode_tiny.npz, decode_tiny_tied.npz")
    return 0


if __name__ == "__main__":
    sys.exit(main())
