"""The decode step on the GPU (efg_decoder_*) against the reference decoder.

Small models: the committed fixtures in tests/golden (reference-quantized .efq files and
the reference's teacher-forced logits). Full size: a random TinyLlama-1.1B-shaped
checkpoint quantized by the reference with its "auto" policy (148 Q4_0 + 6 Q8_0 layer
matrices, Q8_0 lm_head, BF16 embedding), a 23-token prompt and 32 greedy steps,
teacher-forced on the reference's own greedy tokens. Tolerance: logits within 1e-4
absolute at every step.
"""
from __future__ import annotations

import os
from pathlib import Path

import numpy as np
import pytest

import edgeforge_b200 as efg

pytestmark = pytest.mark.gpu

GOLD = Path(__file__).resolve().parent / "golden"
MAX_SEQ = 64
TOL = 1e-4


@pytest.fixture(scope="module")
def z():
    return np.load(GOLD / "decode_tiny.npz")


def _forward_run(dec, prompt, forced):
    dec.reset()
    out, pos = [], 0
    for i, t in enumerate(prompt):
        lg = dec.forward(int(t), pos, compute_logits=i + 1 == len(prompt))
        pos += 1
    out.append(lg)
    for t in forced[:-1]:
        out.append(dec.forward(int(t), pos))
        pos += 1
    return np.stack(out)


@pytest.mark.parametrize("tag", ["uniform", "mixed"])
def test_forward_matches_reference(z, tag):
    with efg.Decoder(GOLD / f"decode_tiny_{tag}.efq", MAX_SEQ) as dec:
        got = _forward_run(dec, z["prompt"], z["forced"])
        err = np.abs(got - z[f"{tag}_scalar"]).max()
        assert err <= TOL, err
        assert dec.bytes_per_token == int(z[f"{tag}_bytes_per_token"])
        # a second pass over the same positions (cache rewound by reset) is deterministic
        again = _forward_run(dec, z["prompt"], z["forced"])
        np.testing.assert_array_equal(got, again)


@pytest.mark.parametrize("tag", ["uniform", "mixed"])
def test_batched_prefill_matches_reference(z, tag):
    """The prompt as one batch gives the reference's logits after the prompt, and the KV
    cache it writes carries the teacher-forced steps that follow; a prompt split in two
    batches (the second at pos0 > 0) agrees."""
    ref = z[f"{tag}_scalar"]
    prompt, forced = z["prompt"], z["forced"]
    with efg.Decoder(GOLD / f"decode_tiny_{tag}.efq", MAX_SEQ) as dec:
        got = [dec.prefill(prompt)]
        pos = len(prompt)
        for t in forced[:-1]:
            got.append(dec.forward(int(t), pos))
            pos += 1
        assert np.abs(np.stack(got) - ref).max() <= TOL
        dec.reset()
        k = len(prompt) // 2
        assert dec.prefill(prompt[:k], compute_logits=False) is None
        assert np.abs(dec.prefill(prompt[k:], pos0=k) - ref[0]).max() <= TOL
        assert efg.device_error() == 0


def test_batched_prefill_errors(z):
    with efg.Decoder(GOLD / "decode_tiny_uniform.efq", 16) as dec:
        with pytest.raises(efg.EdgeForgeError, match="skips ahead"):
            dec.prefill(np.array([1, 2], np.int32), pos0=1)
        with pytest.raises(efg.EdgeForgeError, match="KV-cache capacity"):
            dec.prefill(np.arange(17, dtype=np.int32))
        with pytest.raises(efg.EdgeForgeError, match="outside"):
            dec.prefill(np.array([1, 96], np.int32))
        with pytest.raises(efg.EdgeForgeError, match="no tokens"):
            dec.prefill(np.array([], np.int32))


@pytest.mark.parametrize("tag", ["uniform", "mixed"])
def test_generate_teacher_forced(z, tag):
    ref = z[f"{tag}_scalar"]
    with efg.Decoder(GOLD / f"decode_tiny_{tag}.efq", MAX_SEQ) as dec:
        r = dec.generate(z["prompt"], len(z["forced"]), forced=z["forced"], keep_step_logits=True)
        assert len(r.tokens) == len(z["forced"])
        assert np.abs(r.step_logits - ref[1:]).max() <= TOL
        # each step's token is the argmax of that step's logits
        np.testing.assert_array_equal(np.array(r.tokens), np.argmax(ref, axis=1))


@pytest.mark.parametrize("tag", ["uniform", "mixed"])
def test_generate_greedy_and_eos(z, tag):
    want = z[f"{tag}_greedy"]
    with efg.Decoder(GOLD / f"decode_tiny_{tag}.efq", MAX_SEQ) as dec:
        r = dec.generate(z["prompt"], len(want))
        np.testing.assert_array_equal(np.array(r.tokens), want)
        assert r.decode_forwards == len(want) - 1
        eos = int(want[2])
        stop = int(np.argmax(want == eos))
        r = dec.generate(z["prompt"], len(want), eos_id=eos)
        np.testing.assert_array_equal(np.array(r.tokens), want[: stop + 1])
        # a 1-token prompt and a single step
        r = dec.generate(z["prompt"][:1], 1)
        assert len(r.tokens) == 1


def test_forward_errors(z):
    with efg.Decoder(GOLD / "decode_tiny_uniform.efq", 16) as dec:
        with pytest.raises(efg.EdgeForgeError, match="outside"):
            dec.forward(96, 0)
        with pytest.raises(efg.EdgeForgeError, match="skips ahead"):
            dec.forward(1, 3)
        for p in range(16):
            dec.forward(1, p, compute_logits=False)
        with pytest.raises(efg.EdgeForgeError, match="KV-cache capacity"):
            dec.forward(1, 16)
        with pytest.raises(efg.EdgeForgeError, match="exceeds the KV-cache capacity"):
            dec.generate(z["prompt"], 10)
        with pytest.raises(efg.EdgeForgeError, match="empty prompt"):
            dec.generate([], 2)
        assert efg.device_error() == 0
    with pytest.raises(efg.EdgeForgeError, match="max_position_embeddings"):
        efg.Decoder(GOLD / "decode_tiny_uniform.efq", 65)


def test_rewind_recomputes(z):
    """forward at pos < cached drops the later positions, as Transformer::forward does."""
    with efg.Decoder(GOLD / "decode_tiny_uniform.efq", MAX_SEQ) as dec:
        ref = _forward_run(dec, z["prompt"], z["forced"])
        n = len(z["prompt"])
        lg = dec.forward(int(z["forced"][0]), n)  # rewinds to just after the prompt
        np.testing.assert_array_equal(lg, ref[1])


def test_tiny_models_use_the_graph_path():
    """36-byte rows cannot be bulk-copied: these models run the per-operation graphs."""
    with efg.Decoder(GOLD / "decode_tiny_uniform.efq", MAX_SEQ) as dec:
        assert not dec.persistent
        with pytest.raises(efg.EdgeForgeError, match="persistent kernel cannot run"):
            dec.persistent = True


# ---------------------------------------------------------------- medium model, both modes

MEDIUM_MIXED = "model.layers.0.self_attn.k_proj.weight=q8_0,model.layers.1.mlp.up_proj.weight=q8_0"


@pytest.fixture(scope="module")
def medium(tmp_path_factory):
    """D=256 / F=512 / 4 heads of 64 / 2 KV heads / V=300, written by the GPU writer with
    q/k and gate/up of mixed storage types; the oracle's decoder gives the reference logits."""
    from edgeforge_b200 import synthetic
    from oracle.oracle import Oracle, OracleDecoder

    d = tmp_path_factory.mktemp("medium")
    cfg = synthetic.tiny_config(hidden=256, intermediate=512, layers=2, heads=4, kv_heads=2, vocab=300, max_pos=128)
    synthetic.write_checkpoint(d / "ckpt", cfg, seed=8)
    efq = d / "m.efq"
    efg.quantize_model(d / "ckpt", efq, overrides=MEDIUM_MIXED)
    rng = np.random.default_rng(12)
    prompt = rng.integers(0, 300, 9).astype(np.int32)
    forced = rng.integers(0, 300, 12).astype(np.int32)
    ref = OracleDecoder(Oracle(), efq, 64).run(prompt, forced, threads=4)
    return efq, prompt, forced, ref


def test_medium_batched_prefill(medium):
    """q/k and gate/up of mixed storage types (GEMM and per-token matvecs in one layer):
    the batched prompt gives the reference's logits; a 100-token prompt (two passes) agrees
    with our token-by-token forward, and so does the step after it."""
    efq, prompt, forced, ref = medium
    with efg.Decoder(efq, 128) as dec:
        assert np.abs(dec.prefill(prompt) - ref[0]).max() <= TOL
        long = np.random.default_rng(5).integers(0, 300, 100).astype(np.int32)
        dec.reset()
        for i, t in enumerate(long):
            want = dec.forward(int(t), i, compute_logits=i + 1 == len(long))
        nxt = dec.forward(7, len(long))
        dec.reset()
        assert np.abs(dec.prefill(long) - want).max() <= TOL
        assert np.abs(dec.forward(7, len(long)) - nxt).max() <= TOL
        assert efg.device_error() == 0


def test_medium_multi_sequence_step(medium):
    """Three sequences of different lengths in three slots, stepped together (their rows
    share each GEMM): each one's logits after its last token match the reference decoder
    run on that sequence alone."""
    from oracle.oracle import Oracle, OracleDecoder

    efq = medium[0]
    rng = np.random.default_rng(21)
    seqs = [rng.integers(0, 300, n).astype(np.int32) for n in (9, 4, 13)]
    o = Oracle()
    want = [OracleDecoder(o, efq, 64).run(s, np.array([1], np.int32), threads=4)[0] for s in seqs]
    with efg.Decoder(efq, 64) as dec:
        dec.set_slots(3)
        last = [None] * 3
        for t in range(max(len(s) for s in seqs)):
            live = [i for i, s in enumerate(seqs) if t < len(s)]
            lg, nxt = dec.step_slots(live, [seqs[i][t] for i in live], [t] * len(live))
            np.testing.assert_array_equal(nxt, np.argmax(lg, axis=1))
            for r, i in enumerate(live):
                last[i] = lg[r]
        for i in range(3):
            assert np.abs(last[i] - want[i]).max() <= TOL, i
        assert efg.device_error() == 0


def test_multi_sequence_matches_forward(z):
    """Slot 0 is the decoder's own cache: a step of slot 0 continues a forward() run, and a
    sequence replayed in slot 1 gives forward()'s logits."""
    prompt = z["prompt"]
    with efg.Decoder(GOLD / "decode_tiny_mixed.efq", MAX_SEQ) as dec:
        ref = [dec.forward(int(t), i) for i, t in enumerate(prompt)]
        dec.set_slots(2)
        for i, t in enumerate(prompt):
            lg, _ = dec.step_slots([1], [t], [i])
            assert np.abs(lg[0] - ref[i]).max() <= TOL
        lg, _ = dec.step_slots([0, 1], [5, 5], [len(prompt), len(prompt)])
        assert np.abs(lg[0] - lg[1]).max() <= TOL  # same history in both slots
        want = dec.forward(5, len(prompt))  # rewinds slot 0 to the same position
        assert np.abs(lg[0] - want).max() <= TOL
        with pytest.raises(efg.EdgeForgeError, match="twice"):
            dec.step_slots([1, 1], [1, 2], [0, 0])
        with pytest.raises(efg.EdgeForgeError, match="outside"):
            dec.step_slots([2], [1], [0])
        with pytest.raises(efg.EdgeForgeError, match="skips ahead"):
            dec.step_slots([1], [1], [40])


@pytest.mark.parametrize("persistent", [True, False])
def test_medium_forward_and_generate(medium, persistent):
    efq, prompt, forced, ref = medium
    with efg.Decoder(efq, 64) as dec:
        assert not dec.persistent  # the per-operation graphs are the default
        dec.persistent = persistent
        got = _forward_run(dec, prompt, forced)
        assert np.abs(got - ref).max() <= TOL, np.abs(got - ref).max()
        r = dec.generate(prompt, len(forced), forced=forced, keep_step_logits=True)
        assert np.abs(r.step_logits - ref[1:]).max() <= TOL
        np.testing.assert_array_equal(np.array(r.tokens), np.argmax(ref, axis=1))
        g = dec.generate(prompt, 10)
        eos = g.tokens[3]
        stop = g.tokens.index(eos)
        e = dec.generate(prompt, 10, eos_id=eos)
        assert e.tokens == g.tokens[: stop + 1]
        first = dec.generate(prompt, 10, eos_id=g.tokens[0])  # eos straight after the prompt
        assert first.tokens == g.tokens[:1]
        assert dec.generate(prompt, 0).tokens == []
        assert efg.device_error() == 0


def test_medium_modes_agree(medium):
    efq, prompt, forced, _ = medium
    with efg.Decoder(efq, 64) as a, efg.Decoder(efq, 64) as b:
        a.persistent = True
        ra = a.generate(prompt, 12, forced=forced, keep_step_logits=True)
        rb = b.generate(prompt, 12, forced=forced, keep_step_logits=True)
        assert ra.tokens == rb.tokens
        assert np.abs(ra.step_logits - rb.step_logits).max() <= TOL


# ---------------------------------------------------------------- full TinyLlama shape

FULL_PROMPT = 23
FULL_STEPS = 32


@pytest.mark.parametrize("persistent", [True, False])
def test_full_tinyllama_decode(tinyllama, persistent):
    full_model = tinyllama[1]
    from oracle.oracle import Reference

    ref = Reference()
    V = 32000
    prompt = np.random.default_rng(2).integers(0, V, FULL_PROMPT).astype(np.int32)
    threads = max(1, min(32, os.cpu_count() or 1))
    rd = ref.decoder(full_model, FULL_PROMPT + FULL_STEPS, threads=threads)
    # the reference's greedy run (generate_greedy) gives the ids to teacher-force on
    logits_ref, toks, pos = [], [], 0
    for i, t in enumerate(prompt):
        lg = rd.forward(int(t), pos, V, logits=i + 1 == FULL_PROMPT)
        pos += 1
    for step in range(FULL_STEPS):
        logits_ref.append(lg)
        toks.append(int(np.argmax(lg)))
        if step + 1 == FULL_STEPS:
            break
        lg = rd.forward(toks[-1], pos, V)
        pos += 1
    bpt = rd.bytes_per_token()
    rd.close()
    logits_ref = np.stack(logits_ref)
    with efg.Decoder(full_model, FULL_PROMPT + FULL_STEPS) as dec:
        dec.persistent = persistent
        info = dec.info
        assert (info.n_q4, info.n_q8) == (148, 7)
        assert dec.bytes_per_token == bpt == 616_570_880
        r = dec.generate(prompt, FULL_STEPS, forced=np.array(toks, np.int32), keep_step_logits=True)
        err = np.abs(r.step_logits - logits_ref[1:]).max()
        assert err <= TOL, err
        first = dec.forward(int(prompt[-1]), FULL_PROMPT - 1)  # logits after the prompt
        assert np.abs(first - logits_ref[0]).max() <= TOL
        dec.reset()
        assert np.abs(dec.prefill(prompt) - logits_ref[0]).max() <= TOL  # batched prompt
        # free-running greedy decode agrees with the reference's tokens up to the first
        # step whose top-2 logit margin is within the tolerance (a legitimate near-tie)
        g = dec.generate(prompt, FULL_STEPS)
        top2 = np.sort(logits_ref, axis=1)[:, -2:]
        tie = np.nonzero(top2[:, 1] - top2[:, 0] <= 2 * TOL)[0]
        n = int(tie[0]) if tie.size else FULL_STEPS
        np.testing.assert_array_equal(np.array(g.tokens[:n]), np.array(toks[:n]))
        assert efg.device_error() == 0


def test_non_finite_weight_same_on_both_paths(tmp_path, z):
    """An infinite FP16 scale in layer 0's q_proj (a weight of +-inf, and inf * 0 = NaN at code 8):
    the per-token path (matvec) and the batched prompt path (tensor-core GEMM, whose split of an
    infinite operand gives NaN where the matvec gives +-inf) both end in non-finite logits at the
    same positions, so the GEMM's documented difference does not change what the decoder emits."""
    import json as _json

    src = GOLD / "decode_tiny_uniform.efq"
    raw = bytearray(src.read_bytes())
    hlen = int.from_bytes(raw[8:16], "little")
    hdr = _json.loads(bytes(raw[16:16 + hlen]).decode())
    t = next(t for t in hdr["tensors"] if t["name"] == "model.layers.0.self_attn.q_proj.weight")
    assert t["type"].upper() == "Q4_0"
    off = int(t["offset"])
    raw[off:off + 2] = (0x7C00).to_bytes(2, "little")  # first block's scale: +inf
    bad = tmp_path / "inf_scale.efq"
    bad.write_bytes(bytes(raw))
    prompt = [int(v) for v in z["prompt"]]
    with efg.Decoder(bad, MAX_SEQ) as a, efg.Decoder(bad, MAX_SEQ) as b:
        for i, tok in enumerate(prompt):
            la = a.forward(tok, i, compute_logits=i + 1 == len(prompt))
        lb = b.prefill(np.array(prompt, np.int32), 0)
        assert np.array_equal(np.isfinite(la), np.isfinite(lb))
        assert not np.isfinite(la).all()
    assert efg.device_error() == 0
