"""The GPU .efq writer (efg_quantize_model).

CPU: the argument and checkpoint checks that run before any device work, with the
reference's messages (src/quantizer.cpp:92-115, src/qfile.cpp:79-115,
src/model_config.cpp:179-224). GPU: the written file is byte-identical to the reference
writer's output: the committed reference-written fixtures for the small models, and the
reference's own file for the full TinyLlama-1.1B shape.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

import edgeforge_b200 as efg
from edgeforge_b200 import synthetic

GOLD = Path(__file__).resolve().parent / "golden"
MIXED = "model.layers.0.self_attn.k_proj.weight=q8_0,model.layers.1.mlp.up_proj.weight=q8_0"


@pytest.fixture(scope="module")
def tiny_dir(tmp_path_factory):
    """The checkpoint tests/golden/make_decode_golden.py quantized with the reference."""
    return synthetic.write_checkpoint(tmp_path_factory.mktemp("tiny"), synthetic.tiny_config(max_pos=64), seed=5)


def _fails(tmp, src, what, policy="auto", overrides=""):
    with pytest.raises(efg.EdgeForgeError) as ei:
        efg.quantize_model(src, tmp / "out.efq", policy=policy, overrides=overrides)
    assert what in str(ei.value), str(ei.value)


def test_rejects_bad_arguments(tiny_dir, tmp_path):
    _fails(tmp_path, tmp_path / "nowhere", "cannot open")
    _fails(tmp_path, tiny_dir, "unknown policy", policy="fastest")
    _fails(tmp_path, tiny_dir, "another architecture", policy="tinyllama-1.1b-chat-v1.0")
    _fails(tmp_path, tiny_dir, "must look like TENSOR=TYPE", overrides="model.layers.0.self_attn.k_proj.weight")
    _fails(tmp_path, tiny_dir, "type must be one of", overrides="model.layers.0.self_attn.k_proj.weight=q5_1")
    _fails(tmp_path, tiny_dir, "norms are always F32", overrides="*norm*=q8_0")
    _fails(tmp_path, tiny_dir, "matches no tensor", overrides="model.layers.9.mlp.up_proj.weight=q8_0")


def test_rejects_mismatched_checkpoint(tiny_dir, tmp_path):
    cfg = json.loads((tiny_dir / "config.json").read_text())
    bad = tmp_path / "bad"
    bad.mkdir()
    (bad / "model.safetensors").write_bytes((tiny_dir / "model.safetensors").read_bytes())
    cfg["num_hidden_layers"] = 3
    (bad / "config.json").write_text(json.dumps(cfg))
    _fails(tmp_path, bad, "missing tensor 'model.layers.2.")
    cfg["num_hidden_layers"] = 2
    cfg["intermediate_size"] = 96
    (bad / "config.json").write_text(json.dumps(cfg))
    _fails(tmp_path, bad, "has shape [128, 64], expected [96, 64]")


@pytest.mark.gpu
@pytest.mark.parametrize("tag,overrides", [("uniform", ""), ("mixed", MIXED)])
def test_matches_reference_writer_small(tiny_dir, tmp_path, tag, overrides):
    out = tmp_path / f"{tag}.efq"
    rep = efg.quantize_model(tiny_dir, out, policy="auto", overrides=overrides)
    want = (GOLD / f"decode_tiny_{tag}.efq").read_bytes()
    got = out.read_bytes()
    assert got == want
    assert rep.file_bytes == len(want)
    assert rep.n_tensors == 21
    efg.efq_check(got)


@pytest.mark.gpu
def test_fallback_bf16_rows(tmp_path, reference):
    """Row lengths that are not a multiple of 32 stay BF16 (rule fallback-bf16), as in the
    reference's qfile_falls_back_to_bf16_for_odd_rows (tests/test_quant.cpp:198-206)."""
    src = synthetic.write_checkpoint(tmp_path / "odd", synthetic.tiny_config(hidden=48, intermediate=96, vocab=40,
                                                                             heads=4, kv_heads=2), seed=9)
    efg.quantize_model(src, tmp_path / "a.efq")
    reference.quantize_model(src, tmp_path / "b.efq", policy="auto")
    got, want = (tmp_path / "a.efq").read_bytes(), (tmp_path / "b.efq").read_bytes()
    assert got == want
    assert b'"rule":"fallback-bf16"' in got


@pytest.mark.gpu
def test_matches_reference_writer_tinyllama(tinyllama, tmp_path):
    model_dir, ref_efq = tinyllama
    out = tmp_path / "gpu.efq"
    rep = efg.quantize_model(model_dir, out, policy="auto")
    assert rep.bytes_per_token == 616_570_880
    assert rep.override_extra_bytes == 6 * 256 * 64 * 16  # six [256][2048] matrices, 16 B more per block
    a = np.memmap(out, dtype=np.uint8, mode="r")
    b = np.memmap(ref_efq, dtype=np.uint8, mode="r")
    assert a.size == b.size
    diff = np.nonzero(a != b)[0]
    assert diff.size == 0, f"first difference at byte {diff[0]}"
