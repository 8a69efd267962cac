"""The .efq reader (efg_efq_check) and the decode oracle, on CPU.

The corruption cases follow the reference's qfile_rejects_corruption test
(tests/test_quant.cpp:208-234): each edit of a good file must be rejected with the
reference's message. The decode oracle (oracle/efo.c efo_forward) is pinned to the
reference decoder's logits committed in tests/golden/decode_tiny.npz.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

import edgeforge_b200 as efg
from oracle.oracle import Oracle, OracleDecoder, read_efq

GOLD = Path(__file__).resolve().parent / "golden"
MAX_SEQ = 64


@pytest.fixture(scope="module")
def good() -> bytes:
    return (GOLD / "decode_tiny_uniform.efq").read_bytes()


def _rejects(data: bytes, what: str) -> None:
    with pytest.raises(efg.EdgeForgeError) as ei:
        efg.efq_check(data)
    assert what in str(ei.value), str(ei.value)


def test_reference_files_parse():
    for tag in ("uniform", "mixed"):
        data = (GOLD / f"decode_tiny_{tag}.efq").read_bytes()
        efg.efq_check(data)
        cfg, tensors = read_efq(GOLD / f"decode_tiny_{tag}.efq")
        assert len(tensors) == 2 * 9 + 3
        assert cfg["hidden_size"] == 64


def test_rejects_corruption(good):
    bad = bytearray(good)
    bad[0] = ord("X")
    _rejects(bytes(bad), "bad magic")
    bad = bytearray(good)
    bad[4] = 2
    _rejects(bytes(bad), "unsupported .efq version 2")
    _rejects(good[:-1], "past the end")
    _rejects(good[:10], "too small")
    # nudge the first tensor offset by one (same text length)
    text = good[16:16 + 4096].decode("latin-1")
    p = text.find('"offset":') + 9
    bad = bytearray(good)
    bad[16 + p] = ord("8") if bad[16 + p] == ord("9") else bad[16 + p] + 1
    _rejects(bytes(bad), "64-byte aligned")
    p = text.find('"bytes":', text.find('"tensors"')) + 8
    bad = bytearray(good)
    bad[16 + p] = ord("8") if bad[16 + p] == ord("9") else bad[16 + p] + 1
    _rejects(bytes(bad), "header says")


def test_rejects_policy_mismatch(good):
    # a layer matrix whose stored type disagrees with the recorded policy
    text = good[16:16 + 8192].decode("latin-1")
    i = text.find('"name":"model.layers.0.self_attn.q_proj.weight","type":"Q4_0"')
    assert i > 0
    j = i + len('"name":"model.layers.0.self_attn.q_proj.weight","type":"')
    bad = bytearray(good)
    bad[16 + j:16 + j + 4] = b"Q8_0"
    with pytest.raises(efg.EdgeForgeError):
        efg.efq_check(bytes(bad))


def test_rejects_bad_header_json(good):
    bad = bytearray(good)
    bad[16] = ord("[")
    with pytest.raises(efg.EdgeForgeError) as ei:
        efg.efq_check(bytes(bad))
    assert "header" in str(ei.value)


def test_empty_and_null():
    _rejects(b"", "too small")


def test_decoder_open_missing_file(tmp_path):
    with pytest.raises(efg.EdgeForgeError) as ei:
        efg.Decoder(tmp_path / "missing.efq", 8)
    assert "cannot open" in str(ei.value)


def test_decoder_open_corrupt_file(tmp_path, good):
    f = tmp_path / "bad.efq"
    f.write_bytes(good[:-1])
    with pytest.raises(efg.EdgeForgeError) as ei:
        efg.Decoder(f, 8)
    assert "past the end" in str(ei.value)


@pytest.mark.parametrize("tag", ["uniform", "mixed"])
def test_oracle_decoder_matches_reference(tag):
    """efo_forward is bit-identical to the reference's scalar Transformer::forward."""
    z = np.load(GOLD / "decode_tiny.npz")
    od = OracleDecoder(Oracle(), GOLD / f"decode_tiny_{tag}.efq", MAX_SEQ)
    got = od.run(z["prompt"], z["forced"], threads=2)
    np.testing.assert_array_equal(got, z[f"{tag}_scalar"])
    if f"{tag}_avx2" in z:
        assert np.abs(got - z[f"{tag}_avx2"]).max() < 1e-5


def test_manifest_lists_decode_fixtures():
    man = json.loads((GOLD / "manifest.json").read_text())
    for f in ("decode_tiny_uniform.efq", "decode_tiny_mixed.efq", "decode_tiny.npz"):
        assert f in man["files"]
        assert (GOLD / f).exists()
