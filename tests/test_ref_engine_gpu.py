"""The reference's own decode engine running on the GPU through the drop-in headers.

tests/shim/_build/ref_engine is the reference's src/model.cpp, qfile.cpp, kernels.cpp,
json.cpp, mapped_file.cpp, model_config.cpp, safetensors.cpp and threadpool.cpp compiled
unchanged with include/shim/ef/quant.h and include/shim/ef/qkernels.h in place of the
reference's headers (so every matvec, quantize/dequantize and row lookup of
Transformer::forward, src/model.cpp:184-276, goes to libefg.so), and src/quant.cpp and
src/qkernels.cpp left out (recipe: tests/shim/Makefile, built by __graft_entry__.build() where
the reference tree is present). Its teacher-forced logits must match the reference decoder's
own (the committed fixtures, made by tests/golden/make_decode_golden.py) within 1e-4:
packed Q4_0 / Q8_0 views, the same model as F32 views (Model::dequantized_copy), and a model
whose lm_head is the tied BF16 embedding (src/model.cpp:88, 273)."""
from __future__ import annotations

import subprocess
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent
GOLD = ROOT / "tests" / "golden"
EXE = ROOT / "tests" / "shim" / "_build" / "ref_engine"
TOL = 1e-4


@pytest.fixture(scope="module")
def engine(efg_lib):
    if not EXE.exists():
        from oracle.oracle import reference_tree

        tree = reference_tree()
        if tree is None:
            pytest.fail("tests/shim/_build/ref_engine is not built and no reference tree is present")
        subprocess.run(["make", "-C", str(ROOT / "tests" / "shim"), "-j8", f"REF={tree}"], check=True,
                       capture_output=True)
    return EXE


def _run(engine, efq, prompt, forced, out, *extra):
    ids = lambda a: ",".join(str(int(t)) for t in a)  # noqa: E731
    r = subprocess.run([str(engine), str(efq), ids(prompt), ids(forced), str(out), *extra], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    return np.fromfile(out, dtype=np.float32), r.stdout


@pytest.mark.parametrize("mode", ["packed", "dequantized"])
@pytest.mark.parametrize("tag", ["uniform", "mixed"])
def test_reference_engine_on_the_gpu(engine, tmp_path, tag, mode):
    g = np.load(GOLD / "decode_tiny.npz")
    want = g[f"{tag}_scalar"]
    got, out = _run(engine, GOLD / f"decode_tiny_{tag}.efq", g["prompt"], g["forced"], tmp_path / "lg.f32",
                    *(["dequantized"] if mode == "dequantized" else []))
    got = got.reshape(want.shape)
    assert np.abs(got - want).max() <= TOL, np.abs(got - want).max()
    assert ("F32 views" in out) == (mode == "dequantized")


def test_reference_engine_tied_bf16_lm_head(engine, tmp_path):
    g = np.load(GOLD / "decode_tiny_tied.npz")
    want = g["tied_scalar"]
    got, out = _run(engine, GOLD / "decode_tiny_tied.efq", g["prompt"], g["forced"], tmp_path / "lg.f32")
    got = got.reshape(want.shape)
    assert "embedding BF16" in out
    assert np.abs(got - want).max() <= TOL, np.abs(got - want).max()
    # greedy continuation as the reference takes it (argmax of each row)
    assert list(np.argmax(got, axis=1)[:1]) == list(g["tied_greedy"][:1])
