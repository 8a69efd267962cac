"""Shared pytest setup: the `gpu` marker, the CPU checkers and the CUDA library.

Tests marked `gpu` need a B200; everything else runs on CPU. Missing in-tree builds
(the oracle libraries, libefg.so) are built on first use with the committed Makefiles.
"""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a)")


def _make(target_dir: Path, product: Path):
    if not product.exists():
        subprocess.run(["make", "-C", str(target_dir), "-j8"], check=True, capture_output=True)


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import ORACLE_SO, Oracle

    _make(ROOT / "oracle", ORACLE_SO)
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    """The reference implementation compiled from its own sources, if it was built."""
    from oracle.oracle import REF_SO, Reference, reference_tree

    tree = reference_tree()
    if not REF_SO.exists() and tree is not None:
        subprocess.run(["make", "-C", str(ROOT / "oracle"), "-j8", f"REF={tree}"], check=True, capture_output=True)
    if not REF_SO.exists():
        pytest.skip("oracle/_ref/libefref.so not built (reference sources absent)")
    return Reference()


@pytest.fixture(scope="session")
def efg_lib():
    import edgeforge_b200 as efg

    _make(ROOT / "edgeforge_b200" / "csrc", efg.LIB_PATH)
    efg.load()
    return efg


@pytest.fixture(scope="session")
def cuda(efg_lib):
    import torch

    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for a gpu-marked test")
    torch.cuda.init()
    return torch.device("cuda:0")


def golden(name: str):
    return np.load(GOLDEN / name)


def rel_dot_errors(oracle, qtype, W: np.ndarray, x: np.ndarray, rows: int, got: np.ndarray) -> np.ndarray:
    """|got - exact| / sum|w x| per row (tests/test_qinfer.cpp:58-67 in the reference)."""
    exact, mag = oracle.exact_dots(qtype, W, x, rows)
    return np.abs(got.astype(np.float64) - exact) / np.maximum(mag, 1e-30)


@pytest.fixture(scope="session")
def tinyllama():
    """A random TinyLlama-1.1B-shaped checkpoint (seed 0, BF16) and the reference's own .efq
    of it (quantize_model, policy auto = the TinyLlama recipe). Cached across sessions in
    $EFG_TEST_CACHE (default: the system temp directory). Returns (model_dir, efq_path)."""
    import os
    import tempfile

    from edgeforge_b200 import synthetic
    from oracle.oracle import REF_SO, Reference

    if not REF_SO.exists():
        pytest.fail("oracle/_ref/libefref.so is not built (make -C oracle)")
    d = Path(os.environ.get("EFG_TEST_CACHE", tempfile.gettempdir())) / "efg_tinyllama_seed0"
    efq = d / "model-auto.efq"
    if not efq.exists():
        synthetic.write_checkpoint(d, synthetic.TINYLLAMA, seed=0)
        part = d / "model-auto.efq.part"
        Reference().quantize_model(d, part, policy="auto")
        part.rename(efq)
    return d, efq
