"""Batched Q4_0 / Q8_0 GEMM on the tensor cores (efg_gemm_q4_0, efg_gemm_q8_0, efg_gemm_jobs)
against the reference's per-column matvec semantics: every output column within 1e-5 of
sum|w x| of the exact (float64) dot of the dequantized weights with that column (the
reference's own check, test_qinfer.cpp:58-67), at benchmark config 3's shapes, the lm_head
shape and ragged ones; multi-matrix launches and the residual-add epilogue."""
from __future__ import annotations

import numpy as np
import pytest

import edgeforge_b200 as efg
from edgeforge_b200 import QType

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _weights(torch, M, K, seed, qt=QType.Q4_0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    W = torch.empty(M * (K // 32) * (18 if qt == QType.Q4_0 else 34), dtype=torch.uint8, device="cuda")
    if M * K:
        X = torch.randn(M, K, generator=g, device="cuda") * 0.02
        efg.quantize_rows(qt, X, M, K, W, True)
    return W


def _exact(oracle, W, X, K, qt=QType.Q4_0):
    """(exact, sum|w x|) for every (column, row), in float64."""
    Wd = oracle.dequantize_rows(qt, W.cpu().numpy(), K).astype(np.float64)
    Xd = X.cpu().numpy().astype(np.float64)
    return Xd @ Wd.T, np.abs(Xd) @ np.abs(Wd).T


def _rel_errors(oracle, W, X, Y, M, K):
    """|Y - exact| / sum|w x| for every (column, row)."""
    exact, mag = _exact(oracle, W, X, K)
    return np.abs(Y.cpu().numpy().astype(np.float64) - exact) / np.maximum(mag, 1e-30)


@pytest.mark.parametrize("M,K", [(5632, 2048), (2048, 5632)])
@pytest.mark.parametrize("B", [1, 16, 64, 256])
def test_config3_shapes(cuda, oracle, M, K, B):
    import torch

    W = _weights(torch, M, K, 1)
    X = torch.randn(B, K, generator=torch.Generator(device="cuda").manual_seed(2), device="cuda")
    Y = torch.full((B, M), float("nan"), device="cuda")
    efg.gemm_q4_0(Y, W, X, M, K, B)
    torch.cuda.synchronize()
    exact, mag = _exact(oracle, W, X, K)
    err = np.abs(Y.cpu().numpy().astype(np.float64) - exact) / mag
    assert err.max() <= TOL, err.max()
    # the same columns through the per-column matvec (the reference's formulation)
    y = torch.empty(M, device="cuda")
    for b in {0, B - 1}:
        efg.matvec_q4_0(y, W, X[b].contiguous(), M, K)
        torch.cuda.synchronize()
        diff = np.abs(y.cpu().numpy().astype(np.float64) - Y[b].cpu().numpy())
        assert (diff / mag[b]).max() <= 2 * TOL
    assert efg.device_error() == 0


@pytest.mark.parametrize("M,K,B", [(1000, 2048, 5), (130, 96, 17), (77, 32, 300), (129, 160, 16), (4096, 8192, 33)])
def test_ragged_shapes(cuda, oracle, M, K, B):
    import torch

    W = _weights(torch, M, K, 3)
    X = torch.randn(B, K, generator=torch.Generator(device="cuda").manual_seed(4), device="cuda") * 3
    Y = torch.full((B, M), float("nan"), device="cuda")
    efg.gemm_q4_0(Y, W, X, M, K, B)
    torch.cuda.synchronize()
    assert _rel_errors(oracle, W, X, Y, M, K).max() <= TOL
    Y2 = torch.empty_like(Y)
    efg.gemm_q4_0(Y2, W, X, M, K, B)
    torch.cuda.synchronize()
    assert torch.equal(Y, Y2)  # deterministic: fixed tiling, no atomics


def test_edges_and_errors(cuda):
    import torch

    W = _weights(torch, 64, 64, 5)
    X = torch.randn(4, 64, device="cuda")
    Y = torch.full((4, 64), 7.0, device="cuda")
    efg.gemm_q4_0(Y, W, X, 64, 0, 4)  # K = 0: every dot is empty
    torch.cuda.synchronize()
    assert torch.count_nonzero(Y).item() == 0
    efg.gemm_q4_0(Y, W, X, 0, 64, 4)  # nothing to do
    efg.gemm_q4_0(Y, W, X, 64, 64, 0)
    with pytest.raises(efg.EdgeForgeError, match="divisible by 32"):
        efg.gemm_q4_0(Y, W, X, 64, 48, 4)
    Xbig = torch.randn(4 * 64 + 1, device="cuda")
    with pytest.raises(efg.EdgeForgeError, match="aligned"):
        efg.gemm_q4_0(Y, W, Xbig[1:], 64, 64, 4)
    assert efg.device_error() == 0


@pytest.mark.parametrize("M,K", [(5632, 2048), (2048, 5632), (32000, 2048), (1000, 768)])
@pytest.mark.parametrize("B", [1, 23, 64, 200])
def test_q8_0_shapes(cuda, oracle, M, K, B):
    """efg_gemm_q8_0: three exact BF16 terms per weight; every column within 1e-5 of the
    exact dot and of the per-column Q8_0 matvec (the lm_head and the Q8_0 projections)."""
    import torch

    W = _weights(torch, M, K, 6, QType.Q8_0)
    X = torch.randn(B, K, generator=torch.Generator(device="cuda").manual_seed(7), device="cuda") * 2
    Y = torch.full((B, M), float("nan"), device="cuda")
    efg.gemm_q8_0(Y, W, X, M, K, B)
    torch.cuda.synchronize()
    exact, mag = _exact(oracle, W, X, K, QType.Q8_0)
    err = np.abs(Y.cpu().numpy().astype(np.float64) - exact) / mag
    assert err.max() <= TOL, err.max()
    y = torch.empty(M, device="cuda")
    for b in {0, B - 1}:
        efg.matvec_q8_0(y, W, X[b].contiguous(), M, K)
        torch.cuda.synchronize()
        diff = np.abs(y.cpu().numpy().astype(np.float64) - Y[b].cpu().numpy())
        assert (diff / mag[b]).max() <= 2 * TOL
    Y2 = torch.empty_like(Y)
    efg.gemm_q8_0(Y2, W, X, M, K, B)
    torch.cuda.synchronize()
    assert torch.equal(Y, Y2)
    assert efg.device_error() == 0


def test_q8_0_errors(cuda):
    import torch

    W = _weights(torch, 64, 512, 8, QType.Q8_0)
    X = torch.randn(4, 512, device="cuda")
    Y = torch.empty(4, 64, device="cuda")
    with pytest.raises(efg.EdgeForgeError, match="divisible by 256"):
        efg.gemm_q8_0(Y, W, X, 64, 480, 4)
    Xbig = torch.randn(4 * 512 + 1, device="cuda")
    with pytest.raises(efg.EdgeForgeError, match="aligned"):
        efg.gemm_q8_0(Y, W, Xbig[1:], 64, 512, 4)
    efg.gemm_q8_0(Y, W, X, 0, 512, 4)  # nothing to do
    assert efg.device_error() == 0


@pytest.mark.parametrize("qt", [QType.Q4_0, QType.Q8_0])
def test_jobs_and_accumulate(cuda, oracle, qt):
    """efg_gemm_jobs: q, k and v of TinyLlama's shape in one launch (each within 1e-5 of its
    exact product), and the residual-add epilogue bit-identical to adding the product after."""
    import torch

    K, B = 2048, 23
    Ms = [2048, 256, 256]
    Ws = [_weights(torch, M, K, 10 + i, qt) for i, M in enumerate(Ms)]
    X = torch.randn(B, K, generator=torch.Generator(device="cuda").manual_seed(11), device="cuda")
    Ys = [torch.full((B, M), float("nan"), device="cuda") for M in Ms]
    efg.gemm_jobs(qt, list(zip(Ws, Ys, Ms)), X, K, B)
    torch.cuda.synchronize()
    for W, Y, M in zip(Ws, Ys, Ms):
        exact, mag = _exact(oracle, W, X, K, qt)
        assert (np.abs(Y.cpu().numpy().astype(np.float64) - exact) / mag).max() <= TOL
    # accumulate: Y0 + product, the same launch shape (same split) without accumulate
    base = torch.randn(B, Ms[0], generator=torch.Generator(device="cuda").manual_seed(12), device="cuda")
    P = torch.empty_like(base)
    efg.gemm_jobs(qt, [(Ws[0], P, Ms[0])], X, K, B)
    Yacc = base.clone()
    efg.gemm_jobs(qt, [(Ws[0], Yacc, Ms[0])], X, K, B, accumulate=True)
    torch.cuda.synchronize()
    assert torch.equal(Yacc, base + P)
    assert efg.device_error() == 0


def test_jobs_errors(cuda):
    import torch

    W = _weights(torch, 256, 512, 13)
    X = torch.randn(4, 512, device="cuda")
    Y = torch.empty(4, 256, device="cuda")
    with pytest.raises(efg.EdgeForgeError, match="jobs"):
        efg.gemm_jobs(QType.Q4_0, [(W, Y, 256)] * 4, X, 512, 4)
    with pytest.raises(efg.EdgeForgeError, match="K = 480"):
        efg.gemm_jobs(QType.Q4_0, [(W, Y, 256)], X, 480, 4)
    with pytest.raises(efg.EdgeForgeError, match="jobs"):
        efg.gemm_jobs(2, [(W, Y, 256)], X, 512, 4)
    # empty cases, as efg_gemm_q4_0 has them: K = 0 zero-fills (or adds nothing), B = 0 and
    # zero-row jobs do nothing
    Y.fill_(5.0)
    efg.gemm_jobs(QType.Q4_0, [(W, Y, 256)], X, 0, 4, accumulate=True)
    efg.gemm_jobs(QType.Q4_0, [(W, Y, 256)], X, 512, 0)
    efg.gemm_jobs(QType.Q4_0, [(W, Y, 0)], X, 512, 4)
    torch.cuda.synchronize()
    assert bool((Y == 5.0).all())
    efg.gemm_jobs(QType.Q4_0, [(W, Y, 256)], X, 0, 4)
    torch.cuda.synchronize()
    assert torch.count_nonzero(Y).item() == 0
    assert efg.device_error() == 0


@pytest.mark.parametrize("M,K,B", [(5632, 2048, 23), (2048, 5632, 8), (2560, 2048, 64), (300, 4096, 65)])
def test_small_batch_path_and_switch(cuda, oracle, M, K, B):
    """With efg_set_small_gemm(1), B <= 64 runs on the small-batch integer-MMA kernel (X columns as
    the A operand) and B = 65 stays on the tcgen05 kernel; the default is the tcgen05 kernel for
    every B. Both within 1e-5 of sum|w x|, each deterministic."""
    import torch

    W = _weights(torch, M, K, 21)
    X = torch.randn(B, K, generator=torch.Generator(device="cuda").manual_seed(22), device="cuda") * 2
    Ys = []
    for small in (True, False):
        old = efg.set_small_gemm(small)
        try:
            Y = torch.full((B, M), float("nan"), device="cuda")
            efg.gemm_q4_0(Y, W, X, M, K, B)
            Y2 = torch.empty_like(Y)
            efg.gemm_q4_0(Y2, W, X, M, K, B)
            torch.cuda.synchronize()
        finally:
            efg.set_small_gemm(old)
        assert torch.equal(Y, Y2)
        assert _rel_errors(oracle, W, X, Y, M, K).max() <= TOL
        Ys.append(Y)
    assert torch.equal(Ys[0], Ys[1]) == (B > 64)  # the switch only matters where the paths differ
    assert efg.device_error() == 0


def test_small_batch_non_finite_columns(cuda, oracle):
    """On the small-batch kernel (efg_set_small_gemm(1)): a column of X with an infinity, one with a NaN and one with values beyond the fixed-point
    range come out as the FP32 matvec computes them (signed infinities stay infinities); the
    other columns keep the 1e-5 bound."""
    import torch

    M, K, B = 1000, 2048, 6
    old = efg.set_small_gemm(True)
    W = _weights(torch, M, K, 31)
    X = torch.randn(B, K, generator=torch.Generator(device="cuda").manual_seed(32), device="cuda")
    X[1, 77] = float("inf")
    X[3, 1500] = float("nan")
    X[4] *= 1e31
    Y = torch.full((B, M), 7.0, device="cuda")
    efg.gemm_q4_0(Y, W, X, M, K, B)
    torch.cuda.synchronize()
    y = torch.empty(M, device="cuda")
    for b in range(B):
        efg.matvec_q4_0(y, W, X[b].contiguous(), M, K)
        torch.cuda.synchronize()
        got, want = Y[b].cpu().numpy(), y.cpu().numpy()
        assert np.array_equal(np.isnan(got), np.isnan(want)), b
        assert np.array_equal(np.isinf(got), np.isinf(want)), b
        fin = np.isfinite(want)
        assert np.array_equal(np.sign(got[~fin & ~np.isnan(want)]), np.sign(want[~fin & ~np.isnan(want)]))
        if b in (0, 2, 4, 5):
            assert fin.all()
            assert _rel_errors(oracle, W, X[b:b + 1], Y[b:b + 1], M, K).max() <= TOL, b
    assert np.isinf(Y[1].cpu().numpy()).any()
    efg.set_small_gemm(old)
    assert efg.device_error() == 0
