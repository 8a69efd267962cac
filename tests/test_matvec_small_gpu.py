"""The Q4_0 matvec for small matrices (efg_matvec_mma.cu, matvec_q4_small_kernel): the decode-
step shapes, where each CTA fetches all of its rows at once and the next launch runs beside it.
Every row within 1e-5 of sum|w x| of the exact dot (test_qinfer.cpp:58-67), the same bits on
every call, agreement with the CUDA-core kernel to rounding, the multi-matrix launch, the
plain-FP32 path for x it cannot hold as fixed point, and back-to-back launches in a CUDA graph
with early weight streaming, where each launch reads the x the previous one wrote."""
from __future__ import annotations

import pytest
from conftest import rel_dot_errors

import edgeforge_b200 as efg
from edgeforge_b200 import QType

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _weights(torch, rows, cols, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    X = torch.randn(rows, cols, generator=g, device="cuda") * 0.02
    W = torch.empty(rows * cols // 32 * 18, dtype=torch.uint8, device="cuda")
    efg.quantize_rows(QType.Q4_0, X, rows, cols, W, True)
    return W


def _check(oracle, W, x, rows, y):
    err = rel_dot_errors(oracle, QType.Q4_0, W.cpu().numpy(), x.cpu().numpy(), rows, y.cpu().numpy())
    assert err.max() <= TOL, err.max()


# TinyLlama's gate/up (config 0), down (three K segments, the last one short), q/o, k/v, a
# single unit of the longest rows, ragged last units, and a last segment of 56 blocks
SHAPES = [(5632, 2048), (2048, 5632), (2048, 2048), (256, 2048), (8, 8192), (1001, 2048), (100, 7936), (3, 4096)]


@pytest.mark.parametrize("rows,cols", SHAPES)
def test_small_kernel_rows(cuda, oracle, rows, cols):
    import torch

    W = _weights(torch, rows, cols, 1 + rows)
    x = torch.randn(cols, generator=torch.Generator(device="cuda").manual_seed(2), device="cuda") * 3
    y = torch.full((rows,), float("nan"), device="cuda")
    efg.matvec_q4_0(y, W, x, rows, cols)
    torch.cuda.synchronize()
    _check(oracle, W, x, rows, y)
    y2 = torch.empty_like(y)
    efg.matvec_q4_0(y2, W, x, rows, cols)
    y_cc = torch.empty_like(y)
    assert efg.set_q4_mma(False) is True
    try:
        efg.matvec_q4_0(y_cc, W, x, rows, cols)
    finally:
        efg.set_q4_mma(True)
    torch.cuda.synchronize()
    assert torch.equal(y, y2)  # warp partials added in a fixed order
    _check(oracle, W, x, rows, y_cc)
    assert efg.device_error() == 0


def test_small_kernel_jobs(cuda, oracle):
    """q, k and v of one layer in one launch (kern::matvec_jobs, src/model.cpp:230)."""
    import torch

    cols = 2048
    shapes = [2048, 256, 256]
    Ws = [_weights(torch, r, cols, 10 + i) for i, r in enumerate(shapes)]
    x = torch.randn(cols, device="cuda")
    ys = [torch.full((r,), float("nan"), device="cuda") for r in shapes]
    efg.matvec_jobs([(y, QType.Q4_0, W, r, cols, x) for y, W, r in zip(ys, Ws, shapes)])
    torch.cuda.synchronize()
    for y, W, r in zip(ys, Ws, shapes):
        _check(oracle, W, x, r, y)


@pytest.mark.parametrize("scale", [1e-33, 1e-22, 1e-19, 1e31])
def test_small_kernel_x_range(cuda, oracle, scale):
    """Block maxima near 2^-110, 2^-73 (FP32 path), 2^-63 (MMA path) and 2^103 (FP32 path)."""
    import torch

    rows, cols = 5632, 2048
    W = _weights(torch, rows, cols, 5)
    x = torch.randn(cols, generator=torch.Generator(device="cuda").manual_seed(6), device="cuda") * scale
    y = torch.empty(rows, device="cuda")
    efg.matvec_q4_0(y, W, x, rows, cols)
    torch.cuda.synchronize()
    _check(oracle, W, x, rows, y)
    assert efg.device_error() == 0


def test_small_kernel_nan_x(cuda):
    import torch

    rows, cols = 2048, 2048
    W = _weights(torch, rows, cols, 7)
    x = torch.randn(cols, device="cuda")
    x[1500] = float("nan")
    y = torch.empty(rows, device="cuda")
    efg.matvec_q4_0(y, W, x, rows, cols)
    torch.cuda.synchronize()
    assert torch.isnan(y).all()
    assert efg.device_error() == 0


def test_small_kernel_chained_in_a_graph(cuda, oracle):
    """A chain of square matvecs y_{i+1} = W_i y_i (W_i 2048 x 2048, rescaled so y stays O(1))
    launched back to back with weight prefetch on, as one CUDA graph: every launch reads the x
    its predecessor wrote, so the early weight streaming must not let x be read early."""
    import numpy as np
    import torch

    n, cols = 6, 2048
    Ws = [_weights(torch, cols, cols, 20 + i) for i in range(n)]
    ys = [torch.randn(cols, generator=torch.Generator(device="cuda").manual_seed(3), device="cuda")]
    ys += [torch.empty(cols, device="cuda") for _ in range(n)]
    old = efg.set_weight_prefetch(True)
    try:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
            for i in range(n):
                efg.matvec_q4_0(ys[i + 1], Ws[i], ys[i], cols, cols)
        for _ in range(3):
            for y in ys[1:]:
                y.fill_(float("nan"))
            torch.cuda.synchronize()
            g.replay()
            torch.cuda.synchronize()
            for i in range(n):
                assert not torch.isnan(ys[i + 1]).any()
                _check(oracle, Ws[i], ys[i], cols, ys[i + 1])
        del g
    finally:
        efg.set_weight_prefetch(old)
    assert np.isfinite(ys[-1].cpu().numpy()).all()
    assert efg.device_error() == 0
