"""The Q4_0 matvec on the integer tensor-core MMA (efg_matvec_mma.cu), taken for Q4_0
matrices of 48 MB and more with 2048 <= cols <= 8192, cols % 256 == 0: every row within
1e-5 of sum|w x| of the exact dot (test_qinfer.cpp:58-67), at config 4's row length and at
ragged shapes, with the residual-add epilogue, the plain-FP32 path for non-finite or
out-of-range x, and the CUDA-core kernel for an x it cannot read as float4."""
from __future__ import annotations

import pytest
from conftest import rel_dot_errors

import edgeforge_b200 as efg
from edgeforge_b200 import QType

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _weights(torch, rows, cols, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    W = torch.empty(rows * cols // 32 * 18, dtype=torch.uint8, device="cuda")
    for r0 in range(0, rows, 8192):  # bounded FP32 temporaries
        n = min(8192, rows - r0)
        X = torch.randn(n, cols, generator=g, device="cuda") * 0.02
        efg.quantize_rows(QType.Q4_0, X, n, cols, W[r0 * cols // 32 * 18:], True)
    return W


def _check(oracle, W, x, rows, y):
    err = rel_dot_errors(oracle, QType.Q4_0, W.cpu().numpy(), x.cpu().numpy(), rows, y.cpu().numpy())
    assert err.max() <= TOL, err.max()


@pytest.mark.parametrize("rows,cols", [(16384, 8192), (17411, 5632), (49157, 2048), (12301, 7936)])
def test_mma_path_rows(cuda, oracle, rows, cols):
    """Config 4's row length, three segments with a short last one, single-segment rows,
    ragged last tiles and a last segment of 56 blocks."""
    import torch

    W = _weights(torch, rows, cols, 1)
    x = torch.randn(cols, generator=torch.Generator(device="cuda").manual_seed(2), device="cuda") * 3
    y = torch.full((rows,), float("nan"), device="cuda")
    efg.matvec_q4_0(y, W, x, rows, cols)
    torch.cuda.synchronize()
    _check(oracle, W, x, rows, y)
    y2 = torch.empty_like(y)
    efg.matvec_q4_0(y2, W, x, rows, cols)
    torch.cuda.synchronize()
    assert torch.equal(y, y2)  # the group sums are added in a fixed order
    assert efg.device_error() == 0


def test_mma_path_jobs(cuda, oracle):
    """matvec_jobs with two Q4_0 jobs of 27 MB each (54 MB together): both on the MMA path."""
    import torch

    rows, cols = 6000, 8192
    Wa, Wb = _weights(torch, rows, cols, 3), _weights(torch, rows, cols, 4)
    x = torch.randn(cols, device="cuda")
    ya, yb = torch.empty(rows, device="cuda"), torch.empty(rows, device="cuda")
    efg.matvec_jobs([(ya, QType.Q4_0, Wa, rows, cols, x), (yb, QType.Q4_0, Wb, rows, cols, x)])
    torch.cuda.synchronize()
    _check(oracle, Wa, x, rows, ya)
    _check(oracle, Wb, x, rows, yb)


@pytest.mark.parametrize("scale", [1e-33, 1e-22, 1e-19, 1e31])
def test_mma_path_x_range(cuda, oracle, scale):
    """x scaled to block maxima near 2^-110, 2^-73 (FP32 path), 2^-63 (MMA path) and 2^103
    (FP32 path): every row within the tolerance either way."""
    import torch

    rows, cols = 24576, 2048  # 56.6 MB
    W = _weights(torch, rows, cols, 5)
    x = torch.randn(cols, generator=torch.Generator(device="cuda").manual_seed(6), device="cuda") * scale
    y = torch.empty(rows, device="cuda")
    efg.matvec_q4_0(y, W, x, rows, cols)
    torch.cuda.synchronize()
    _check(oracle, W, x, rows, y)
    assert efg.device_error() == 0


def test_mma_path_nan_x(cuda):
    import torch

    rows, cols = 24576, 2048
    W = _weights(torch, rows, cols, 7)
    x = torch.randn(cols, device="cuda")
    x[100] = float("nan")
    y = torch.empty(rows, device="cuda")
    efg.matvec_q4_0(y, W, x, rows, cols)
    torch.cuda.synchronize()
    assert torch.isnan(y).all()  # every row meets the NaN: (c - 8) * d * NaN
    assert efg.device_error() == 0


def test_switch_to_cuda_cores(cuda, oracle):
    """efg_set_q4_mma(0) sends the same call to the CUDA-core kernel: same tolerance, and
    the two kernels agree to rounding."""
    import torch

    rows, cols = 16384, 8192
    W = _weights(torch, rows, cols, 9)
    x = torch.randn(cols, device="cuda")
    y_mma, y_cc = torch.empty(rows, device="cuda"), torch.empty(rows, device="cuda")
    efg.matvec_q4_0(y_mma, W, x, rows, cols)
    assert efg.set_q4_mma(False) is True
    try:
        efg.matvec_q4_0(y_cc, W, x, rows, cols)
    finally:
        assert efg.set_q4_mma(True) is False
    torch.cuda.synchronize()
    _check(oracle, W, x, rows, y_cc)
    _check(oracle, W, x, rows, y_mma)
    assert not torch.equal(y_mma, y_cc)  # different arithmetic, so the switch took effect


def test_unaligned_x_takes_the_other_kernel(cuda, oracle):
    """x at a 4-byte offset cannot be read as float4: the CUDA-core kernel runs instead."""
    import torch

    rows, cols = 24576, 2048
    W = _weights(torch, rows, cols, 8)
    buf = torch.randn(cols + 1, device="cuda")
    x = buf[1:]
    y = torch.empty(rows, device="cuda")
    efg.matvec_q4_0(y, W, x, rows, cols)
    torch.cuda.synchronize()
    _check(oracle, W, x, rows, y)


def test_config4_full_shape(cuda, oracle):
    """Config 4's whole matrix on one GPU: Q4_0 131072 x 8192 (604 MB) drawn N(0, 0.02) and
    quantized on the device, x ~ N(0, 1); every one of the 131072 rows within 1e-5 of
    sum|w x| of the exact dot of the reference's kern::matvec (src/qkernels.cpp:275-297),
    and two calls give the same bits."""
    import torch

    rows, cols = 131072, 8192
    W = _weights(torch, rows, cols, 100)
    x = torch.randn(cols, generator=torch.Generator(device="cuda").manual_seed(5), device="cuda")
    y = torch.full((rows,), float("nan"), device="cuda")
    efg.matvec_q4_0(y, W, x, rows, cols)
    y2 = torch.empty_like(y)
    efg.matvec_q4_0(y2, W, x, rows, cols)
    torch.cuda.synchronize()
    assert torch.equal(y, y2)
    _check(oracle, W, x, rows, y)
    assert efg.device_error() == 0
