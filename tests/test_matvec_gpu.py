"""Packed Q4_0/Q8_0 matvec on the GPU against the CPU oracle, through the C ABI.

Tolerance: the reference's own metric, |y - exact| / sum_i |w_i x_i| <= 1e-5 per row
(tests/test_qinfer.cpp:58-67, eval_quant.cpp:31), where exact is the double-precision
dot of the dequantized row. The oracle's scalar kernel is checked against the same
bound and against the GPU result (their difference is summation order only).
"""
from __future__ import annotations

import numpy as np
import pytest
from conftest import golden, rel_dot_errors

from oracle.oracle import BF16, F16, F32, Q4_0, Q8_0, row_bytes

pytestmark = pytest.mark.gpu
TOL = 1e-5


def dev(a, cuda):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def run_matvec(efg, cuda, qt, W: np.ndarray, x: np.ndarray, rows: int, offset: int = 0) -> np.ndarray:
    import torch

    Wf = np.ascontiguousarray(W).reshape(-1)
    if offset:
        # place W at a byte offset to force the generic (unaligned) path
        buf = torch.zeros(Wf.size + 64, dtype=torch.uint8, device=cuda)
        buf[offset:offset + Wf.size] = dev(Wf, cuda)
        dW = buf[offset:offset + Wf.size]
    else:
        dW = dev(Wf, cuda)
    dx = dev(x.astype(np.float32), cuda)
    dy = torch.full((max(rows, 1),), float("nan"), dtype=torch.float32, device=cuda)
    efg.matvec(qt, dy, dW, dx, rows, x.size)
    torch.cuda.synchronize()
    return dy.cpu().numpy()[:rows]


def random_packed(qt, rows, cols, rng):
    rb = row_bytes(qt, cols)
    v = rng.integers(0, 256, rows * rb, dtype=np.uint8).reshape(-1, 18 if qt == Q4_0 else 34)
    h = rng.uniform(-0.05, 0.05, v.shape[0]).astype(np.float16).view(np.uint16)
    v[:, 0] = (h & 0xFF).astype(np.uint8)
    v[:, 1] = (h >> 8).astype(np.uint8)
    return v.reshape(rows, rb)


@pytest.mark.parametrize("n", [32, 64, 96, 2048, 5632])
@pytest.mark.parametrize("qt", [Q4_0, Q8_0])
def test_matvec_golden_vectors(efg_lib, cuda, oracle, n, qt):
    g = golden("matvec.npz")
    name = "q4" if qt == Q4_0 else "q8"
    W, x = g[f"{name}_W_{n}"], g[f"x_{n}"]
    y = run_matvec(efg_lib, cuda, qt, W, x, 24)
    assert rel_dot_errors(oracle, qt, W, x, 24, y).max() < TOL
    ys = g[f"{name}_y_scalar_{n}"]  # the reference's scalar kernel
    mag = oracle.exact_dots(qt, W, x, 24)[1]
    assert (np.abs(y.astype(np.float64) - ys) / np.maximum(mag, 1e-30)).max() < 2 * TOL


def test_hand_blocks_exact(efg_lib, cuda, oracle):
    """test_qinfer.cpp:100-122: exact results on hand-written blocks."""
    one = oracle.f32_to_fp16(1.0)
    blk = np.zeros(18 * 2, np.uint8)  # two blocks (64 columns: the fast path)
    blk[0], blk[1] = one & 0xFF, one >> 8
    blk[2:18] = 0x88
    blk[2 + 3] = 0x0F
    blk[18], blk[19] = one & 0xFF, one >> 8
    blk[20:36] = 0x88
    x = np.zeros(64, np.float32)
    x[3], x[19] = 2.0, 0.5
    assert run_matvec(efg_lib, cuda, Q4_0, blk, x, 1)[0] == 10.0
    assert run_matvec(efg_lib, cuda, Q4_0, blk[:18], x[:32], 1)[0] == 10.0  # generic path
    blk[0] = blk[1] = 0
    assert run_matvec(efg_lib, cuda, Q4_0, blk, x, 1)[0] == 0.0
    b8 = np.zeros(68, np.uint8)
    for o in (0, 34):
        b8[o], b8[o + 1] = one & 0xFF, one >> 8
        b8[o + 2] = np.uint8(256 - 127)
        b8[o + 2 + 31] = 127
    x[:] = 1.0
    assert run_matvec(efg_lib, cuda, Q8_0, b8, x, 1)[0] == 0.0
    b8[2 + 5] = 3
    assert run_matvec(efg_lib, cuda, Q8_0, b8, x, 1)[0] == 3.0


@pytest.mark.parametrize("qt", [Q4_0, Q8_0])
@pytest.mark.parametrize("rows,cols", [(1, 64), (3, 128), (37, 192), (300, 256), (5, 320), (129, 1024),
                                       (7, 96), (11, 32), (1000, 4096), (33, 8192), (2, 11264)])
def test_matvec_shapes(efg_lib, cuda, oracle, qt, rows, cols):
    rng = np.random.default_rng(rows * 7919 + cols)
    W = random_packed(qt, rows, cols, rng)
    x = rng.standard_normal(cols).astype(np.float32) * np.where(rng.standard_normal(cols) > 2, 30, 1).astype(np.float32)
    y = run_matvec(efg_lib, cuda, qt, W, x, rows)
    assert rel_dot_errors(oracle, qt, W, x, rows, y).max() < TOL


@pytest.mark.parametrize("qt", [Q4_0, Q8_0])
def test_unaligned_weights_take_the_generic_path(efg_lib, cuda, oracle, qt):
    rng = np.random.default_rng(5)
    W = random_packed(qt, 40, 256, rng)
    x = rng.standard_normal(256).astype(np.float32)
    for off in (2, 6, 8):
        y = run_matvec(efg_lib, cuda, qt, W, x, 40, offset=off)
        assert rel_dot_errors(oracle, qt, W, x, 40, y).max() < TOL


def test_empty_and_zero_width(efg_lib, cuda):
    import torch

    y = torch.full((4,), 5.0, device=cuda)
    efg_lib.matvec(Q4_0, y, torch.zeros(1, dtype=torch.uint8, device=cuda), torch.zeros(1, device=cuda), 0, 64)
    torch.cuda.synchronize()
    assert y.cpu().tolist() == [5.0] * 4  # rows == 0: nothing written
    efg_lib.matvec(Q4_0, y, torch.zeros(1, dtype=torch.uint8, device=cuda), torch.zeros(1, device=cuda), 4, 0)
    torch.cuda.synchronize()
    assert y.cpu().tolist() == [0.0] * 4  # zero blocks: every dot is 0


def test_bad_row_length_raises_like_the_reference(efg_lib, cuda):
    import torch

    t = torch.zeros(64, device=cuda)
    with pytest.raises(efg_lib.EdgeForgeError, match="Q4_0 needs a row length divisible by 32, got 30"):
        efg_lib.matvec_q4_0(t, t, t, 1, 30)


def test_deterministic_and_jobs_equal_single_calls(efg_lib, cuda, oracle):
    """matvec_jobs computes each job exactly like matvec (qkernels.h:68-69), and results
    do not change between calls."""
    import torch

    rng = np.random.default_rng(9)
    x = dev(rng.standard_normal(2048).astype(np.float32), cuda)
    mats = [dev(random_packed(Q4_0, r, 2048, rng), cuda) for r in (2048, 256, 256)]
    ys = [torch.empty(r, device=cuda) for r in (2048, 256, 256)]
    efg_lib.matvec_jobs([(y, Q4_0, W, y.numel(), 2048, x) for y, W in zip(ys, mats)])
    singles = []
    for W, y in zip(mats, ys):
        s = torch.empty_like(y)
        efg_lib.matvec_q4_0(s, W, x, y.numel(), 2048)
        singles.append(s)
    torch.cuda.synchronize()
    for a, b in zip(ys, singles):
        assert torch.equal(a.view(torch.int32), b.view(torch.int32))
    again = torch.empty_like(ys[0])
    efg_lib.matvec_q4_0(again, mats[0], x, 2048, 2048)
    torch.cuda.synchronize()
    assert torch.equal(again.view(torch.int32), ys[0].view(torch.int32))
    assert efg_lib.device_error() == 0


@pytest.mark.parametrize("cfg", ["c0_q4_5632x2048", "c1_q8_32000x2048", "down_q4_2048x5632"])
def test_config_shapes_quantized_gaussian(efg_lib, cuda, oracle, cfg):
    """Benchmark configs 0/1 (and the down_proj shape of config 3): W ~ N(0, 0.02)
    quantized by the reference algorithm, x ~ N(0, 1)."""
    qt, rows, cols = {"c0_q4_5632x2048": (Q4_0, 5632, 2048), "c1_q8_32000x2048": (Q8_0, 32000, 2048),
                      "down_q4_2048x5632": (Q4_0, 2048, 5632)}[cfg]
    rng = np.random.default_rng(0)
    X = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    W = oracle.quantize_rows(qt, X, search=True)
    x = rng.standard_normal(cols).astype(np.float32)
    y = run_matvec(efg_lib, cuda, qt, W, x, rows)
    assert rel_dot_errors(oracle, qt, W, x, rows, y).max() < TOL
    yo = oracle.matvec_mt(qt, W, x, rows)
    assert np.abs(y - yo).max() <= 1e-5 * np.abs(yo).max() * 10


def test_host_pointer_matvec_registered_and_fresh_weights(efg_lib, cuda, oracle):
    """Registered weights stay resident (views inside the range included); an unregistered
    buffer is read anew on every call, so rewriting it between calls is safe."""
    rng = np.random.default_rng(3)
    W = random_packed(Q8_0, 500, 2048, rng)
    efg_lib.host_register_weights(W)
    rb = row_bytes(Q8_0, 2048)
    for _ in range(3):
        x = rng.standard_normal(2048).astype(np.float32)
        y = efg_lib.host_matvec(Q8_0, W, x, 500)
        assert rel_dot_errors(oracle, Q8_0, W, x, 500, y).max() < TOL
        sub = W[100:140]  # a view inside the registered range
        ys = efg_lib.host_matvec(Q8_0, sub, x, 40)
        assert np.array_equal(ys.view(np.uint32), y[100:140].view(np.uint32))
    efg_lib.host_unregister_weights(W)
    U = random_packed(Q4_0, 64, 256, rng)
    x = rng.standard_normal(256).astype(np.float32)
    y1 = efg_lib.host_matvec(Q4_0, U, x, 64)
    U[:, 0:2] = 0  # zero every first-block scale in place
    y2 = efg_lib.host_matvec(Q4_0, U, x, 64)
    assert rel_dot_errors(oracle, Q4_0, U, x, 64, y2).max() < TOL
    assert not np.array_equal(y1, y2)
    efg_lib.host_release_weights()
    _ = rb


def test_reference_cpp_cases_through_the_shim(efg_lib, cuda, tmp_path):
    """Reference test cases written against the reference's C++ API (ef::kern::matvec_q4_0,
    ef::quantize_row, ...) compile unchanged against include/efg_ref_shim.hpp and pass on
    the GPU (tests/shim/shim_test.cpp)."""
    import subprocess
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent
    exe = tmp_path / "shim_test"
    subprocess.run(["g++", "-std=c++20", "-O2", "-I", str(root / "include"), str(root / "tests" / "shim" / "shim_test.cpp"),
                    "-L", str(root / "edgeforge_b200"), "-lefg", f"-Wl,-rpath,{root / 'edgeforge_b200'}", "-o", str(exe)],
                   check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failures" in r.stdout


def test_host_matvec_pinned_buffers_reused(efg_lib, cuda, oracle):
    """Repeated host calls with the same page-locked x and y buffers (y then written by the
    kernel's own stores) read the current x every time and overwrite all of y, for registered
    weights, views inside them and, after unregistering, weights read from host memory."""
    import torch

    rng = np.random.default_rng(5)
    W = random_packed(Q8_0, 700, 2048, rng)
    efg_lib.host_register_weights(W)
    x = torch.empty(2048, dtype=torch.float32).pin_memory().numpy()
    y = torch.empty(700, dtype=torch.float32).pin_memory().numpy()
    sub = W[200:300]
    ys = torch.empty(100, dtype=torch.float32).pin_memory().numpy()
    for _ in range(4):
        x[:] = rng.standard_normal(2048).astype(np.float32)
        y[:] = np.nan
        efg_lib.host_matvec(Q8_0, W, x, 700, y=y)
        assert rel_dot_errors(oracle, Q8_0, W, x, 700, y).max() < TOL
        efg_lib.host_matvec(Q8_0, sub, x, 100, y=ys)
        assert np.array_equal(ys.view(np.uint32), y[200:300].view(np.uint32))
    efg_lib.host_unregister_weights(W)
    W[:, 0:2] = 0  # first-block scales zeroed: now read from host memory on every call
    efg_lib.host_matvec(Q8_0, W, x, 700, y=y)
    assert rel_dot_errors(oracle, Q8_0, W, x, 700, y).max() < TOL
    efg_lib.host_release_weights()
    assert efg_lib.device_error() == 0


@pytest.mark.parametrize("n", [32, 64, 96, 2048, 5632])
@pytest.mark.parametrize("qt", [Q4_0, Q8_0])
def test_dot_golden_vectors(efg_lib, cuda, oracle, n, qt):
    """efg_dot_q4_0 / efg_dot_q8_0 (kern::dot_q4_0 / dot_q8_0, include/ef/qkernels.h:47-48)
    on each golden row: within 1e-5 of sum|w x|, and equal to the matvec's row result."""
    import torch

    g = golden("matvec.npz")
    name = "q4" if qt == Q4_0 else "q8"
    W, x = g[f"{name}_W_{n}"], g[f"x_{n}"]
    y = run_matvec(efg_lib, cuda, qt, W, x, 24)
    dx = dev(x.astype(np.float32), cuda)
    out = torch.full((1,), float("nan"), device=cuda)
    fn = efg_lib.dot_q4_0 if qt == Q4_0 else efg_lib.dot_q8_0
    for r in range(W.shape[0]):
        fn(out, dev(W[r], cuda), dx, n)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert rel_dot_errors(oracle, qt, W[r:r + 1], x, 1, got).max() < TOL
        assert got[0] == y[r]


def test_dot_hand_blocks(efg_lib, cuda):
    """Hand-built blocks of the reference's tests (test_qinfer.cpp:100-122): exact answers."""
    import torch

    x = np.ones(32, np.float32)
    q8 = np.zeros(34, np.uint8)
    q8[0:2] = np.frombuffer(np.float16(1.0).tobytes(), np.uint8)
    q8[2:34] = np.array([127, 256 - 127] * 16, np.uint8)  # +-127 cancel
    out = torch.full((1,), float("nan"), device=cuda)
    efg_lib.dot_q8_0(out, dev(q8, cuda), dev(x, cuda), 32)
    torch.cuda.synchronize()
    assert out.item() == 0.0
    q8[2:34] = 0
    q8[2] = 3  # a single code 3 with d = 1
    efg_lib.dot_q8_0(out, dev(q8, cuda), dev(x, cuda), 32)
    torch.cuda.synchronize()
    assert out.item() == 3.0
    q4 = np.zeros(18, np.uint8)
    q4[0:2] = np.frombuffer(np.float16(0.5).tobytes(), np.uint8)
    q4[2:18] = 0x88  # every code 8 -> weight 0
    q4[2] = 0x8A     # code 10 at column 0 -> 2 * 0.5
    efg_lib.dot_q4_0(out, dev(q4, cuda), dev(x, cuda), 32)
    torch.cuda.synchronize()
    assert out.item() == 1.0
    efg_lib.dot_q4_0(out, dev(q4, cuda), dev(x, cuda), 0)  # n = 0: a sum over no blocks is 0
    torch.cuda.synchronize()
    assert out.item() == 0.0


def _plain_rows(qt, X):
    """[rows][cols] float32 -> the plain storage bytes (F32 bits, F16 and BF16 rounded to nearest even)."""
    from edgeforge_b200.synthetic import bf16_bits

    if qt == F32:
        return np.ascontiguousarray(X, np.float32).view(np.uint8).reshape(X.shape[0], -1)
    if qt == F16:
        return X.astype(np.float16).view(np.uint8).reshape(X.shape[0], -1)
    return bf16_bits(X).view(np.uint8).reshape(X.shape[0], -1)


@pytest.mark.parametrize("qt", [F32, F16, BF16])
@pytest.mark.parametrize("rows,cols,offset", [(257, 2048, 0), (100, 96, 0), (33, 1003, 0), (64, 2048, 2), (5, 0, 0)])
def test_plain_type_matvec(efg_lib, cuda, oracle, qt, rows, cols, offset):
    """kern::matvec for F32 / F16 / BF16 views (src/qkernels.cpp:237-269): every row within 1e-5
    of sum|w x| of the exact dot; ragged lengths and a misaligned W take the scalar loads."""
    rng = np.random.default_rng(51 + rows + cols)
    X = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    W = _plain_rows(qt, X)
    x = rng.standard_normal(cols).astype(np.float32)
    y = run_matvec(efg_lib, cuda, qt, W, x, rows, offset)
    if cols == 0:
        assert (y == 0).all()
        return
    assert rel_dot_errors(oracle, qt, W, x, rows, y).max() < TOL


def test_tied_bf16_lm_head_shape(efg_lib, cuda, oracle):
    """A tied lm_head: the BF16 32000 x 2048 embedding as the matrix (src/model.cpp:88, 273), and
    the same product through matvec_jobs next to a Q8_0 job."""
    import torch

    rng = np.random.default_rng(61)
    rows, cols = 32000, 2048
    W = _plain_rows(BF16, (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32))
    x = rng.standard_normal(cols).astype(np.float32)
    y = run_matvec(efg_lib, cuda, BF16, W, x, rows)
    assert rel_dot_errors(oracle, BF16, W, x, rows, y).max() < TOL
    Wq = random_packed(Q8_0, 64, cols, rng)
    dW, dWq, dx = dev(W.reshape(-1), cuda), dev(Wq.reshape(-1), cuda), dev(x, cuda)
    y1, y2 = torch.empty(rows, device=cuda), torch.empty(64, device=cuda)
    efg_lib.matvec_jobs([(y1, BF16, dW, rows, cols, dx), (y2, Q8_0, dWq, 64, cols, dx)])
    torch.cuda.synchronize()
    assert np.array_equal(y1.cpu().numpy(), y)
    assert rel_dot_errors(oracle, Q8_0, Wq, x, 64, y2.cpu().numpy()).max() < TOL
