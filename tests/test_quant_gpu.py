"""Q4_0 / Q8_0 quantize and dequantize on the GPU: bit-exact with the reference
(golden vectors made by the reference, and the oracle on config-1-size inputs)."""
from __future__ import annotations

import numpy as np
import pytest
from conftest import golden

from oracle.oracle import BF16, F16, F32, Q4_0, Q8_0, row_bytes

pytestmark = pytest.mark.gpu


def dev(a, cuda):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def gpu_quantize(efg, cuda, qt, X, search=True):
    import torch

    rows, cols = X.shape
    out = torch.zeros(rows * row_bytes(qt, cols), dtype=torch.uint8, device=cuda)
    efg.quantize_rows(qt, dev(X, cuda), rows, cols, out, search)
    torch.cuda.synchronize()
    return out.cpu().numpy().reshape(rows, -1)


def gpu_dequantize(efg, cuda, qt, Q, cols):
    import torch

    rows = Q.size // row_bytes(qt, cols)
    out = torch.zeros(rows * cols, dtype=torch.float32, device=cuda)
    efg.dequantize_rows(qt, dev(Q.reshape(-1), cuda), rows, cols, out)
    torch.cuda.synchronize()
    return out.cpu().numpy().reshape(rows, cols)


def bits(a):
    return np.asarray(a, dtype=np.float32).view(np.uint32)


def test_quantize_golden_bit_exact(efg_lib, cuda):
    g = golden("quant.npz")
    X = g["x"]
    assert np.array_equal(gpu_quantize(efg_lib, cuda, Q4_0, X, True), g["q4_search"])
    assert np.array_equal(gpu_quantize(efg_lib, cuda, Q4_0, X, False), g["q4_absmax"])
    assert np.array_equal(gpu_quantize(efg_lib, cuda, Q8_0, X), g["q8"])


def test_dequantize_golden_bit_exact(efg_lib, cuda):
    g = golden("quant.npz")
    assert np.array_equal(bits(gpu_dequantize(efg_lib, cuda, Q4_0, g["q4_search"], 256)), bits(g["q4_search_deq"]))
    assert np.array_equal(bits(gpu_dequantize(efg_lib, cuda, Q8_0, g["q8"], 256)), bits(g["q8_deq"]))


def test_fp16_scale_rounding_edges(efg_lib, cuda, oracle):
    """Blocks whose scales land on every fp16 regime: subnormal, normal, the 65504 clamp."""
    rng = np.random.default_rng(4)
    mags = 10.0 ** rng.uniform(-9, 7, 4096)
    X = (rng.standard_normal((4096, 32)) * mags[:, None]).astype(np.float32)
    for qt in (Q4_0, Q8_0):
        for search in (True, False):
            assert np.array_equal(gpu_quantize(efg_lib, cuda, qt, X, search), oracle.quantize_rows(qt, X, search))


def test_random_bit_patterns(efg_lib, cuda, oracle):
    """Arbitrary float bit patterns (NaN, inf, subnormal, huge) stay bit-exact."""
    rng = np.random.default_rng(5)
    X = rng.integers(0, 2**32, (1024, 64), dtype=np.uint64).astype(np.uint32).view(np.float32)
    for qt in (Q4_0, Q8_0):
        assert np.array_equal(gpu_quantize(efg_lib, cuda, qt, X), oracle.quantize_rows(qt, X))
    Q = rng.integers(0, 256, 1024 * 18, dtype=np.uint8)
    assert np.array_equal(bits(gpu_dequantize(efg_lib, cuda, Q4_0, Q, 1024)),
                          bits(oracle.dequantize_rows(Q4_0, Q, 1024)))


def test_config1_round_trip_bit_exact(efg_lib, cuda, oracle):
    """Benchmark config 1: the seeded 32000x2048 N(0, 0.02) matrix through Q4_0 and Q8_0
    quantize -> dequantize, bit-exact with quant.cpp."""
    rng = np.random.default_rng(1)
    X = (rng.standard_normal((32000, 2048)) * 0.02).astype(np.float32)
    for qt in (Q4_0, Q8_0):
        q = gpu_quantize(efg_lib, cuda, qt, X, True)
        assert np.array_equal(q, oracle.quantize_rows(qt, X, True))
        d = gpu_dequantize(efg_lib, cuda, qt, q, 2048)
        assert np.array_equal(bits(d), bits(oracle.dequantize_rows(qt, q, 2048)))
    # size-independent property: Q8_0 codes are a fixed point of quantize(dequantize(.))
    q8 = gpu_quantize(efg_lib, cuda, Q8_0, X)
    assert np.array_equal(gpu_quantize(efg_lib, cuda, Q8_0, gpu_dequantize(efg_lib, cuda, Q8_0, q8, 2048)), q8)


def test_row_f32_lookup(efg_lib, cuda, oracle):
    import torch

    rng = np.random.default_rng(6)
    X = rng.standard_normal((50, 96)).astype(np.float32)
    for qt in (F32, F16, BF16, Q8_0, Q4_0):
        W = np.concatenate([oracle.quantize_row(qt, r) for r in X])
        dW = dev(W, cuda)
        out = torch.zeros(96, device=cuda)
        efg_lib.row_f32(out, qt, dW, 50, 96, r=17)
        idx = torch.tensor([33], dtype=torch.int32, device=cuda)
        out2 = torch.zeros(96, device=cuda)
        efg_lib.row_f32(out2, qt, dW, 50, 96, r_dev=idx)
        torch.cuda.synchronize()
        rb = row_bytes(qt, 96)
        assert np.array_equal(bits(out.cpu().numpy()), bits(oracle.dequantize_row(qt, W[17 * rb:18 * rb], 96)))
        assert np.array_equal(bits(out2.cpu().numpy()), bits(oracle.dequantize_row(qt, W[33 * rb:34 * rb], 96)))
    assert efg_lib.device_error() == 0


def test_host_pointer_quantize_roundtrip(efg_lib, cuda, oracle):
    x = np.random.default_rng(8).standard_normal(4096).astype(np.float32)
    q = efg_lib.host_quantize_row(Q4_0, x)
    assert np.array_equal(q, oracle.quantize_row(Q4_0, x))
    assert np.array_equal(bits(efg_lib.host_dequantize_row(Q4_0, q, 4096)), bits(oracle.dequantize_row(Q4_0, q, 4096)))


def _edge_floats(rng, n):
    """Random bit patterns (NaN payloads, infinities, subnormals) plus values at the F16/BF16
    rounding and overflow edges."""
    v = rng.integers(0, 2**32, n, dtype=np.uint64).astype(np.uint32).view(np.float32)
    edges = np.array([0.0, -0.0, 65504, 65519.996, 65520, -65520, 2.0**-24, 2.0**-25, 3 * 2.0**-26, 2.0**-14,
                      np.inf, -np.inf, np.nan, 3.3895314e38, 1.0 + 2.0**-8, 1.0 + 3 * 2.0**-8], dtype=np.float32)
    return np.concatenate([v, edges, (rng.standard_normal(n) * 0.02).astype(np.float32)])


@pytest.mark.parametrize("qt", [F32, F16, BF16])
def test_plain_type_quantize_row_bit_exact(efg_lib, cuda, oracle, qt):
    """quantize_row for F32 / F16 / BF16 (src/quant.cpp:186-200) on the device: the bits of
    every value, NaN payloads included, equal the oracle's (itself pinned to the reference);
    an odd length and an odd byte offset of the output."""
    import torch

    rng = np.random.default_rng(41)
    x = _edge_floats(rng, 4001)
    want = oracle.quantize_row(qt, x)
    got = efg_lib.host_quantize_row(qt, x)
    np.testing.assert_array_equal(got, want)
    buf = torch.zeros(want.size + 8, dtype=torch.uint8, device=cuda)
    efg_lib.quantize_row(qt, dev(x, cuda), x.size, buf[3:3 + want.size])
    torch.cuda.synchronize()
    np.testing.assert_array_equal(buf.cpu().numpy()[3:3 + want.size], want)
    assert not buf.cpu().numpy()[:3].any() and not buf.cpu().numpy()[3 + want.size:].any()


@pytest.mark.parametrize("n", [32, 64, 100, 128, 256, 300])
def test_fake_quant_q4_group_bit_exact(efg_lib, cuda, oracle, n):
    """fake_quant_q4_group (src/quant.cpp:243-248) for groups of any size, with and without the
    scale search; a zero group, a non-finite one and a group of tiny values."""
    rng = np.random.default_rng(43 + n)
    groups = [(rng.standard_normal(n) * 0.02).astype(np.float32), np.zeros(n, np.float32),
              (rng.standard_normal(n) * 1e-9).astype(np.float32)]
    bad = groups[0].copy()
    bad[n // 2] = np.nan
    groups.append(bad)
    for x in groups:
        for search in (True, False):
            np.testing.assert_array_equal(bits(efg_lib.host_fake_quant_q4_group(x, search)),
                                          bits(oracle.fake_quant_q4_group(x, search)))
