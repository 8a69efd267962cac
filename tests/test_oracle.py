"""The CPU oracle pinned against the reference (CPU only).

Three anchors: the committed golden vectors produced by the reference
(tests/golden/*.npz), the reference's own known-answer tests restated here
(tests/test_quant.cpp, test_qinfer.cpp, test_fp16.cpp), and, when oracle/_ref is built,
the live reference on fresh seeded inputs.
"""
from __future__ import annotations

import numpy as np
import pytest
from conftest import golden, rel_dot_errors

from oracle.oracle import BF16, F16, F32, Q4_0, Q8_0, row_bytes


def bits(a):
    return np.asarray(a, dtype=np.float32).view(np.uint32)


# ---------------------------------------------------------------- fp16 (test_fp16.cpp)


def test_fp16_to_f32_all_65536_match_golden(oracle):
    g = golden("fp16.npz")
    got = np.array([oracle.fp16_to_f32(h) for h in range(65536)], dtype=np.float32)
    want = g["fp16_to_f32"]
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(bits(got)[~nan], bits(want)[~nan])
    # NaN payloads are kept (fp16.h:61): compare bits too
    assert np.array_equal(bits(got), bits(want))


def test_f32_to_fp16_matches_golden(oracle):
    g = golden("fp16.npz")
    got = np.array([oracle.f32_to_fp16(float(f)) for f in g["f32_samples"]], dtype=np.uint16)
    assert np.array_equal(got, g["f32_to_fp16"])


def test_fp16_known_values_and_roundtrip(oracle):
    # test_fp16.cpp: fp16_half_known_values / roundtrip_all_65536
    assert oracle.fp16_to_f32(0x3C00) == 1.0
    assert oracle.fp16_to_f32(0x7BFF) == 65504.0
    assert oracle.fp16_to_f32(0x0001) == 2.0**-24
    assert oracle.fp16_to_f32(0x03FF) == 1023 * 2.0**-24
    assert oracle.f32_to_fp16(65520.0) == 0x7C00  # >= 65520 -> inf
    assert oracle.f32_to_fp16(2.0**-25) == 0  # tie to even -> 0
    assert oracle.f32_to_fp16(3 * 2.0**-26) == 1
    bad = 0
    for h in range(65536):
        e, m = (h >> 10) & 31, h & 0x3FF
        back = oracle.f32_to_fp16(oracle.fp16_to_f32(h))
        if e == 31 and m:
            bad += not ((back >> 10) & 31 == 31 and back & 0x3FF)
        else:
            bad += back != h
    assert bad == 0
    assert oracle.f32_to_bf16(np.float32(1.0)) == 0x3F80
    assert oracle.bf16_to_f32(0xC000) == -2.0


# ---------------------------------------------------------------- blocks (test_quant.cpp)


def test_quantize_matches_reference_golden_bit_for_bit(oracle):
    g = golden("quant.npz")
    X = g["x"]
    assert np.array_equal(oracle.quantize_rows(Q4_0, X, search=True), g["q4_search"])
    assert np.array_equal(oracle.quantize_rows(Q4_0, X, search=False), g["q4_absmax"])
    assert np.array_equal(oracle.quantize_rows(Q8_0, X), g["q8"])
    assert np.array_equal(bits(oracle.dequantize_rows(Q4_0, g["q4_search"], 256)), bits(g["q4_search_deq"]))
    assert np.array_equal(bits(oracle.dequantize_rows(Q8_0, g["q8"], 256)), bits(g["q8_deq"]))


def test_q4_exact_on_grid_and_nibble_layout(oracle):
    # test_quant.cpp:52-69
    x = ((np.arange(32) % 16) - 8).astype(np.float32) * 0.25
    b = oracle.quantize_row(Q4_0, x)
    assert np.array_equal(oracle.dequantize_row(Q4_0, b, 32), x)
    m = np.zeros(18, np.uint8)
    h = oracle.f32_to_fp16(1.0)
    m[0], m[1] = h & 0xFF, h >> 8
    m[2] = 0x2F
    y = oracle.dequantize_row(Q4_0, m, 32)
    assert y[0] == 7.0 and y[16] == -6.0 and y[1] == -8.0
    z = oracle.quantize_row(Q4_0, np.zeros(32, np.float32))
    assert z[0] == 0 and z[1] == 0 and z[2] == 0x88
    assert oracle.dequantize_row(Q4_0, z, 32)[5] == 0.0


def test_q4_search_never_worse_and_absmax_within_one_step(oracle):
    # test_quant.cpp:71-100 (2,000 blocks here instead of 20,000)
    rng = np.random.default_rng(11)
    X = (rng.standard_normal((2000, 32)) * 0.02).astype(np.float32)
    for k in range(0, 2000, 7):
        X[k, k % 32] *= 6.0
    qs = oracle.quantize_rows(Q4_0, X, search=True)
    qp = oracle.quantize_rows(Q4_0, X, search=False)
    a = oracle.dequantize_rows(Q4_0, qs, 32).astype(np.float64)
    p = oracle.dequantize_rows(Q4_0, qp, 32).astype(np.float64)
    es = ((X - a) ** 2).sum(1)
    ep = ((X - p) ** 2).sum(1)
    assert (es > ep * (1 + 1e-12)).sum() == 0
    d = np.abs(qp[:, :2].copy().view(np.uint16)[:, 0].view(np.float16).astype(np.float32))
    assert (np.abs(X - p) > d[:, None] * 1.01).sum() == 0
    ref = (X.astype(np.float64) ** 2).sum()
    assert np.sqrt(es.sum() / ref) < np.sqrt(ep.sum() / ref) < 0.2


def test_q8_error_bound(oracle):
    # test_quant.cpp:102-123
    rng = np.random.default_rng(12)
    X = rng.standard_normal((5000, 32)).astype(np.float32)
    q = oracle.quantize_rows(Q8_0, X)
    y = oracle.dequantize_rows(Q8_0, q, 32)
    d = q[:, :2].copy().view(np.uint16)[:, 0].view(np.float16).astype(np.float32)
    assert (np.abs(X - y) > d[:, None] * 0.5001 + 1e-7).sum() == 0
    assert np.sqrt(((X - y).astype(np.float64) ** 2).sum() / (X.astype(np.float64) ** 2).sum()) < 0.01


def test_row_bytes_and_types(oracle):
    # test_quant.cpp:125-130
    from oracle.oracle import _Lib  # noqa: F401

    assert row_bytes(Q4_0, 2048) == 64 * 18
    assert row_bytes(Q8_0, 2048) == 64 * 34
    assert row_bytes(BF16, 2048) == 4096
    with pytest.raises(ValueError):
        row_bytes(Q4_0, 30)
    x = np.random.default_rng(13).standard_normal(256).astype(np.float32)
    for t in (F32, F16, BF16, Q8_0, Q4_0):
        y = oracle.dequantize_row(t, oracle.quantize_row(t, x), 256)
        e = np.abs(x - y).max()
        assert (t != F32 or e == 0.0) and e < 0.6


# ---------------------------------------------------------------- packed dots (test_qinfer.cpp)


@pytest.mark.parametrize("n", [32, 64, 96, 2048, 5632])
def test_scalar_matvec_matches_reference_golden(oracle, n):
    g = golden("matvec.npz")
    x = g[f"x_{n}"]
    for qt, name in ((Q4_0, "q4"), (Q8_0, "q8")):
        W = g[f"{name}_W_{n}"]
        y = oracle.matvec(qt, W, x, 24)
        assert np.array_equal(bits(y), bits(g[f"{name}_y_scalar_{n}"]))  # bit for bit
        for r in range(24):
            assert bits(oracle.dot(qt, W[r], x)) == bits(y[r])  # matvec = row dots
        assert rel_dot_errors(oracle, qt, W, x, 24, y).max() < 1e-5
        assert rel_dot_errors(oracle, qt, W, x, 24, g[f"{name}_y_avx2_{n}"]).max() < 1e-5


def test_packed_dot_layout_and_edge_codes(oracle):
    # test_qinfer.cpp:100-122
    blk = np.zeros(18, np.uint8)
    one = oracle.f32_to_fp16(1.0)
    blk[0], blk[1] = one & 0xFF, one >> 8
    blk[2:] = 0x88
    blk[2 + 3] = 0x0F
    x = np.zeros(32, np.float32)
    x[3], x[19] = 2.0, 0.5
    assert oracle.dot(Q4_0, blk, x) == 7.0 * 2.0 + -8.0 * 0.5
    blk[0] = blk[1] = 0
    assert oracle.dot(Q4_0, blk, x) == 0.0
    b8 = np.zeros(34, np.uint8)
    b8[0], b8[1] = one & 0xFF, one >> 8
    b8[2] = np.uint8(256 - 127)
    b8[2 + 31] = 127
    x[:] = 1.0
    assert oracle.dot(Q8_0, b8, x) == 0.0
    b8[2 + 5] = 3
    assert oracle.dot(Q8_0, b8, x) == 3.0


def test_threaded_matvec_is_bit_identical(oracle):
    # test_qinfer.cpp:227-263
    g = golden("matvec.npz")
    x, W = g["x_2048"], g["q4_W_2048"]
    ref = oracle.matvec(Q4_0, W, x, 24)
    for t in (2, 3, 5, 8):
        assert np.array_equal(bits(oracle.matvec_mt(Q4_0, W, x, 24, threads=t)), bits(ref))


# ---------------------------------------------------------------- decode ops (kernels.cpp)


def test_decode_ops_match_reference_golden(oracle):
    g = golden("decode_ops.npz")
    assert np.array_equal(bits(oracle.rmsnorm(g["rms_x"], g["rms_w"], 1e-5)), bits(g["rms_out"]))
    c, s = oracle.rope_table(64, 64, 10000.0)
    assert np.array_equal(bits(c), bits(g["rope_cos"])) and np.array_equal(bits(s), bits(g["rope_sin"]))
    q = oracle.rope_apply(g["rope_q"], 32, 64, c[37], s[37])
    assert np.array_equal(bits(q), bits(g["rope_q_out_pos37"]))
    a = oracle.attention(g["attn_q"], g["attn_k"], g["attn_v"], 40, 32, 4, 64)
    assert np.array_equal(bits(a), bits(g["attn_out"]))
    assert np.array_equal(bits(oracle.swiglu(g["swiglu_g"], g["swiglu_u"])), bits(g["swiglu_out"]))
    assert oracle.argmax(g["argmax_x"]) == int(g["argmax"]) == 17


def test_rope_attention_swiglu_match_pytorch_tinyllama_layer0(oracle):
    """Weight-free ops against the reference's PyTorch FP32 golden of the real model
    (golden_format.md: elementwise outputs within 1e-4 of the tensor's max |x|)."""
    g = golden("tinyllama_layer0.npz")
    pos = g["positions"]
    cos, sin = oracle.rope_table(23, 64, 10000.0)
    assert np.abs(cos - g["rope_cos"][:, :32]).max() < 1e-6
    for i, p in enumerate(pos):
        q = oracle.rope_apply(g["q"][i], 32, 64, cos[p], sin[p])
        assert np.abs(q - g["q_rope"][i]).max() <= 1e-4 * np.abs(g["q_rope"][i]).max()
    k = np.stack([oracle.rope_apply(g["k"][t], 4, 64, cos[t], sin[t]) for t in range(23)])
    assert np.abs(k - g["k_rope"]).max() <= 1e-4 * np.abs(g["k_rope"]).max()
    for i, p in enumerate(pos):
        ctx = oracle.attention(g["q_rope"][i], g["k_rope"][: p + 1], g["v"][: p + 1], p + 1, 32, 4, 64)
        assert np.abs(ctx - g["attn_context"][i]).max() <= 1e-4 * np.abs(g["attn_context"][i]).max()
    act = oracle.swiglu(g["gate"][1], g["up"][1])
    assert np.abs(act - g["mlp_act"][1]).max() <= 1e-4 * np.abs(g["mlp_act"][1]).max()


# ---------------------------------------------------------------- live reference


def test_oracle_equals_live_reference(oracle, reference):
    rng = np.random.default_rng(7)
    X = (rng.standard_normal((300, 512)) * 0.02).astype(np.float32)
    X[0, :32] = 0
    X[1, 5] = 40.0
    for qt in (Q4_0, Q8_0):
        for search in (True, False):
            a = oracle.quantize_rows(qt, X, search)
            assert np.array_equal(a, reference.quantize_rows(qt, X, search))
            x = rng.standard_normal(512).astype(np.float32)
            y = reference.matvec_backend(qt, a, x, 300, avx2=False)
            assert np.array_equal(bits(oracle.matvec(qt, a, x, 300)), bits(y))


def test_fake_quant_q4_group_matches_reference(oracle, reference):
    """fake_quant_q4_group (src/quant.cpp:243-248): groups of 32/64/128/256 and a 300-value group
    (only the first 256 are written), with and without the search; zero and non-finite groups."""
    rng = np.random.default_rng(31)
    cases = [(rng.standard_normal(n) * 0.02).astype(np.float32) for n in (32, 64, 100, 128, 256, 300)]
    cases.append(np.zeros(64, np.float32))
    bad = cases[1].copy(); bad[3] = np.inf; cases.append(bad)
    tiny = (rng.standard_normal(64) * 1e-9).astype(np.float32); cases.append(tiny)
    for x in cases:
        for search in (True, False):
            a = oracle.fake_quant_q4_group(x, search)
            b = reference.fake_quant_q4_group(x, search)
            np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
