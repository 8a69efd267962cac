#!/usr/bin/env python3
"""Regenerates the golden fixtures in tests/golden/ (run in a checkout next to the
reference source tree; the GPU box only reads the committed .npz files).

Sources:
  * the reference implementation itself, compiled from its own sources into
    oracle/_ref/libefref.so (make -C oracle): fp16 conversions, Q4_0/Q8_0
    quantize/dequantize, the scalar and AVX2 packed dots, RMSNorm, RoPE, attention,
    SwiGLU, argmax, all on seeded inputs;
  * the reference's PyTorch FP32 golden tensors of the real TinyLlama-1.1B
    (tests/golden/prompts/p0_factual/layer0 in the reference tree): a slice that pins
    the weight-free decode ops (RoPE, attention, SwiGLU).

    python tests/golden/make_golden.py [--ref-tree <reference source tree>]
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from oracle.oracle import Q4_0, Q8_0, Reference, reference_tree, row_bytes  # noqa: E402


def f32_from_bits(u):
    return np.asarray(u, dtype=np.uint32).view(np.float32)


def quant_inputs(rng) -> np.ndarray:
    """64 rows x 256 cols: N(0, 0.02) blocks plus the edge cases the reference tests
    and the quantizer's branches meet (test_quant.cpp:52-123)."""
    X = (rng.standard_normal((64, 256)) * 0.02).astype(np.float32)
    X[1] = (rng.standard_normal(256)).astype(np.float32)
    X[2, :32] = 0.0                                            # all-zero block -> d = 0, codes 8
    X[2, 32:64] = np.float32(np.inf)                           # non-finite amax
    X[2, 64] = np.float32(np.nan)                              # one NaN in a finite block
    X[2, 96:128] = 1e-30                                       # every candidate underflows fp16
    X[3, :32] = (np.arange(32) % 16 - 8).astype(np.float32) * 0.25  # exact grid values
    X[4] *= 1000.0                                             # large values
    X[5, :32] = 7e4                                            # beyond fp16 range -> clamped scale
    X[5, 32:64] = -7e4
    X[5, 64:96] = np.linspace(-1e6, 1e6, 32, dtype=np.float32)
    X[6, 7] = 50.0                                             # single outlier
    X[7, :32] = -1e-7                                          # fp16-subnormal scales
    X[8] = (rng.standard_normal(256) * 1e-5).astype(np.float32)
    for r in range(9, 64, 7):
        X[r, (r * 5) % 256] *= 6.0                             # outliers like test_quant.cpp:80
    X[10, :32] = np.float32(3.0e38)                            # near float max
    X[11, 32:64] = 2.5e-5                                      # ties around the fp16 subnormal grid
    return X


def random_rows(qtype, rows, cols, rng) -> np.ndarray:
    """Arbitrary codes with random fp16 scales in [-0.05, 0.05) (test_qinfer.cpp:28-40)."""
    rb = row_bytes(qtype, cols)
    v = rng.integers(0, 256, rows * rb, dtype=np.uint8)
    bsz = 18 if qtype == Q4_0 else 34
    scales = rng.uniform(-0.05, 0.05, rows * rb // bsz).astype(np.float32)
    h = scales.astype(np.float16).view(np.uint16)
    v = v.reshape(-1, bsz)
    v[:, 0] = (h & 0xFF).astype(np.uint8)
    v[:, 1] = (h >> 8).astype(np.uint8)
    return v.reshape(rows, rb)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-tree", type=Path, default=None,
                    help="reference source tree (default: $EFG_REF_TREE or BASELINE.json's reference_path)")
    args = ap.parse_args()
    if args.ref_tree is None:
        args.ref_tree = reference_tree()
    if args.ref_tree is None:
        ap.error("no reference source tree: pass --ref-tree or set EFG_REF_TREE")
    ref = Reference()
    rng = np.random.default_rng(20261201)
    manifest = {"generator": "tests/golden/make_golden.py", "reference": "oracle/_ref/libefref.so", "files": {}}

    # ---- fp16 (include/ef/fp16.h): every half pattern, and sampled floats
    h_all = np.arange(65536, dtype=np.uint32)
    f_of_h = np.array([ref.fp16_to_f32(int(h)) for h in h_all], dtype=np.float32)
    f_samples = np.concatenate([
        f32_from_bits(rng.integers(0, 2**32, 6000, dtype=np.uint64)),
        (rng.standard_normal(2000) * 10.0 ** rng.integers(-9, 6, 2000)).astype(np.float32),
        np.array([0.0, -0.0, 65504, 65519.996, 65520, -65520, 2.0**-24, 2.0**-25, 3 * 2.0**-26,
                  2.0**-14, np.inf, -np.inf, np.nan], dtype=np.float32),
    ])
    h_of_f = np.array([ref.f32_to_fp16(float(f)) for f in f_samples], dtype=np.uint16)
    np.savez_compressed(HERE / "fp16.npz", fp16_to_f32=f_of_h, f32_samples=f_samples, f32_to_fp16=h_of_f)
    manifest["files"]["fp16.npz"] = "fp16_to_f32 of all 65536 halves; f32_to_fp16 of sampled floats"

    # ---- quantize / dequantize (src/quant.cpp)
    X = quant_inputs(rng)
    q4s = ref.quantize_rows(Q4_0, X, search=True)
    q4a = ref.quantize_rows(Q4_0, X, search=False)
    q8 = ref.quantize_rows(Q8_0, X)
    np.savez_compressed(
        HERE / "quant.npz", x=X, q4_search=q4s, q4_absmax=q4a, q8=q8,
        q4_search_deq=ref.dequantize_rows(Q4_0, q4s, 256), q8_deq=ref.dequantize_rows(Q8_0, q8, 256))
    manifest["files"]["quant.npz"] = "64x256 floats with edge cases -> Q4_0 (search, absmax), Q8_0 and dequantized"

    # ---- packed dots (src/qkernels.cpp), scalar and AVX2 backends
    mv = {}
    for n in (32, 64, 96, 2048, 5632):
        x = rng.standard_normal(n).astype(np.float32)
        x *= np.where(rng.standard_normal(n) > 2.0, 30.0, 1.0).astype(np.float32)  # test_qinfer.cpp:77
        mv[f"x_{n}"] = x
        for qt, name in ((Q4_0, "q4"), (Q8_0, "q8")):
            W = random_rows(qt, 24, n, rng)
            mv[f"{name}_W_{n}"] = W
            mv[f"{name}_y_scalar_{n}"] = ref.matvec_backend(qt, W, x, 24, avx2=False)
            mv[f"{name}_y_avx2_{n}"] = ref.matvec_backend(qt, W, x, 24, avx2=True)
    np.savez_compressed(HERE / "matvec.npz", **mv)
    manifest["files"]["matvec.npz"] = "24 random packed rows per n in {32,64,96,2048,5632}; reference scalar/AVX2 y"

    # ---- decode-step ops (src/kernels.cpp)
    ops = {}
    x = rng.standard_normal(2048).astype(np.float32)
    w = (1.0 + 0.1 * rng.standard_normal(2048)).astype(np.float32)
    ops["rms_x"], ops["rms_w"], ops["rms_out"] = x, w, ref.rmsnorm(x, w, 1e-5)
    c, s = ref.rope_table(64, 64, 10000.0)
    ops["rope_cos"], ops["rope_sin"] = c, s
    q = rng.standard_normal(32 * 64).astype(np.float32)
    ops["rope_q"], ops["rope_q_out_pos37"] = q, ref.rope_apply(q, 32, 64, c[37], s[37])
    n_pos = 40
    kc = rng.standard_normal(n_pos * 256).astype(np.float32)
    vc = rng.standard_normal(n_pos * 256).astype(np.float32)
    ops["attn_q"], ops["attn_k"], ops["attn_v"] = q, kc, vc
    ops["attn_out"] = ref.attention(q, kc, vc, n_pos, 32, 4, 64)
    g = (rng.standard_normal(5632) * 3).astype(np.float32)
    u = rng.standard_normal(5632).astype(np.float32)
    ops["swiglu_g"], ops["swiglu_u"], ops["swiglu_out"] = g, u, ref.swiglu(g, u)
    lg = rng.standard_normal(32000).astype(np.float32)
    lg[[17, 31000]] = lg.max() + 1.0  # tie: the first index wins
    ops["argmax_x"], ops["argmax"] = lg, np.int64(ref.argmax(lg))
    np.savez_compressed(HERE / "decode_ops.npz", **ops)
    manifest["files"]["decode_ops.npz"] = "rmsnorm, rope table/apply, GQA attention, swiglu, argmax on seeded inputs"

    # ---- TinyLlama layer-0 tensors from the reference's PyTorch golden (real weights)
    p0 = args.ref_tree / "tests" / "golden" / "prompts" / "p0_factual"
    if p0.exists():
        S, D, KVD, F = 23, 2048, 256, 5632

        def rd(name, shape):
            return np.fromfile(p0 / name, dtype="<f4").reshape(shape)

        pos = [0, 11, 22]
        L0 = {
            "positions": np.array(pos, dtype=np.int64),
            "rope_cos": rd("rope_cos.f32", (S, 64)), "rope_sin": rd("rope_sin.f32", (S, 64)),
            "q": rd("layer0/q.f32", (S, D))[pos], "q_rope": rd("layer0/q_rope.f32", (S, D))[pos],
            "k": rd("layer0/k.f32", (S, KVD)), "k_rope": rd("layer0/k_rope.f32", (S, KVD)),
            "v": rd("layer0/v.f32", (S, KVD)),
            "attn_context": rd("layer0/attn_context.f32", (S, D))[pos],
            "gate": rd("layer0/gate.f32", (S, F))[[0, 22]], "up": rd("layer0/up.f32", (S, F))[[0, 22]],
            "mlp_act": rd("layer0/mlp_act.f32", (S, F))[[0, 22]],
        }
        np.savez_compressed(HERE / "tinyllama_layer0.npz", **L0)
        manifest["files"]["tinyllama_layer0.npz"] = (
            "PyTorch FP32 layer-0 tensors of TinyLlama-1.1B-Chat (reference tests/golden/prompts/p0_factual): "
            "q/k before and after RoPE, v, attention context at positions 0/11/22, gate/up/silu*up at 0/22")
    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1) + "\n")
    print("wrote", ", ".join(manifest["files"]))
    return 0


if __name__ == "__main__":
    sys.exit(main())
