"""Random Llama-architecture checkpoints in the reference's input format (config.json +
BF16 model.safetensors), for tests and benchmarks: weights N(0, 0.02), norm weights
1 + 0.1 N(0, 1), float32 draws from numpy's default_rng(seed) rounded to BF16 (round to
nearest even), tensors in name order. These are the distributions of the reference's
synthetic checkpoint tool (tools/make_synthetic_checkpoint.py); the file format is
safetensors (8-byte header length, JSON header, raw little-endian data).
"""
from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np

TINYLLAMA = {
    "architectures": ["LlamaForCausalLM"], "attention_bias": False, "bos_token_id": 1, "eos_token_id": 2,
    "hidden_act": "silu", "hidden_size": 2048, "initializer_range": 0.02, "intermediate_size": 5632,
    "max_position_embeddings": 2048, "model_type": "llama", "num_attention_heads": 32, "num_hidden_layers": 22,
    "num_key_value_heads": 4, "rms_norm_eps": 1e-05, "rope_scaling": None, "rope_theta": 10000.0,
    "tie_word_embeddings": False, "torch_dtype": "bfloat16", "use_cache": True, "vocab_size": 32000,
}


def tiny_config(hidden=64, intermediate=128, layers=2, heads=4, kv_heads=2, vocab=96, max_pos=64) -> dict:
    c = dict(TINYLLAMA)
    c.update(hidden_size=hidden, intermediate_size=intermediate, num_hidden_layers=layers, num_attention_heads=heads,
             num_key_value_heads=kv_heads, vocab_size=vocab, max_position_embeddings=max_pos)
    return c


def tensor_list(c: dict) -> list[tuple[str, list[int]]]:
    D, F, V = c["hidden_size"], c["intermediate_size"], c["vocab_size"]
    KV = c["num_key_value_heads"] * (D // c["num_attention_heads"])
    out = [("model.embed_tokens.weight", [V, D])]
    for i in range(c["num_hidden_layers"]):
        p = f"model.layers.{i}."
        out += [(p + "self_attn.q_proj.weight", [D, D]), (p + "self_attn.k_proj.weight", [KV, D]),
                (p + "self_attn.v_proj.weight", [KV, D]), (p + "self_attn.o_proj.weight", [D, D]),
                (p + "mlp.gate_proj.weight", [F, D]), (p + "mlp.up_proj.weight", [F, D]),
                (p + "mlp.down_proj.weight", [D, F]), (p + "input_layernorm.weight", [D]),
                (p + "post_attention_layernorm.weight", [D])]
    out.append(("model.norm.weight", [D]))
    if not c["tie_word_embeddings"]:
        out.append(("lm_head.weight", [V, D]))
    return out


def bf16_bits(a: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def write_checkpoint(out: Path, config: dict, seed: int = 0) -> Path:
    """Writes out/config.json and out/model.safetensors; returns out."""
    out = Path(out)
    out.mkdir(parents=True, exist_ok=True)
    tensors = sorted(tensor_list(config), key=lambda t: t[0])
    header: dict = {"__metadata__": {"format": "pt"}}
    off = 0
    for name, shape in tensors:
        n = int(np.prod(shape))
        header[name] = {"dtype": "BF16", "shape": shape, "data_offsets": [off, off + 2 * n]}
        off += 2 * n
    hj = json.dumps(header, separators=(",", ":")).encode()
    hj += b" " * ((8 - (8 + len(hj)) % 8) % 8)
    (out / "config.json").write_text(json.dumps(config, indent=2) + "\n")
    rng = np.random.default_rng(seed)
    with open(out / "model.safetensors", "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for name, shape in tensors:
            n = int(np.prod(shape))
            chunk = 1 << 24
            for start in range(0, n, chunk):  # bounded memory for the 1.1B-parameter shape
                m = min(chunk, n - start)
                if name.endswith("norm.weight"):
                    vals = 1.0 + 0.1 * rng.standard_normal(m, dtype=np.float32)
                else:
                    vals = 0.02 * rng.standard_normal(m, dtype=np.float32)
                bf16_bits(vals).astype("<u2").tofile(f)
    return out
