"""ctypes access to the CPU checkers. TEST INFRASTRUCTURE ONLY.

Two libraries:
  * ``Oracle`` -> oracle/liboracle.so: the plain-C restatement (efo.c) of the
    reference's algorithm for the quantized matrix-product path.
  * ``Reference`` -> oracle/_ref/libefref.so: the reference implementation
    itself, compiled from its own sources by oracle/Makefile.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs import this
module. The product library (edgeforge_b200) never does.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle.so"
REF_SO = HERE / "_ref" / "libefref.so"


def reference_tree() -> Path | None:
    """The reference's source tree, when this machine has it: $EFG_REF_TREE, else the
    `reference_path` that the benchmark's BASELINE.json at the repository root names.
    None when neither points at a tree holding src/quant.cpp (as on a GPU box, which runs
    the prebuilt oracle/_ref library instead)."""
    cands = []
    if os.environ.get("EFG_REF_TREE"):
        cands.append(Path(os.environ["EFG_REF_TREE"]))
    base = HERE.parent / "BASELINE.json"
    if base.exists():
        import json

        try:
            rp = json.loads(base.read_text()).get("reference_path")
        except ValueError:
            rp = None
        if rp:
            cands.append(Path(rp))
    for c in cands:
        if (c / "src" / "quant.cpp").exists():
            return c
    return None

F32, F16, BF16, Q8_0, Q4_0 = 0, 1, 2, 3, 4
BLOCK_BYTES = {Q4_0: 18, Q8_0: 34}

_fp = C.POINTER(C.c_float)
_u8 = C.POINTER(C.c_uint8)
_vp = C.c_void_p
_sz = C.c_size_t


def _p(a: np.ndarray, t=_vp):
    return a.ctypes.data_as(t)


def row_bytes(qtype: int, cols: int) -> int:
    if qtype in BLOCK_BYTES:
        if cols % 32:
            raise ValueError(f"cols={cols} is not a multiple of 32")
        return cols // 32 * BLOCK_BYTES[qtype]
    return cols * (4 if qtype == F32 else 2)


class _Lib:
    """Shared numpy-level helpers; subclasses bind the symbol prefix."""

    prefix = ""

    def __init__(self, path: Path):
        if not path.exists():
            raise FileNotFoundError(f"{path} is not built (run: make -C {HERE})")
        self.lib = C.CDLL(str(path))
        self._bind()

    def _fn(self, name, restype, *argtypes):
        f = getattr(self.lib, self.prefix + name)
        f.restype = restype
        f.argtypes = list(argtypes)
        return f

    def _bind(self):
        self.fp16_to_f32 = self._fn("fp16_to_f32", C.c_float, C.c_uint16)
        self.f32_to_fp16 = self._fn("f32_to_fp16", C.c_uint16, C.c_float)
        self.bf16_to_f32 = self._fn("bf16_to_f32", C.c_float, C.c_uint16)
        self.f32_to_bf16 = self._fn("f32_to_bf16", C.c_uint16, C.c_float)
        self._qrow = self._fn("quantize_row", C.c_int, C.c_int, _fp, _sz, _vp, C.c_int)
        self._drow = self._fn("dequantize_row", C.c_int, C.c_int, _vp, _sz, _fp)
        self._fq = self._fn("fake_quant_q4_group", None, _fp, _sz, _fp, C.c_int)
        self._dot4 = self._fn("dot_q4_0", C.c_float, _u8, _fp, _sz)
        self._dot8 = self._fn("dot_q8_0", C.c_float, _u8, _fp, _sz)
        self._mv4 = self._fn("matvec_q4_0", None, _fp, _u8, _fp, _sz, _sz)
        self._mv8 = self._fn("matvec_q8_0", None, _fp, _u8, _fp, _sz, _sz)
        self._rms = self._fn("rmsnorm", None, _fp, _fp, _fp, _sz, C.c_float)
        self._swiglu = self._fn("swiglu", None, _fp, _fp, _fp, _sz)
        self._argmax = self._fn("argmax", _sz, _fp, _sz)
        self._ropet = self._fn("rope_table", None, _fp, _fp, _sz, _sz, C.c_float)
        self._ropea = self._fn("rope_apply", None, _fp, _sz, _sz, _fp, _fp)
        self._attn = self._fn("attention", None, _fp, _fp, _fp, _fp, _sz, _sz, _sz, _sz, _fp)

    # ---- rows -------------------------------------------------------------
    def quantize_row(self, qtype: int, x: np.ndarray, search: bool = True) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.zeros(row_bytes(qtype, x.size), dtype=np.uint8)
        if self._qrow(qtype, _p(x, _fp), x.size, _p(out), int(search)) != 0:
            raise ValueError("quantize_row rejected the input")
        return out

    def fake_quant_q4_group(self, x: np.ndarray, search: bool = True) -> np.ndarray:
        """quant.cpp:243-248; values past the first 256 stay 0."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.zeros(x.size, dtype=np.float32)
        self._fq(_p(x, _fp), x.size, _p(out, _fp), int(search))
        return out

    def dequantize_row(self, qtype: int, data: np.ndarray, n: int) -> np.ndarray:
        data = np.ascontiguousarray(data, dtype=np.uint8)
        out = np.zeros(n, dtype=np.float32)
        if self._drow(qtype, _p(data), n, _p(out, _fp)) != 0:
            raise ValueError("dequantize_row rejected the input")
        return out

    # ---- packed dots --------------------------------------------------------
    def dot(self, qtype: int, row: np.ndarray, x: np.ndarray) -> float:
        f = self._dot4 if qtype == Q4_0 else self._dot8
        return f(_p(row, _u8), _p(x, _fp), x.size)

    def matvec(self, qtype: int, W: np.ndarray, x: np.ndarray, rows: int) -> np.ndarray:
        W = np.ascontiguousarray(W, dtype=np.uint8)
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.zeros(rows, dtype=np.float32)
        f = self._mv4 if qtype == Q4_0 else self._mv8
        f(_p(y, _fp), _p(W, _u8), _p(x, _fp), rows, x.size)
        return y

    # ---- FP32 ops -----------------------------------------------------------
    def rmsnorm(self, x, w, eps):
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        out = np.zeros_like(x)
        self._rms(_p(out, _fp), _p(x, _fp), _p(w, _fp), x.size, eps)
        return out

    def swiglu(self, g, u):
        g = np.ascontiguousarray(g, np.float32)
        u = np.ascontiguousarray(u, np.float32)
        out = np.zeros_like(g)
        self._swiglu(_p(out, _fp), _p(g, _fp), _p(u, _fp), g.size)
        return out

    def argmax(self, x):
        x = np.ascontiguousarray(x, np.float32)
        return int(self._argmax(_p(x, _fp), x.size))

    def rope_table(self, max_pos, hd, theta):
        c = np.zeros((max_pos, hd // 2), np.float32)
        s = np.zeros((max_pos, hd // 2), np.float32)
        self._ropet(_p(c, _fp), _p(s, _fp), max_pos, hd, theta)
        return c, s

    def rope_apply(self, x, n_heads, hd, cos_row, sin_row):
        x = np.array(x, np.float32, copy=True)
        cos_row = np.ascontiguousarray(cos_row, np.float32)
        sin_row = np.ascontiguousarray(sin_row, np.float32)
        self._ropea(_p(x, _fp), n_heads, hd, _p(cos_row, _fp), _p(sin_row, _fp))
        return x

    def attention(self, q, k_cache, v_cache, n_pos, H, KV, hd):
        q = np.ascontiguousarray(q, np.float32)
        k_cache = np.ascontiguousarray(k_cache, np.float32)
        v_cache = np.ascontiguousarray(v_cache, np.float32)
        out = np.zeros(H * hd, np.float32)
        scores = np.zeros(max(n_pos, 1), np.float32)
        self._attn(_p(out, _fp), _p(q, _fp), _p(k_cache, _fp), _p(v_cache, _fp), n_pos, H, KV, hd, _p(scores, _fp))
        return out


class Oracle(_Lib):
    """The C restatement (oracle/efo.c)."""

    prefix = "efo_"

    def __init__(self, path: Path = ORACLE_SO):
        super().__init__(path)

    def _bind(self):
        super()._bind()
        self._qrows = self._fn("quantize_rows", C.c_int, C.c_int, _fp, _sz, _sz, _vp, C.c_int, C.c_int)
        self._drows = self._fn("dequantize_rows", C.c_int, C.c_int, _vp, _sz, _sz, _fp, C.c_int)
        self._mvmt = self._fn("matvec_mt", None, C.c_int, _fp, _u8, _fp, _sz, _sz, C.c_int)
        self._exact = self._fn("exact_dot", None, C.c_int, _u8, _fp, _sz,
                               C.POINTER(C.c_double), C.POINTER(C.c_double))
        self._exact_rows = self._fn("exact_dots", C.c_int, C.c_int, _u8, _fp, _sz, _sz,
                                    C.POINTER(C.c_double), C.POINTER(C.c_double), C.c_int)

    def quantize_rows(self, qtype, X, search=True, threads=os.cpu_count() or 1):
        X = np.ascontiguousarray(X, dtype=np.float32)
        rows, cols = X.shape
        out = np.zeros((rows, row_bytes(qtype, cols)), dtype=np.uint8)
        if self._qrows(qtype, _p(X, _fp), rows, cols, _p(out), int(search), int(threads)) != 0:
            raise ValueError("quantize_rows rejected the input")
        return out

    def dequantize_rows(self, qtype, Wq, cols, threads=os.cpu_count() or 1):
        Wq = np.ascontiguousarray(Wq, dtype=np.uint8)
        rows = Wq.size // row_bytes(qtype, cols)
        out = np.zeros((rows, cols), dtype=np.float32)
        if self._drows(qtype, _p(Wq), rows, cols, _p(out, _fp), int(threads)) != 0:
            raise ValueError("dequantize_rows rejected the input")
        return out

    def matvec_mt(self, qtype, W, x, rows, threads=os.cpu_count() or 1):
        W = np.ascontiguousarray(W, dtype=np.uint8)
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.zeros(rows, dtype=np.float32)
        self._mvmt(qtype, _p(y, _fp), _p(W, _u8), _p(x, _fp), rows, x.size, int(threads))
        return y

    def exact_dots(self, qtype, W, x, rows):
        """(exact, magnitude) per row: double dot of the dequantized row with x, sum|w x|."""
        W = np.ascontiguousarray(W, dtype=np.uint8).reshape(rows, -1)
        x = np.ascontiguousarray(x, dtype=np.float32)
        ex = np.zeros(rows)
        mag = np.zeros(rows)
        if rows and W.shape[1] != row_bytes(qtype, x.size):
            raise ValueError(f"rows of {W.shape[1]} bytes do not hold {x.size} weights")
        if rows:
            threads = min(os.cpu_count() or 1, max(1, rows * x.size // (1 << 20)))
            rc = self._exact_rows(qtype, _p(W, _u8), _p(x, _fp), rows, x.size, _p(ex, C.POINTER(C.c_double)),
                                  _p(mag, C.POINTER(C.c_double)), threads)
            if rc != 0:
                raise ValueError(f"cols={x.size} is not a multiple of 32")
        return ex, mag


class Reference(_Lib):
    """The reference implementation, compiled from its own sources (oracle/_ref)."""

    prefix = "efr_"

    def __init__(self, path: Path = REF_SO):
        super().__init__(path)

    def _bind(self):
        super()._bind()
        self._fn("last_error", C.c_char_p)
        self.avx2 = bool(self._fn("avx2_compiled", C.c_int)())
        self._pool_new = self._fn("pool_new", _vp, C.c_uint)
        self._pool_free = self._fn("pool_free", None, _vp)
        self._mv = self._fn("matvec", C.c_int, C.c_int, _vp, C.c_int, _fp, _u8, _fp, _sz, _sz)
        self._qrows = self._fn("quantize_rows", C.c_int, _vp, C.c_int, _fp, _sz, _sz, _vp, C.c_int)
        self._drows = self._fn("dequantize_rows", C.c_int, _vp, C.c_int, _vp, _sz, _sz, _fp)
        self._qmodel = self._fn("quantize_model", C.c_int, C.c_char_p, C.c_char_p, C.c_char_p, C.c_char_p, C.c_uint)
        self._dec_new = self._fn("decoder_new", _vp, C.c_char_p, _sz, C.c_uint)
        self._dec_free = self._fn("decoder_free", None, _vp)
        self._dec_reset = self._fn("decoder_reset", None, _vp)
        self._dec_fwd = self._fn("decoder_forward", C.c_int, _vp, C.c_int, C.c_int32, _sz, _fp)
        self._dec_bpt = self._fn("decoder_bytes_per_token", C.c_uint64, _vp)

    def error(self) -> str:
        return self.lib.efr_last_error().decode()

    def pool(self, threads: int):
        return _Pool(self, threads)

    def matvec_backend(self, qtype, W, x, rows, avx2=True, pool=None, y=None):
        if y is None:
            y = np.zeros(rows, dtype=np.float32)
        h = pool.handle if pool is not None else None
        if self._mv(int(avx2), h, qtype, _p(y, _fp), _p(W, _u8), _p(x, _fp), rows, x.size) != 0:
            raise RuntimeError(self.error())
        return y

    def quantize_rows(self, qtype, X, search=True, pool=None):
        X = np.ascontiguousarray(X, dtype=np.float32)
        rows, cols = X.shape
        out = np.zeros((rows, row_bytes(qtype, cols)), dtype=np.uint8)
        h = pool.handle if pool is not None else None
        if self._qrows(h, qtype, _p(X, _fp), rows, cols, _p(out), int(search)) != 0:
            raise RuntimeError(self.error())
        return out

    def dequantize_rows(self, qtype, Wq, cols, pool=None):
        Wq = np.ascontiguousarray(Wq, dtype=np.uint8)
        rows = Wq.size // row_bytes(qtype, cols)
        out = np.zeros((rows, cols), dtype=np.float32)
        h = pool.handle if pool is not None else None
        if self._drows(h, qtype, _p(Wq), rows, cols, _p(out, _fp)) != 0:
            raise RuntimeError(self.error())
        return out

    def quantize_model(self, model_dir, out_file, policy="auto", overrides="", threads=0):
        """quantize_model (src/quantizer.cpp:151-290): a named policy, or explicit overrides
        in the reference's TENSOR=TYPE,... form."""
        if self._qmodel(str(model_dir).encode(), str(out_file).encode(), policy.encode(), overrides.encode(),
                        threads) != 0:
            raise RuntimeError(self.error())

    def decoder(self, efq_file, max_seq, threads=1):
        return _Decoder(self, efq_file, max_seq, threads)


class _Pool:
    def __init__(self, ref: Reference, threads: int):
        self.ref = ref
        self.threads = threads
        self.handle = ref._pool_new(threads)

    def close(self):
        if self.handle:
            self.ref._pool_free(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


class _Decoder:
    """Model::load_efq + Transformer from the reference (one token per forward)."""

    def __init__(self, ref: Reference, efq_file, max_seq, threads):
        self.ref = ref
        self.h = ref._dec_new(str(efq_file).encode(), max_seq, threads)
        if not self.h:
            raise RuntimeError(ref.error())

    def forward(self, token: int, pos: int, vocab: int, avx2=True, logits=True):
        out = np.zeros(vocab, dtype=np.float32) if logits else None
        if self.ref._dec_fwd(self.h, int(avx2), token, pos, _p(out, _fp) if logits else None) != 0:
            raise RuntimeError(self.ref.error())
        return out

    def reset(self):
        self.ref._dec_reset(self.h)

    def bytes_per_token(self):
        return int(self.ref._dec_bpt(self.h))

    def close(self):
        if self.h:
            self.ref._dec_free(self.h)
            self.h = None


def reference_available() -> bool:
    return REF_SO.exists()


# ---------------------------------------------------------------- the decode step on the C restatement


class _Weight(C.Structure):
    _fields_ = [("type", C.c_int), ("data", _vp), ("rows", _sz), ("cols", _sz)]


class _Layer(C.Structure):
    _fields_ = [(n, _Weight) for n in ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down")] + [
        ("attn_norm", _fp), ("ffn_norm", _fp)]


class _Model(C.Structure):
    _fields_ = [(n, _sz) for n in ("D", "F", "H", "KV", "hd", "V", "L", "max_seq")] + [
        ("eps", C.c_float), ("rope_theta", C.c_float), ("embed", _Weight), ("lm_head", _Weight),
        ("final_norm", _fp), ("layers", C.POINTER(_Layer))]


_TYPES = {"F32": F32, "F16": F16, "BF16": BF16, "Q8_0": Q8_0, "Q4_0": Q4_0}


def read_efq(path):
    """(config dict, {name: (type, shape, uint8 view of the tensor's bytes)}) of an .efq file
    (layout of src/qfile.cpp:79-123: "EFQ1", u32 version, u64 header length, JSON header,
    tensors at absolute 64-byte aligned offsets)."""
    import json

    raw = np.fromfile(path, dtype=np.uint8)
    if bytes(raw[:4]) != b"EFQ1":
        raise ValueError("bad magic")
    hlen = int(raw[8:16].view("<u8")[0])
    hdr = json.loads(bytes(raw[16:16 + hlen]).decode())
    tensors = {}
    for t in hdr["tensors"]:
        off, n = int(t["offset"]), int(t["bytes"])
        tensors[t["name"]] = (_TYPES[t["type"].upper()], [int(s) for s in t["shape"]], raw[off:off + n])
    return hdr["config"], tensors


class OracleDecoder:
    """efo_forward (oracle/efo.c, restating src/model.cpp:184-276) over an .efq file."""

    def __init__(self, oracle: Oracle, efq_file, max_seq: int):
        self.o = oracle
        cfg, t = read_efq(efq_file)
        self._keep = t
        D, H = int(cfg["hidden_size"]), int(cfg["num_attention_heads"])
        L = int(cfg["num_hidden_layers"])
        self.vocab = int(cfg["vocab_size"])

        def w(name):
            ty, shape, data = t[name]
            return _Weight(ty, data.ctypes.data, shape[0] if len(shape) == 2 else 1, shape[-1])

        def v(name):
            return C.cast(C.c_void_p(t[name][2].ctypes.data), _fp)

        layers = (_Layer * L)()
        for i in range(L):
            p = f"model.layers.{i}."
            layers[i] = _Layer(w(p + "self_attn.q_proj.weight"), w(p + "self_attn.k_proj.weight"),
                               w(p + "self_attn.v_proj.weight"), w(p + "self_attn.o_proj.weight"),
                               w(p + "mlp.gate_proj.weight"), w(p + "mlp.up_proj.weight"),
                               w(p + "mlp.down_proj.weight"), v(p + "input_layernorm.weight"),
                               v(p + "post_attention_layernorm.weight"))
        self._layers = layers
        tied = bool(cfg.get("tie_word_embeddings", False))
        m = _Model(D, int(cfg["intermediate_size"]), H, int(cfg.get("num_key_value_heads", H)),
                   int(cfg.get("head_dim", D // H)), self.vocab, L, int(max_seq), float(cfg["rms_norm_eps"]),
                   float(cfg.get("rope_theta", 10000.0)), w("model.embed_tokens.weight"),
                   w("model.embed_tokens.weight" if tied else "lm_head.weight"), v("model.norm.weight"), layers)
        self._model = m
        lib = oracle.lib
        lib.efo_state_new.restype = _vp
        lib.efo_state_new.argtypes = [C.POINTER(_Model)]
        lib.efo_state_free.argtypes = [_vp]
        lib.efo_forward.restype = C.c_int
        lib.efo_forward.argtypes = [_vp, C.c_int32, _sz, _fp, C.c_int]
        self._s = lib.efo_state_new(C.byref(m))
        if not self._s:
            raise MemoryError("efo_state_new failed")

    def forward(self, token: int, pos: int, logits=True, threads=os.cpu_count() or 1):
        out = np.zeros(self.vocab, np.float32) if logits else None
        if self.o.lib.efo_forward(self._s, int(token), int(pos), _p(out, _fp) if logits else None, threads) != 0:
            raise ValueError("efo_forward rejected the token or position")
        return out

    def close(self):
        if self._s:
            self.o.lib.efo_state_free(self._s)
            self._s = None

    def __del__(self):
        self.close()

    def run(self, prompt, forced, threads=os.cpu_count() or 1):
        """Teacher-forced greedy run: the prompt, then the `forced` ids. Returns the logits
        after the last prompt token and after each forced token but the last, as
        [len(forced)][vocab] (the logits generate_greedy takes its argmax from)."""
        out = []
        pos = 0
        for i, tok in enumerate(prompt):
            lg = self.forward(tok, pos, logits=i + 1 == len(prompt), threads=threads)
            pos += 1
        out.append(lg)
        for tok in list(forced)[:-1]:
            out.append(self.forward(tok, pos, threads=threads))
            pos += 1
        return np.stack(out)
