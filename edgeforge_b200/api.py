"""Python mirror of the reference's kernel API for the packed matrix-product path.

Names and argument meaning follow the reference (include/ef/qkernels.h,
include/ef/quant.h): ``matvec_q4_0(y, W, x, rows, cols)``, ``quantize_row(t, x, n,
out, search)``, ... The arrays are torch CUDA tensors on the current device, and every
call is queued on torch's current CUDA stream. Errors raise EdgeForgeError, the way the
reference throws ef::Error (a row length that is not a multiple of 32 gives the
reference's message, "Q4_0 needs a row length divisible by 32, got 30").

The ``host_*`` functions take numpy arrays and are synchronous, exactly the
reference's host-pointer calls (the weight matrix stays resident on the device).
"""
from __future__ import annotations

import ctypes as C
from enum import IntEnum

import numpy as np

from ._lib import EdgeForgeError, MatvecJob, ModelInfo, QuantizeReport, check, load


class QType(IntEnum):
    """ef::QType (include/ef/quant.h:35)."""

    F32 = 0
    F16 = 1
    BF16 = 2
    Q8_0 = 3
    Q4_0 = 4


QK = 32
BLOCK_BYTES = {QType.Q4_0: 18, QType.Q8_0: 34}


def row_bytes(qtype: int, cols: int) -> int:
    """ef::qtype_row_bytes (include/ef/quant.h:42): raises for cols % 32 != 0."""
    n = load().efg_row_bytes(int(qtype), int(cols))
    if n == 0 and cols != 0:
        raise EdgeForgeError(1, load().efg_last_error().decode())
    return int(n)


def _stream():
    import torch

    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t) -> C.c_void_p:
    if t is None:
        return C.c_void_p(0)
    if not t.is_cuda:
        raise EdgeForgeError(1, "expected a CUDA tensor")
    if not t.is_contiguous():
        raise EdgeForgeError(1, "expected a contiguous tensor")
    return C.c_void_p(t.data_ptr())


# ---------------------------------------------------------------- matvec


def matvec_q4_0(y, W, x, rows: int, cols: int) -> None:
    """y[r] = dot(row r of W, x) for Q4_0 W (ef::kern::matvec_q4_0, qkernels.h:50)."""
    check(load().efg_matvec_q4_0(_ptr(y), _ptr(W), _ptr(x), rows, cols, _stream()))


def matvec_q8_0(y, W, x, rows: int, cols: int) -> None:
    """ef::kern::matvec_q8_0 (qkernels.h:51)."""
    check(load().efg_matvec_q8_0(_ptr(y), _ptr(W), _ptr(x), rows, cols, _stream()))


def matvec(qtype: int, y, W, x, rows: int, cols: int) -> None:
    """ef::kern::matvec for a WeightView of a packed type (qkernels.h:66)."""
    check(load().efg_matvec(int(qtype), _ptr(y), _ptr(W), _ptr(x), rows, cols, _stream()))


def matvec_jobs(jobs) -> None:
    """ef::kern::matvec_jobs (qkernels.h:70-75). jobs: iterable of
    (y, qtype, W, rows, cols, x) tuples of CUDA tensors."""
    arr = (MatvecJob * len(jobs))()
    for i, (y, qt, W, rows, cols, x) in enumerate(jobs):
        arr[i] = MatvecJob(_ptr(y).value, int(qt), _ptr(W).value, rows, cols, _ptr(x).value)
    check(load().efg_matvec_jobs(arr, len(jobs), _stream()))


def dot_q4_0(out, row, x, n: int) -> None:
    """ef::kern::dot_q4_0 (qkernels.h:47), result written to out[0]."""
    check(load().efg_dot_q4_0(_ptr(out), _ptr(row), _ptr(x), n, _stream()))


def dot_q8_0(out, row, x, n: int) -> None:
    """ef::kern::dot_q8_0 (qkernels.h:48)."""
    check(load().efg_dot_q8_0(_ptr(out), _ptr(row), _ptr(x), n, _stream()))


# ---------------------------------------------------------------- quantize / dequantize


def quantize_row(qtype: int, x, n: int, out, search: bool = True) -> None:
    """ef::quantize_row (quant.h:52), bit-exact."""
    check(load().efg_quantize_row(int(qtype), _ptr(x), n, _ptr(out), int(search), _stream()))


def dequantize_row(qtype: int, data, n: int, out) -> None:
    """ef::dequantize_row (quant.h:53), bit-exact."""
    check(load().efg_dequantize_row(int(qtype), _ptr(data), n, _ptr(out), _stream()))


def quantize_rows(qtype: int, X, rows: int, cols: int, out, search: bool = True) -> None:
    """quantize_row over every row of a [rows][cols] matrix in one launch."""
    check(load().efg_quantize_rows(int(qtype), _ptr(X), rows, cols, _ptr(out), int(search), _stream()))


def dequantize_rows(qtype: int, data, rows: int, cols: int, out) -> None:
    check(load().efg_dequantize_rows(int(qtype), _ptr(data), rows, cols, _ptr(out), _stream()))


def row_f32(out, qtype: int, W, rows: int, cols: int, r: int | None = None, r_dev=None) -> None:
    """ef::kern::row_f32 (qkernels.h:78): row r of W as FP32. r_dev: an int32 CUDA tensor
    holding the row index (read on the device)."""
    rp = C.cast(C.c_void_p(r_dev.data_ptr()), C.POINTER(C.c_int32)) if r_dev is not None else None
    check(load().efg_row_f32(_ptr(out), int(qtype), _ptr(W), rows, cols, rp, r or 0, _stream()))


def set_q4_mma(enable: bool) -> bool:
    """efg_set_q4_mma: large Q4_0 matvecs on this thread use the integer tensor-core
    kernel (True, the default) or the CUDA-core kernel (False). Returns the previous
    setting."""
    return bool(load().efg_set_q4_mma(int(enable)))


def set_small_gemm(enable: bool) -> bool:
    """efg_set_small_gemm: Q4_0 GEMMs of B <= 64 columns on this thread use the small-batch
    integer-MMA kernel (default off). Returns the old setting."""
    return bool(load().efg_set_small_gemm(int(enable)))


def set_weight_prefetch(enable: bool) -> bool:
    """efg_set_weight_prefetch: lets later matvec launches on this thread stream their
    weights while the previous kernel finishes (weights must not be written just
    before). Returns the previous setting."""
    return bool(load().efg_set_weight_prefetch(int(enable)))


def device_error() -> int:
    """Reads and clears the device error word (EFG_OK or EFG_ETIMEOUT / EFG_EINVAL)."""
    code = C.c_int(0)
    check(load().efg_device_error(C.byref(code)))
    return code.value


# ---------------------------------------------------------------- host-pointer forms


def _np(a, dtype):
    a = np.ascontiguousarray(a, dtype=dtype)
    return a, C.c_void_p(a.ctypes.data)


def host_register_weights(W: np.ndarray) -> None:
    """Uploads W once and keeps it resident; later host calls on views inside W use the
    device copy. W must not change while registered (efg_host_register_weights)."""
    if not W.flags["C_CONTIGUOUS"]:
        raise EdgeForgeError(1, "register_weights needs a contiguous array")
    check(load().efg_host_register_weights(C.c_void_p(W.ctypes.data), W.nbytes))


def host_unregister_weights(W: np.ndarray) -> None:
    check(load().efg_host_unregister_weights(C.c_void_p(W.ctypes.data)))


def host_matvec(qtype: int, W: np.ndarray, x: np.ndarray, rows: int, y: np.ndarray | None = None) -> np.ndarray:
    """Synchronous host-pointer matvec (W read from a registered resident copy when it
    lies inside one, else uploaded for this call)."""
    W, pw = _np(W, np.uint8)
    x, px = _np(x, np.float32)
    if y is None:
        y = np.zeros(rows, dtype=np.float32)
    check(load().efg_host_matvec(int(qtype), C.c_void_p(y.ctypes.data), pw, px, rows, x.size))
    return y


def host_quantize_row(qtype: int, x: np.ndarray, search: bool = True) -> np.ndarray:
    x, px = _np(x, np.float32)
    out = np.zeros(row_bytes(qtype, x.size), dtype=np.uint8)
    check(load().efg_host_quantize_row(int(qtype), px, x.size, C.c_void_p(out.ctypes.data), int(search)))
    return out


def host_fake_quant_q4_group(x: np.ndarray, search: bool = True) -> np.ndarray:
    """ef::fake_quant_q4_group (quant.h:58): Q4 quantize -> dequantize of one group of any size
    (the first min(n, 256) values are written; the rest of the result stays 0)."""
    x, px = _np(x, np.float32)
    out = np.zeros(x.size, dtype=np.float32)
    check(load().efg_host_fake_quant_q4_group(px, x.size, C.c_void_p(out.ctypes.data), int(search)))
    return out


def fake_quant_q4_group(x, n: int, out, search: bool = True) -> None:
    """efg_fake_quant_q4_group on CUDA tensors (torch's current stream)."""
    check(load().efg_fake_quant_q4_group(_ptr(x), n, _ptr(out), int(search), _stream()))


def host_dequantize_row(qtype: int, data: np.ndarray, n: int) -> np.ndarray:
    data, pd = _np(data, np.uint8)
    out = np.zeros(n, dtype=np.float32)
    check(load().efg_host_dequantize_row(int(qtype), pd, n, C.c_void_p(out.ctypes.data)))
    return out


def host_release_weights() -> None:
    check(load().efg_host_release_weights())


def host_matvec_static(qtype: int, W: np.ndarray, x: np.ndarray, rows: int) -> np.ndarray:
    """efg_host_matvec_static: host_matvec staged through the library's fixed 8 MiB device
    area (no device allocation; calls must not overlap)."""
    W, pw = _np(W, np.uint8)
    x, px = _np(x, np.float32)
    y = np.zeros(rows, dtype=np.float32)
    check(load().efg_host_matvec_static(int(qtype), C.c_void_p(y.ctypes.data), pw, px, rows, x.size))
    return y


# ---------------------------------------------------------------- batched GEMM


def gemm_q4_0(Y, W, X, M: int, K: int, B: int) -> None:
    """Y[b][m] = sum_k W[m][k] X[b][k] on the tensor cores: W packed Q4_0 [M] rows, X FP32
    [B][K], Y FP32 [B][M] (CUDA tensors). Each column equals ef::kern::matvec of that
    column within 1e-5 of sum|w x|."""
    check(load().efg_gemm_q4_0(_ptr(Y), _ptr(W), _ptr(X), M, K, B, _stream()))


def gemm_q8_0(Y, W, X, M: int, K: int, B: int) -> None:
    """gemm_q4_0 for Q8_0 weights (K a multiple of 256): each column equals
    ef::kern::matvec_q8_0 of that column within 1e-5 of sum|w x|."""
    check(load().efg_gemm_q8_0(_ptr(Y), _ptr(W), _ptr(X), M, K, B, _stream()))


def gemm_jobs(qtype: int, jobs, X, K: int, B: int, accumulate: bool = False) -> None:
    """efg_gemm_jobs: one launch for 1-3 (W, Y, M) matrices of one type sharing X; with
    `accumulate`, Y += W X."""
    n = len(jobs)
    Ws = (C.c_void_p * n)(*[_ptr(w).value for w, _, _ in jobs])
    Ys = (C.c_void_p * n)(*[_ptr(y).value for _, y, _ in jobs])
    Ms = (C.c_size_t * n)(*[m for _, _, m in jobs])
    check(load().efg_gemm_jobs(int(qtype), n, Ws, Ys, Ms, _ptr(X), K, B, int(accumulate), _stream()))


# ---------------------------------------------------------------- row-sharded matvec


def shard_rows(rows: int, nranks: int, rank: int) -> tuple[int, int]:
    """(begin, count) of rank's contiguous rows (ef::ThreadPool::chunk_begin split)."""
    b, c = C.c_size_t(0), C.c_size_t(0)
    check(load().efg_shard_rows(int(rows), int(nranks), int(rank), C.byref(b), C.byref(c)))
    return b.value, c.value


class Comm:
    """The library's NCCL communicator over the GPUs of one node (efg_comm_*)."""

    ID_BYTES = 128

    @staticmethod
    def unique_id() -> bytes:
        buf = (C.c_uint8 * Comm.ID_BYTES)()
        check(load().efg_comm_unique_id(C.cast(buf, C.c_void_p)))
        return bytes(buf)

    def __init__(self, uid: bytes, nranks: int, rank: int):
        if len(uid) != Comm.ID_BYTES:
            raise EdgeForgeError(1, "a communicator id is 128 bytes")
        buf = (C.c_uint8 * Comm.ID_BYTES).from_buffer_copy(uid)
        h = C.c_void_p(0)
        check(load().efg_comm_init(C.cast(buf, C.c_void_p), int(nranks), int(rank), C.byref(h)))
        self._h, self.nranks, self.rank = h, nranks, rank

    @classmethod
    def from_torch(cls, group=None) -> "Comm":
        """Every rank of a torch.distributed group joins one communicator (the id goes from
        rank 0 to the others through the group)."""
        import torch.distributed as dist

        rank, world = dist.get_rank(group), dist.get_world_size(group)
        obj = [cls.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0, group=group)
        return cls(obj[0], world, rank)

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    def register(self, buf) -> None:
        """efg_comm_register: every rank registers its own CUDA tensor of the same size, so
        that efg_matvec_sharded into it moves the slices by the kernel's own peer stores."""
        check(load().efg_comm_register(self._h, _ptr(buf), buf.numel() * buf.element_size()))

    def deregister(self, buf) -> None:
        check(load().efg_comm_deregister(self._h, _ptr(buf)))

    def close(self) -> None:
        if self._h:
            check(load().efg_comm_destroy(self._h))
            self._h = C.c_void_p(0)


def matvec_sharded(qtype: int, y, W_shard, x, rows: int, cols: int, comm: Comm) -> None:
    """Row-sharded matvec: W_shard = this rank's rows (shard_rows) of the packed [rows][cols]
    matrix; y (rows floats) receives the full result on every rank."""
    check(load().efg_matvec_sharded(int(qtype), _ptr(y), _ptr(W_shard), _ptr(x), rows, cols, comm.handle,
                                    _stream()))


def argmax(x, out=None):
    """efg_argmax (ef::kern::argmax): index of the first maximum of the CUDA float tensor x,
    written to `out` (a CUDA int32 tensor of one element, made if None); returns `out`."""
    import torch

    if out is None:
        out = torch.empty(1, dtype=torch.int32, device=x.device)
    check(load().efg_argmax(_ptr(x), x.numel(), _ptr(out), _stream()))
    return out


def lm_head_argmax_sharded(qtype: int, logits_shard, token, W_shard, x, norm_w, eps: float, rows: int, cols: int,
                           comm: Comm) -> None:
    """Row-sharded lm_head with the greedy argmax: this rank's logits into logits_shard, the
    argmax over all rows into token (CUDA int32, one element) on every rank."""
    check(load().efg_lm_head_argmax_sharded(int(qtype), _ptr(logits_shard) if logits_shard is not None else None,
                                            _ptr(token), _ptr(W_shard) if W_shard is not None else None, _ptr(x),
                                            _ptr(norm_w) if norm_w is not None else None, float(eps), rows, cols,
                                            comm.handle, _stream()))


# ---------------------------------------------------------------- .efq and the decode step


def efq_check(data: bytes | np.ndarray) -> None:
    """Validates an .efq file image (ef::parse_efq, src/qfile.cpp:125-223); raises
    EdgeForgeError carrying the reference's message on a malformed file."""
    buf = np.frombuffer(data, dtype=np.uint8) if isinstance(data, (bytes, bytearray)) else np.ascontiguousarray(data)
    check(load().efg_efq_check(C.c_void_p(buf.ctypes.data if buf.size else 0), buf.size))


def quantize_model(model_dir, out_file, policy: str = "auto", overrides: str = "") -> QuantizeReport:
    """ef::quantize_model (src/quantizer.cpp:151-290) on the GPU: config.json +
    model.safetensors -> .efq, byte-identical to the reference's writer."""
    rep = QuantizeReport()
    check(load().efg_quantize_model(str(model_dir).encode(), str(out_file).encode(), policy.encode(),
                                    overrides.encode(), C.byref(rep)))
    return rep


class GreedyResult:
    """ef::GreedyResult (include/ef/model.h:117-123)."""

    def __init__(self, tokens, step_logits, prefill_seconds, decode_seconds):
        self.tokens = tokens
        self.step_logits = step_logits
        self.prefill_seconds = prefill_seconds
        self.decode_seconds = decode_seconds
        self.decode_forwards = max(len(tokens) - 1, 0)


class Decoder:
    """ef::Model::load_efq + ef::Transformer (src/model.cpp:66-111, 153-276) on the GPU:
    the .efq's tensors are uploaded once, the KV cache is FP32 on the device, and one
    decode step is a recorded CUDA graph."""

    def __init__(self, efq_path, max_seq: int):
        h = C.c_void_p(0)
        check(load().efg_decoder_open(str(efq_path).encode(), int(max_seq), C.byref(h)))
        self._h = h
        info = ModelInfo()
        check(load().efg_decoder_info(h, C.byref(info)))
        self.info = info
        self.vocab = info.vocab
        self.max_seq = info.max_seq

    def close(self) -> None:
        if self._h:
            load().efg_decoder_close(self._h)
            self._h = C.c_void_p(0)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def bytes_per_token(self) -> int:
        """ef::Model::weight_bytes_per_token (src/qfile.cpp:237-241)."""
        return int(self.info.bytes_per_token)

    @property
    def persistent(self) -> bool:
        """True when the decode step runs as one persistent kernel; False (the default): a CUDA
        graph of one kernel per operation."""
        return load().efg_decoder_mode(self._h) == 1

    @persistent.setter
    def persistent(self, on: bool) -> None:
        check(load().efg_decoder_set_mode(self._h, int(bool(on))))

    def reset(self) -> None:
        check(load().efg_decoder_reset(self._h))

    def forward(self, token: int, pos: int, compute_logits: bool = True) -> np.ndarray | None:
        """ef::Transformer::forward: logits (vocab floats) or None."""
        out = np.empty(self.vocab, np.float32) if compute_logits else None
        check(load().efg_decoder_forward(self._h, int(token), int(pos),
                                         C.c_void_p(out.ctypes.data) if out is not None else None))
        return out

    def prefill(self, tokens, pos0: int = 0, compute_logits: bool = True) -> np.ndarray | None:
        """efg_decoder_prefill: tokens at positions pos0.. as one batch (Q4_0 projections on
        the tensor-core GEMM); the last token's logits or None."""
        arr = np.ascontiguousarray(tokens, np.int32)
        out = np.empty(self.vocab, np.float32) if compute_logits else None
        check(load().efg_decoder_prefill(self._h, C.c_void_p(arr.ctypes.data), len(arr), int(pos0),
                                         C.c_void_p(out.ctypes.data) if out is not None else None))
        return out

    def set_slots(self, n: int) -> None:
        """efg_decoder_set_slots: n sequence slots (0 = this decoder's own cache)."""
        check(load().efg_decoder_set_slots(self._h, int(n)))

    def step_slots(self, slots, tokens, positions, compute_logits: bool = True):
        """efg_decoder_step_slots: one step of several sequences; returns (logits
        [n][vocab] or None, argmax tokens [n])."""
        sl = np.ascontiguousarray(slots, np.int32)
        tk = np.ascontiguousarray(tokens, np.int32)
        ps = np.ascontiguousarray(positions, np.int32)
        n = len(sl)
        if len(tk) != n or len(ps) != n:
            raise EdgeForgeError(1, "step_slots: slots, tokens and positions differ in length")
        lg = np.empty((n, self.vocab), np.float32) if compute_logits else None
        nxt = np.empty(n, np.int32)
        check(load().efg_decoder_step_slots(self._h, C.c_void_p(sl.ctypes.data), C.c_void_p(tk.ctypes.data),
                                            C.c_void_p(ps.ctypes.data), n,
                                            C.c_void_p(lg.ctypes.data) if lg is not None else None,
                                            C.c_void_p(nxt.ctypes.data)))
        return lg, nxt

    def generate(self, prompt, max_new: int, eos_id: int = -1, forced=None,
                 keep_step_logits: bool = False) -> GreedyResult:
        """ef::generate_greedy (src/model.cpp:278-304). `forced` (max_new ids) teacher-forces
        the decode steps; the returned tokens are still each step's argmax."""
        prompt = np.ascontiguousarray(prompt, np.int32)
        toks = np.zeros(max(max_new, 1), np.int32)
        n = C.c_size_t(0)
        pf = C.c_double(0)
        dc = C.c_double(0)
        f = None
        if forced is not None:
            f = np.ascontiguousarray(forced, np.int32)
            if f.size != max_new:
                raise EdgeForgeError(1, "forced needs max_new ids")
        logits = np.zeros((max(max_new - 1, 0), self.vocab), np.float32) if keep_step_logits else None
        check(load().efg_decoder_generate(
            self._h, C.c_void_p(prompt.ctypes.data), prompt.size, int(max_new), int(eos_id),
            C.c_void_p(f.ctypes.data) if f is not None else None, C.c_void_p(toks.ctypes.data), C.byref(n),
            C.c_void_p(logits.ctypes.data) if logits is not None and logits.size else None,
            C.byref(pf), C.byref(dc)))
        k = n.value
        steps = logits[: max(k - 1, 0)] if logits is not None else None
        return GreedyResult(toks[:k].tolist(), steps, pf.value, dc.value)
