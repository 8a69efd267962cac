"""ctypes binding of libefg.so (the C ABI declared in include/efg.h).

The library is loaded from this package directory only. There is no fallback: if it
is missing, importing any operation raises, so a GPU run can never silently take a
CPU or PyTorch path.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libefg.so"

_vp, _sz, _i = C.c_void_p, C.c_size_t, C.c_int
_u64, _i32p = C.c_uint64, C.POINTER(C.c_int32)


class EdgeForgeError(RuntimeError):
    """A failed library call (the counterpart of ef::Error, include/ef/error.h:11-13)."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class MatvecJob(C.Structure):
    """efg_matvec_job (include/efg.h)."""

    _fields_ = [("d_y", _vp), ("qtype", _i), ("d_W", _vp), ("rows", _sz), ("cols", _sz), ("d_x", _vp)]


class QuantizeReport(C.Structure):
    """efg_quantize_report (include/efg.h)."""

    _fields_ = [("file_bytes", C.c_uint64), ("bytes_per_token", C.c_uint64), ("source_tensor_bytes", C.c_uint64),
                ("override_extra_bytes", C.c_int64), ("n_tensors", C.c_int32), ("seconds", C.c_double)]


class ModelInfo(C.Structure):
    """efg_model_info (include/efg.h)."""

    _fields_ = [(n, C.c_int32) for n in ("hidden", "intermediate", "layers", "heads", "kv_heads", "head_dim", "vocab",
                                          "max_seq", "n_q4", "n_q8", "embed_type")] + [("bytes_per_token", C.c_uint64)]


# name -> (restype, argtypes); every symbol include/efg.h declares.
SIGNATURES = {
    "efg_abi_version": (_i, []),
    "efg_last_error": (C.c_char_p, []),
    "efg_status_string": (C.c_char_p, [_i]),
    "efg_device_error": (_i, [C.POINTER(_i)]),
    "efg_set_weight_prefetch": (_i, [_i]),
    "efg_set_q4_mma": (_i, [_i]),
    "efg_set_small_gemm": (_i, [_i]),
    "efg_row_bytes": (_u64, [_i, _u64]),
    "efg_matvec_q4_0": (_i, [_vp, _vp, _vp, _sz, _sz, _vp]),
    "efg_matvec_q8_0": (_i, [_vp, _vp, _vp, _sz, _sz, _vp]),
    "efg_matvec": (_i, [_i, _vp, _vp, _vp, _sz, _sz, _vp]),
    "efg_matvec_jobs": (_i, [C.POINTER(MatvecJob), _sz, _vp]),
    "efg_dot_q4_0": (_i, [_vp, _vp, _vp, _sz, _vp]),
    "efg_dot_q8_0": (_i, [_vp, _vp, _vp, _sz, _vp]),
    "efg_quantize_row": (_i, [_i, _vp, _sz, _vp, _i, _vp]),
    "efg_dequantize_row": (_i, [_i, _vp, _sz, _vp, _vp]),
    "efg_quantize_rows": (_i, [_i, _vp, _sz, _sz, _vp, _i, _vp]),
    "efg_dequantize_rows": (_i, [_i, _vp, _sz, _sz, _vp, _vp]),
    "efg_row_f32": (_i, [_vp, _i, _vp, _sz, _sz, _i32p, _sz, _vp]),
    "efg_host_matvec": (_i, [_i, _vp, _vp, _vp, _sz, _sz]),
    "efg_host_quantize_row": (_i, [_i, _vp, _sz, _vp, _i]),
    "efg_host_fake_quant_q4_group": (_i, [_vp, _sz, _vp, _i]),
    "efg_fake_quant_q4_group": (_i, [_vp, _sz, _vp, _i, _vp]),
    "efg_host_dequantize_row": (_i, [_i, _vp, _sz, _vp]),
    "efg_host_register_weights": (_i, [_vp, _sz]),
    "efg_host_unregister_weights": (_i, [_vp]),
    "efg_host_release_weights": (_i, []),
    "efg_host_matvec_static": (_i, [_i, _vp, _vp, _vp, _sz, _sz]),
    "efg_gemm_q4_0": (_i, [_vp, _vp, _vp, _sz, _sz, _sz, _vp]),
    "efg_gemm_q8_0": (_i, [_vp, _vp, _vp, _sz, _sz, _sz, _vp]),
    "efg_gemm_jobs": (_i, [_i, _i, _vp, _vp, _vp, _vp, _sz, _sz, _i, _vp]),
    "efg_shard_rows": (_i, [_sz, _i, _i, C.POINTER(_sz), C.POINTER(_sz)]),
    "efg_comm_unique_id": (_i, [_vp]),
    "efg_comm_init": (_i, [_vp, _i, _i, C.POINTER(_vp)]),
    "efg_comm_destroy": (_i, [_vp]),
    "efg_comm_register": (_i, [_vp, _vp, _sz]),
    "efg_comm_deregister": (_i, [_vp, _vp]),
    "efg_matvec_sharded": (_i, [_i, _vp, _vp, _vp, _sz, _sz, _vp, _vp]),
    "efg_argmax": (_i, [_vp, _sz, _vp, _vp]),
    "efg_lm_head_argmax_sharded": (_i, [C.c_int, _vp, _vp, _vp, _vp, _vp, C.c_float, _sz, _sz, _vp, _vp]),
    "efg_efq_check": (_i, [_vp, _u64]),
    "efg_quantize_model": (_i, [C.c_char_p, C.c_char_p, C.c_char_p, C.c_char_p, C.POINTER(QuantizeReport)]),
    "efg_decoder_open": (_i, [C.c_char_p, _sz, C.POINTER(_vp)]),
    "efg_decoder_close": (_i, [_vp]),
    "efg_decoder_info": (_i, [_vp, C.POINTER(ModelInfo)]),
    "efg_decoder_reset": (_i, [_vp]),
    "efg_decoder_forward": (_i, [_vp, C.c_int32, _sz, _vp]),
    "efg_decoder_prefill": (_i, [_vp, _vp, _sz, _sz, _vp]),
    "efg_decoder_set_slots": (_i, [_vp, _sz]),
    "efg_decoder_step_slots": (_i, [_vp, _vp, _vp, _vp, _sz, _vp, _vp]),
    "efg_decoder_set_mode": (_i, [_vp, _i]),
    "efg_decoder_mode": (_i, [_vp]),
    "efg_decoder_generate": (_i, [_vp, _vp, _sz, _sz, C.c_int32, _vp, _vp, C.POINTER(_sz), _vp,
                                  C.POINTER(C.c_double), C.POINTER(C.c_double)]),
}

_lib = None


def load() -> C.CDLL:
    """Loads libefg.so once and binds every declared symbol (raises if any is missing)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is not built: run `python -c 'import __graft_entry__ as g; g.build()'`")
        lib = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            f = getattr(lib, name)
            f.restype = res
            f.argtypes = args
        _lib = lib
    return _lib


def check(status: int) -> None:
    if status != 0:
        lib = load()
        raise EdgeForgeError(status, f"{lib.efg_status_string(status).decode()}: {lib.efg_last_error().decode()}")
