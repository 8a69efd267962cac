"""EdgeForge-B200: EdgeForge's packed Q4_0/Q8_0 matrix-product path on NVIDIA B200.

The compute path is libefg.so (hand-written sm_100a CUDA behind the C ABI in
include/efg.h); this package is the Python mirror of the reference's kernel API over it.
"""
from ._lib import EdgeForgeError, LIB_PATH, load  # noqa: F401
from .api import (  # noqa: F401
    BLOCK_BYTES,
    Comm,
    Decoder,
    GreedyResult,
    QK,
    QType,
    dequantize_row,
    dequantize_rows,
    device_error,
    dot_q4_0,
    dot_q8_0,
    efq_check,
    fake_quant_q4_group,
    gemm_q4_0,
    gemm_q8_0,
    gemm_jobs,
    host_dequantize_row,
    host_fake_quant_q4_group,
    host_matvec,
    host_matvec_static,
    host_quantize_row,
    host_register_weights,
    host_unregister_weights,
    host_release_weights,
    matvec,
    matvec_jobs,
    matvec_q4_0,
    matvec_q8_0,
    argmax,
    lm_head_argmax_sharded,
    matvec_sharded,
    quantize_model,
    quantize_row,
    quantize_rows,
    row_bytes,
    row_f32,
    set_q4_mma,
    set_small_gemm,
    set_weight_prefetch,
    shard_rows,
)

__version__ = "0.1.0"
