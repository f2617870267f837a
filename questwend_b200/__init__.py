"""questwend_b200 - B200 (sm_100a) kernels for QuestWend's quantized MoE expert hot path.

The compute lives in libqwb.so (hand-written CUDA, C ABI in include/qwb.h); this
package is its host-side mirror of the ggml operators (``ops``) and the build script.
Importing it does not touch the GPU; the first op call loads libqwb.so and fails loudly
if it is missing.
"""
from . import ops  # noqa: F401
from ._lib import LIB_PATH, QwbError, lib  # noqa: F401
from .ops import (QTensor, get_rows, moe_ffn, moe_route, moe_weighted_sum, mul_mat, mul_mat_id,  # noqa: F401
                  pool_audit_slabs, pool_write_slabs, quantize_q8_0, quantize_q8_K, read_status, swiglu)
