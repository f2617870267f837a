"""ctypes binding of libqwb.so (the C ABI declared in include/qwb.h).

The library is built in-tree by ``questwend_b200.build``.  There is no fallback: if the
shared object is missing or cannot be loaded, every entry point raises.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqwb.so")

# ggml enum ggml_type values
F32, F16, Q8_0, Q4_K, Q6_K, Q8_K, I32 = 0, 1, 8, 12, 14, 15, 26
Q8_0_CPU, Q8_0_REF = 0, 1

STATUS = {
    0: "QWB_OK", 1: "QWB_ERR_INVALID_ARG", 2: "QWB_ERR_UNSUPPORTED_TYPE", 3: "QWB_ERR_SHAPE",
    4: "QWB_ERR_LAYOUT", 5: "QWB_ERR_ALIGNMENT", 6: "QWB_ERR_WORKSPACE", 7: "QWB_ERR_CUDA",
    8: "QWB_ERR_DEVICE", 9: "QWB_ERR_LIMIT",
}
DEVERR_ID_RANGE, DEVERR_ROW_RANGE, DEVERR_TIMEOUT = 1, 2, 4
NOALLOC_SCRATCH_BYTES = 8 << 20  # QWB_NOALLOC_SCRATCH_BYTES


class QwbError(RuntimeError):
    """A qwb entry point returned a non-zero qwb_status."""

    def __init__(self, fn: str, code: int):
        super().__init__(f"{fn} failed: {STATUS.get(code, code)}")
        self.code = code


class Tensor(C.Structure):
    """struct qwb_tensor: data, type, reserved, ne[4], nb[4] (bytes)."""
    _fields_ = [("data", C.c_void_p), ("type", C.c_int32), ("reserved", C.c_int32),
                ("ne", C.c_int64 * 4), ("nb", C.c_size_t * 4)]


class StatusBlock(C.Structure):
    _fields_ = [("flags", C.c_uint32), ("bad_value", C.c_int32), ("count", C.c_uint32),
                ("reserved", C.c_uint32)]


class MoeFfnDesc(C.Structure):
    _fields_ = [("x", C.c_void_p), ("router_w", C.c_void_p), ("mask", C.c_void_p), ("g2s", C.c_void_p),
                ("gate", Tensor), ("up", Tensor), ("down", Tensor),
                ("H", C.c_int64), ("F", C.c_int64), ("E", C.c_int64), ("n_used", C.c_int64),
                ("T", C.c_int64), ("residual", C.c_void_p), ("out", C.c_void_p),
                ("selected", C.c_void_p), ("weights", C.c_void_p), ("act", C.c_void_p),
                ("norm_w", C.c_void_p), ("norm_eps", C.c_float),
                ("shexp_gate", Tensor), ("shexp_up", Tensor), ("shexp_down", Tensor),
                ("shexp_gate_inp", C.c_void_p)]


class MoeEpLayerDesc(C.Structure):
    _fields_ = [("x", C.c_void_p), ("norm_w", C.c_void_p), ("norm_eps", C.c_float), ("reserved", C.c_int32),
                ("router_w", C.c_void_p), ("mask", C.c_void_p),
                ("gate", Tensor), ("up", Tensor), ("down", Tensor), ("expert_lo", C.c_int64),
                ("H", C.c_int64), ("F", C.c_int64), ("E", C.c_int64), ("n_used", C.c_int64), ("T", C.c_int64),
                ("residual", C.c_void_p), ("out", C.c_void_p), ("selected", C.c_void_p), ("weights", C.c_void_p),
                ("shexp_gate", Tensor), ("shexp_up", Tensor), ("shexp_down", Tensor),
                ("shexp_gate_inp", C.c_void_p)]


_lib = None

# (name, restype, argtypes) for every QWB_API symbol of include/qwb.h
_P, _TP = C.c_void_p, C.POINTER(Tensor)
class SlabCopy(C.Structure):
    """struct qwb_slab_copy: a slab's bytes and its pool slot."""
    _fields_ = [("src", C.c_void_p), ("slot", C.c_int64)]


class SlabAudit(C.Structure):
    """struct qwb_slab_audit: the byte audit record of one pool slot."""
    _fields_ = [("equal", C.c_int32), ("reserved", C.c_int32), ("first_difference", C.c_uint64),
                ("expected_byte", C.c_uint32), ("actual_byte", C.c_uint32),
                ("expected_fnv1a64", C.c_uint64), ("actual_fnv1a64", C.c_uint64)]


SIGNATURES = [
    ("qwb_abi_version", C.c_int, []),
    ("qwb_status_string", C.c_char_p, [C.c_int]),
    ("qwb_status_block_read", C.c_int, [_P, C.POINTER(StatusBlock), C.c_int, _P]),
    ("qwb_quantize_row_q8_K", C.c_int, [_P, _P, C.c_int64, C.c_int64, C.c_int64, _P]),
    ("qwb_quantize_row_q8_0", C.c_int, [_P, _P, C.c_int64, C.c_int64, C.c_int64, C.c_int, _P]),
    ("qwb_get_rows", C.c_int, [_TP, _TP, _TP, _P, _P]),
    ("qwb_mul_mat_id_workspace_size", C.c_size_t, [_TP, _TP, _TP]),
    ("qwb_mul_mat_id", C.c_int, [_TP, _TP, _TP, _TP, _P, C.c_size_t, _P, _P]),
    ("qwb_mul_mat_workspace_size", C.c_size_t, [_TP, _TP]),
    ("qwb_mul_mat", C.c_int, [_TP, _TP, _TP, _P, C.c_size_t, _P, _P]),
    ("qwb_mul_mat_id_noalloc", C.c_int, [_TP, _TP, _TP, _TP, _P, _P]),
    ("qwb_moe_route", C.c_int, [_P, _P, C.c_int64, C.c_int64, C.c_int64, C.c_int, C.c_float, _P, _P, _P]),
    ("qwb_swiglu", C.c_int, [_P, _P, _P, C.c_int64, _P]),
    ("qwb_moe_weighted_sum", C.c_int, [_P, _P, _P, C.c_int64, C.c_int64, C.c_int64, _P]),
    ("qwb_moe_ffn_workspace_size", C.c_size_t, [C.POINTER(MoeFfnDesc)]),
    ("qwb_moe_ffn", C.c_int, [C.POINTER(MoeFfnDesc), _P, C.c_size_t, _P, _P]),
    ("qwb_moe_ep_layer_workspace_size", C.c_size_t, [C.POINTER(MoeEpLayerDesc)]),
    ("qwb_moe_ep_layer", C.c_int, [C.POINTER(MoeEpLayerDesc), _P, C.c_size_t, _P, _P]),
    ("qwb_ep_comm_handle_size", C.c_size_t, []),
    ("qwb_ep_comm_create", C.c_int, [C.c_int, C.c_int, C.c_size_t, C.POINTER(C.c_void_p), _P]),
    ("qwb_ep_comm_connect", C.c_int, [_P, _P]),
    ("qwb_ep_allreduce_f32", C.c_int, [_P, _P, _P, C.c_int64, _P, _P]),
    ("qwb_ep_comm_destroy", None, [_P]),
    ("qwb_pool_write_slabs", C.c_int, [_TP, C.c_size_t, C.POINTER(SlabCopy), C.c_int, _P]),
    ("qwb_pool_audit_slabs", C.c_int, [_TP, C.POINTER(SlabCopy), C.c_int, C.c_int, _P, _P]),
    ("qwb_profile_enable", C.c_int, [C.c_int]),
    ("qwb_profile_reset", C.c_int, []),
    ("qwb_profile_count", C.c_int, []),
    ("qwb_profile_read", C.c_int, [C.POINTER(C.c_float), C.POINTER(C.c_int32), C.c_int]),
]


def lib():
    """Load libqwb.so (raises if it is missing: there is no CPU fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m questwend_b200.build`")
        L = C.CDLL(LIB_PATH)
        for name, res, args in SIGNATURES:
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(fn: str, code: int):
    if code != 0:
        raise QwbError(fn, code)
