"""C-ABI checks that need no GPU: the library loads, exports every entry point that
include/qwb.h declares, and rejects malformed calls on the host before launching."""
import ctypes as C
import os
import re

import pytest

from questwend_b200 import _lib as L
from questwend_b200 import build as B

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for f in os.listdir(os.path.join(ROOT, "include")):
        if f.endswith(".h"):
            src = open(os.path.join(ROOT, "include", f)).read()
            names |= set(re.findall(r"QWB_API\s+[\w\s\*]*?\b(qwb_\w+)\s*\(", src))
    return names


@pytest.fixture(scope="module")
def lib():
    B.build()
    return L.lib()


def test_declared_symbols_exported(lib):
    names = declared_symbols()
    assert len(names) >= 13
    for n in sorted(names):
        assert hasattr(lib, n), n
    assert {n for n, _, _ in L.SIGNATURES} >= names


def test_abi_version_and_strings(lib):
    assert lib.qwb_abi_version() == 1
    for code, name in L.STATUS.items():
        assert lib.qwb_status_string(code)
    assert lib.qwb_status_string(999) == b"unknown status"


def _t(data, typ, ne, nb):
    d = L.Tensor()
    d.data, d.type = data, typ
    for i in range(4):
        d.ne[i], d.nb[i] = ne[i], nb[i]
    return d


def test_mul_mat_id_host_validation(lib):
    # as [512, 64, 8] Q4_K, b [512, 1, 5] f32, ids [3, 5] i32
    rs = 512 // 256 * 144
    a = _t(0x1000, L.Q4_K, (512, 64, 8, 1), (144, rs, rs * 64, rs * 64 * 8))
    b = _t(0x2000, L.F32, (512, 1, 5, 1), (4, 2048, 2048, 2048 * 5))
    ids = _t(0x3000, L.I32, (3, 5, 1, 1), (4, 12, 60, 60))
    dst = _t(0x4000, L.F32, (64, 3, 5, 1), (4, 256, 768, 3840))
    need = lib.qwb_mul_mat_id_workspace_size(C.byref(a), C.byref(b), C.byref(ids))
    assert need > 0
    # no workspace -> QWB_ERR_WORKSPACE, nothing launched
    assert lib.qwb_mul_mat_id(C.byref(a), C.byref(b), C.byref(ids), C.byref(dst), None, 0, None, None) == 6
    # unsupported weight type
    a_bad = _t(0x1000, 2, (512, 64, 8, 1), (18, rs, rs * 64, rs * 64 * 8))
    assert lib.qwb_mul_mat_id(C.byref(a_bad), C.byref(b), C.byref(ids), C.byref(dst), None, 0, None, None) == 2
    # K mismatch
    b_bad = _t(0x2000, L.F32, (256, 1, 5, 1), (4, 1024, 1024, 1024 * 5))
    assert lib.qwb_mul_mat_id(C.byref(a), C.byref(b_bad), C.byref(ids), C.byref(dst), None, 0, None, None) == 3
    # n_used % n_b != 0
    b2 = _t(0x2000, L.F32, (512, 2, 5, 1), (4, 2048, 4096, 4096 * 5))
    assert lib.qwb_mul_mat_id(C.byref(a), C.byref(b2), C.byref(ids), C.byref(dst), None, 0, None, None) == 3
    # misaligned Q4_K weights
    a_mis = _t(0x1004, L.Q4_K, (512, 64, 8, 1), (144, rs, rs * 64, rs * 64 * 8))
    assert lib.qwb_mul_mat_id(C.byref(a_mis), C.byref(b), C.byref(ids), C.byref(dst), 0x10000, need, None,
                              None) == 5


def test_get_rows_host_validation(lib):
    src = _t(0x1000, L.Q4_K, (512, 16, 1, 1), (144, 288, 288 * 16, 288 * 16))
    idx = _t(0x2000, L.I32, (8, 1, 1, 1), (4, 32, 32, 32))
    dst = _t(0x3000, L.F32, (512, 8, 1, 1), (4, 2048, 2048 * 8, 2048 * 8))
    bad_dst = _t(0x3000, L.I32, (512, 8, 1, 1), (4, 2048, 2048 * 8, 2048 * 8))
    assert lib.qwb_get_rows(C.byref(src), C.byref(idx), C.byref(bad_dst), None, None) == 2
    short = _t(0x3000, L.F32, (256, 8, 1, 1), (4, 1024, 1024 * 8, 1024 * 8))
    assert lib.qwb_get_rows(C.byref(src), C.byref(idx), C.byref(short), None, None) == 3
    empty = _t(0x2000, L.I32, (0, 1, 1, 1), (4, 0, 0, 0))
    dst0 = _t(0x3000, L.F32, (512, 0, 1, 1), (4, 2048, 0, 0))
    assert lib.qwb_get_rows(C.byref(src), C.byref(empty), C.byref(dst0), None, None) == 0


def test_quantizer_host_validation(lib):
    assert lib.qwb_quantize_row_q8_K(0x1000, 0x2000, 1, 100, 100, None) == 3  # k % 256
    assert lib.qwb_quantize_row_q8_0(0x1000, 0x2000, 1, 48, 48, 0, None) == 3  # k % 32
    assert lib.qwb_quantize_row_q8_0(0x1000, 0x2000, 1, 64, 64, 7, None) == 1  # bad variant
    assert lib.qwb_quantize_row_q8_K(0x1004, 0x2000, 1, 256, 256, None) == 5  # x misaligned
    assert lib.qwb_quantize_row_q8_K(0x1000, 0x2000, 0, 256, 256, None) == 0  # empty: no-op


def test_moe_route_limits(lib):
    assert lib.qwb_moe_route(0x1000, None, 2048, 1, 8, 1, 0.0, 0x2000, 0x3000, None) == 9
    assert lib.qwb_moe_route(0x1000, None, 128, 1, 64, 1, 0.0, 0x2000, 0x3000, None) == 9
    assert lib.qwb_moe_route(0x1000, None, 128, 0, 8, 1, 0.0, 0x2000, 0x3000, None) == 0


def test_moe_ffn_workspace_size(lib):
    H, F, E, k = 2048, 768, 128, 8
    rs_gu, rs_d = H // 256 * 144, F // 256 * 210
    d = L.MoeFfnDesc()
    d.gate = _t(0x1000, L.Q4_K, (H, F, E, 1), (144, rs_gu, rs_gu * F, rs_gu * F * E))
    d.up = _t(0x2000, L.Q4_K, (H, F, E, 1), (144, rs_gu, rs_gu * F, rs_gu * F * E))
    d.down = _t(0x3000, L.Q6_K, (F, H, E, 1), (210, rs_d, rs_d * H, rs_d * H * E))
    d.H, d.F, d.E, d.n_used, d.T = H, F, E, k, 1
    n1 = lib.qwb_moe_ffn_workspace_size(C.byref(d))
    d.T = 64
    n64 = lib.qwb_moe_ffn_workspace_size(C.byref(d))
    assert 0 < n1 < n64
    d.up.type = L.Q6_K  # gate and up must share a type
    assert lib.qwb_moe_ffn_workspace_size(C.byref(d)) == 0
