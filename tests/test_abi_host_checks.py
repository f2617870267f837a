"""Host-side argument checks of the remaining C entry points, without a GPU: every call
here returns from its checks before any CUDA call (fake device addresses are never
dereferenced)."""
import ctypes as C

import pytest

from questwend_b200 import _lib as L
from questwend_b200 import build as B

OK, INVALID, UNSUPPORTED, SHAPE, LIMIT, WORKSPACE = 0, 1, 2, 3, 9, 6


@pytest.fixture(scope="module")
def lib():
    B.build()
    return L.lib()


def _t(data, typ, ne, nb):
    d = L.Tensor()
    d.data, d.type = data, typ
    for i in range(4):
        d.ne[i], d.nb[i] = ne[i], nb[i]
    return d


def test_swiglu_checks(lib):
    assert lib.qwb_swiglu(0x1000, 0x2000, 0x3000, -1, None) == INVALID
    assert lib.qwb_swiglu(None, None, None, 0, None) == OK  # empty: nothing to do
    assert lib.qwb_swiglu(None, 0x2000, 0x3000, 16, None) == INVALID


def test_weighted_sum_checks(lib):
    assert lib.qwb_moe_weighted_sum(0x1000, 0x2000, 0x3000, -1, 8, 1, None) == INVALID
    assert lib.qwb_moe_weighted_sum(0x1000, 0x2000, 0x3000, 2048, 0, 1, None) == INVALID
    assert lib.qwb_moe_weighted_sum(None, None, None, 2048, 8, 0, None) == OK
    assert lib.qwb_moe_weighted_sum(0x1000, None, 0x3000, 2048, 8, 1, None) == INVALID


def test_mul_mat_checks(lib):
    K, M, T = 2048, 300, 4
    rs = K // 256 * 144
    a = _t(0x10000, L.Q4_K, (K, M, 1, 1), (144, rs, rs * M, rs * M))
    b = _t(0x20000, L.F32, (K, T, 1, 1), (4, 4 * K, 4 * K * T, 4 * K * T))
    dst = _t(0x30000, L.F32, (M, T, 1, 1), (4, 4 * M, 4 * M * T, 4 * M * T))
    need = lib.qwb_mul_mat_workspace_size(C.byref(a), C.byref(b))
    assert need > 0
    # K mismatch, batched a: no workspace size, shape errors
    b_bad = _t(0x20000, L.F32, (K // 2, T, 1, 1), (4, 2 * K, 2 * K * T, 2 * K * T))
    assert lib.qwb_mul_mat_workspace_size(C.byref(a), C.byref(b_bad)) == 0
    a3 = _t(0x10000, L.Q4_K, (K, M, 2, 1), (144, rs, rs * M, rs * M * 2))
    assert lib.qwb_mul_mat_workspace_size(C.byref(a3), C.byref(b)) == 0
    assert lib.qwb_mul_mat(C.byref(a), C.byref(b_bad), C.byref(dst), 0x40000, need, None, None) == SHAPE
    dst_bad = _t(0x30000, L.F32, (M + 1, T, 1, 1), (4, 4 * M + 4, 4 * (M + 1) * T, 4 * (M + 1) * T))
    assert lib.qwb_mul_mat(C.byref(a), C.byref(b), C.byref(dst_bad), 0x40000, need, None, None) == SHAPE
    assert lib.qwb_mul_mat(C.byref(a), C.byref(b), None, 0x40000, need, None, None) == INVALID
    # missing workspace is reported before anything is queued
    assert lib.qwb_mul_mat(C.byref(a), C.byref(b), C.byref(dst), None, 0, None, None) == WORKSPACE
    # no tokens: nothing to do
    b0 = _t(0x20000, L.F32, (K, 0, 1, 1), (4, 4 * K, 0, 0))
    d0 = _t(0x30000, L.F32, (M, 0, 1, 1), (4, 4 * M, 0, 0))
    assert lib.qwb_mul_mat(C.byref(a), C.byref(b0), C.byref(d0), None, 0, None, None) == OK


def test_expert_parallel_workspace_queries(lib):
    H, F, E, n_loc = 2048, 768, 128, 16
    rg, rd = H // 256 * 144, F // 256 * 210
    p = L.MoeEpLayerDesc()
    p.gate = _t(0x100000, L.Q4_K, (H, F, n_loc, 1), (144, rg, rg * F, rg * F * n_loc))
    p.up = _t(0x200000, L.Q4_K, (H, F, n_loc, 1), (144, rg, rg * F, rg * F * n_loc))
    p.down = _t(0x300000, L.Q6_K, (F, H, n_loc, 1), (210, rd, rd * H, rd * H * n_loc))
    p.expert_lo, p.H, p.F, p.E, p.n_used, p.T = 32, H, F, E, 8, 8
    assert lib.qwb_moe_ep_layer_workspace_size(C.byref(p)) > 0
    p.expert_lo = E - n_loc + 1
    assert lib.qwb_moe_ep_layer_workspace_size(C.byref(p)) == 0  # shard past the last expert
    p.expert_lo, p.H = 0, 2000
    assert lib.qwb_moe_ep_layer_workspace_size(C.byref(p)) == 0  # H % 1024
    p.H, p.n_used = H, 200
    assert lib.qwb_moe_ep_layer_workspace_size(C.byref(p)) == 0  # more experts used than exist
    assert lib.qwb_moe_ep_layer(C.byref(p), None, 0, None, None) == LIMIT
    p.n_used, p.up.type = 8, L.Q6_K
    assert lib.qwb_moe_ep_layer(C.byref(p), None, 0, None, None) == UNSUPPORTED  # gate and up differ
    p.up.type, p.T = L.Q4_K, 0
    assert lib.qwb_moe_ep_layer(C.byref(p), None, 0, None, None) == OK  # no tokens
    p.T = 4
    assert lib.qwb_moe_ep_layer(C.byref(p), None, 0, None, None) == INVALID  # no x / router / out


def test_noalloc_limit_without_gpu(lib):
    # a problem whose workspace exceeds the fixed scratch array is refused before any
    # device call; malformed shapes report the regular entry point's status
    K, M, n_as, T, n_used = 4096, 1536, 128, 8192, 8
    rs = K // 256 * 144
    a = _t(0x100000, L.Q4_K, (K, M, n_as, 1), (144, rs, rs * M, rs * M * n_as))
    b = _t(0x200000, L.F32, (K, 1, T, 1), (4, 4 * K, 4 * K, 4 * K * T))
    ids = _t(0x300000, L.I32, (n_used, T, 1, 1), (4, 4 * n_used, 4 * n_used * T, 4 * n_used * T))
    dst = _t(0x400000, L.F32, (M, n_used, T, 1), (4, 4 * M, 4 * M * n_used, 4 * M * n_used * T))
    assert lib.qwb_mul_mat_id_noalloc(C.byref(a), C.byref(b), C.byref(ids), C.byref(dst), None, None) == LIMIT
    b_bad = _t(0x200000, L.F32, (K // 2, 1, T, 1), (4, 2 * K, 2 * K, 2 * K * T))
    assert lib.qwb_mul_mat_id_noalloc(C.byref(a), C.byref(b_bad), C.byref(ids), C.byref(dst), None, None) == SHAPE
    a_bad = _t(0x100000, 2, (K, M, n_as, 1), (18, rs, rs * M, rs * M * n_as))
    assert lib.qwb_mul_mat_id_noalloc(C.byref(a_bad), C.byref(b), C.byref(ids), C.byref(dst), None,
                                      None) == UNSUPPORTED


def test_ep_comm_argument_checks(lib):
    # refused before any CUDA call
    assert lib.qwb_ep_comm_handle_size() > 0
    h = (C.c_char * lib.qwb_ep_comm_handle_size())()
    p = C.c_void_p()
    assert lib.qwb_ep_comm_create(2, 2, 1 << 20, C.byref(p), h) == INVALID   # rank outside the world
    assert lib.qwb_ep_comm_create(0, 0, 1 << 20, C.byref(p), h) == INVALID
    assert lib.qwb_ep_comm_create(2, 0, 0, C.byref(p), h) == INVALID        # no message size
    assert lib.qwb_ep_comm_create(16, 0, 1 << 20, C.byref(p), h) == LIMIT   # more GPUs than one node's 8
    assert lib.qwb_ep_comm_create(2, 0, 1 << 20, None, h) == INVALID
    assert lib.qwb_ep_comm_connect(None, h) == INVALID
    assert lib.qwb_ep_allreduce_f32(None, 0x1000, 0x1000, 16, None, None) == INVALID
    lib.qwb_ep_comm_destroy(None)  # no-op
