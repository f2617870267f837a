"""GPU parity: MUL_MAT_ID through the tensor-core grouped GEMM (many tokens per expert).

qwb_mul_mat_id takes the tcgen05 path for Q4_K weights when the routed (token, slot)
pairs average at least 32 per used expert.  Bar: normalized RMS error <= 1e-4 against
the CPU oracle on the same inputs (the superblock sums are exact integers in f32; the
min term carries a ~2^-22 relative error from its hi/lo fp16 split); the max abs-rel
error is reported in the assertion message.  The GEMV path (qwb_mul_mat_id_noalloc
keeps it at every size) is compared on the same inputs."""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle as O
import _data as D

pytestmark = pytest.mark.gpu
TOL = 1e-4


@pytest.fixture(scope="module")
def qwb():
    import questwend_b200 as q
    q.lib()
    return q


def cu(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _gemv(q, W, b, ids, out):
    from questwend_b200 import _lib as L
    ad, bd, idd, od = q.ops.desc(W), q.ops.desc(b), q.ops.desc(ids), q.ops.desc(out)
    rc = L.lib().qwb_mul_mat_id_noalloc(C.byref(ad), C.byref(bd), C.byref(idd), C.byref(od),
                                       q.ops.status_block().data_ptr(),
                                       C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    return out


def _ws_bytes(q, W, b, ids):
    from questwend_b200 import _lib as L
    ad, bd, idd = q.ops.desc(W), q.ops.desc(b), q.ops.desc(ids)
    return L.lib().qwb_mul_mat_id_workspace_size(C.byref(ad), C.byref(bd), C.byref(idd))


def _check(qwb, w, K, M, n_as, b, ids, ref=False):
    t = O.Q4_K
    W = qwb.QTensor.from_bytes(w, t, (K, M, n_as))
    bb, ii = cu(b), cu(ids)
    # the tensor-core path carries fp16 B tiles: its workspace dwarfs the GEMV's
    assert _ws_bytes(qwb, W, bb, ii) > 2 * ids.size * K
    got = qwb.mul_mat_id(W, bb, ii).cpu().numpy()
    st = qwb.ops.read_status()
    want, rc = O.mul_mat_id(t, w, K, M, n_as, b, ids, impl="ref" if ref else "port")
    assert ref or rc == 0
    e = O.nrmse(got, want)
    assert e <= TOL, (e, O.max_abs_rel(got, want))
    return got, want, st


CASES = [
    # K, M, n_as, T, n_used, n_b
    (2048, 768, 16, 256, 8, 1),    # gate/up shape
    (768, 2048, 8, 128, 8, 8),     # down shape (b = act per slot), several token tiles per expert
    (512, 200, 4, 64, 4, 1),       # partial weight tile (M % 128 != 0)
    (256, 128, 2, 80, 1, 1),       # one superblock, ragged token tiles
]


@pytest.mark.parametrize("K,M,n_as,T,n_used,n_b", CASES)
def test_uniform_routing(qwb, K, M, n_as, T, n_used, n_b):
    w = D.weights(O.Q4_K, n_as, M, K, seed=K + 3 * M + T)
    b = D.acts((T, n_b, K), seed=T + 7)
    r = D.rng(T + 11)
    ids = np.stack([r.choice(n_as, n_used, replace=False) for _ in range(T)]).astype(np.int32)
    _check(qwb, w, K, M, n_as, b, ids)


def test_zipf_routing_against_reference_build(qwb):
    # skewed routing: 0 to several hundred pairs per expert; checked against the reference's
    # own ggml CPU backend (its tiled path takes experts with >= 8 rows)
    K, M, n_as, T, n_used = 1024, 256, 128, 512, 8
    w = D.weights(O.Q4_K, n_as, M, K, seed=77)
    b = D.acts((T, 1, K), seed=78)
    ids = D.zipf_ids(T, n_as, n_used, seed=79)
    counts = np.bincount(ids.ravel(), minlength=n_as)
    assert counts.max() > 128 and (counts < 8).any()
    O.set_ref_threads(8)
    got, want, _ = _check(qwb, w, K, M, n_as, b, ids, ref=O.ref_available())


def test_matches_gemv_path(qwb):
    K, M, n_as, T, n_used = 1024, 384, 8, 96, 8
    w = D.weights(O.Q4_K, n_as, M, K, seed=90)
    b = D.acts((T, 1, K), seed=91)
    ids = np.stack([D.rng(92 + i).permutation(n_as)[:n_used] for i in range(T)]).astype(np.int32)
    got, want, _ = _check(qwb, w, K, M, n_as, b, ids)
    W = qwb.QTensor.from_bytes(w, O.Q4_K, (K, M, n_as))
    out = torch.empty((T, n_used, M), dtype=torch.float32, device="cuda")
    gv = _gemv(qwb, W, cu(b), cu(ids), out).cpu().numpy()
    assert O.nrmse(gv, got) <= TOL


def test_degenerate_superblock_scales(qwb):
    # superblocks with d = 0, with d tiny against dmin, and with d = dmin = 0: the kernel
    # switches the row scale to dmin (or zero) there; results still match the oracle
    K, M, n_as, T, n_used = 512, 128, 2, 64, 2
    w = D.weights(O.Q4_K, n_as, M, K, seed=31).copy()
    rb = O.row_size(O.Q4_K, K)
    v = w.view(np.uint8).reshape(n_as * M, rb)
    h = lambda x: np.frombuffer(np.float16(x).tobytes(), np.uint8)
    for row in range(0, n_as * M, 7):
        sb = (row // 7) % 2
        o = sb * 144
        kind = (row // 7) % 3
        if kind == 0:
            v[row, o:o + 2] = h(0.0)                     # d = 0
        elif kind == 1:
            v[row, o:o + 2] = h(1e-7)                    # d << dmin
        else:
            v[row, o:o + 4] = 0                          # d = dmin = 0
    b = D.acts((T, 1, K), seed=32)
    ids = np.stack([np.arange(n_as) for _ in range(T)]).astype(np.int32)
    _check(qwb, w, K, M, n_as, b, ids)


def test_out_of_range_ids_zero_rows(qwb):
    K, M, n_as, T, n_used = 512, 128, 4, 64, 4
    w = D.weights(O.Q4_K, n_as, M, K, seed=41)
    b = D.acts((T, 1, K), seed=42)
    ids = np.stack([np.arange(n_as) for _ in range(T)]).astype(np.int32)
    ids[5, 2] = n_as + 3
    ids[9, 0] = -1
    W = qwb.QTensor.from_bytes(w, O.Q4_K, (K, M, n_as))
    qwb.ops.read_status()
    got = qwb.mul_mat_id(W, cu(b), cu(ids)).cpu().numpy()
    flags, bad, count = qwb.ops.read_status()
    assert flags & 1 and count >= 2
    assert not got[5, 2].any() and not got[9, 0].any()
    ok = ids.copy()
    ok[5, 2] = 0
    ok[9, 0] = 0
    want, _ = O.mul_mat_id(O.Q4_K, w, K, M, n_as, b, ok)
    mask = np.ones((T, n_used), bool)
    mask[5, 2] = mask[9, 0] = False
    assert O.nrmse(got[mask], want[mask]) <= TOL
