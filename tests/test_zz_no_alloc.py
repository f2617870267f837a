"""qwb_mul_mat_id_noalloc: MUL_MAT_ID for callers that cannot allocate device memory.

Callers such as a ggml backend's graph_compute, code running under someone else's CUDA
graph capture, or a host whose device memory is fully committed to its expert pool can
neither allocate nor hand over a workspace; this entry point runs from scratch space the
library carries in its own device image.  The tests drive it through the C ABI and
compare it with qwb_mul_mat_id (which takes a caller workspace) at the tolerance the other
MUL_MAT_ID tests use:
  * two calls in a row, the larger first, so the second runs over the first's leftovers;
  * a Q4_K batch with many tokens per expert, where qwb_mul_mat_id_workspace_size (which
    also plans for the tensor-core GEMM) is over the scratch size but the GEMV plan this
    entry point uses fits: it is accepted and matches the oracle;
  * the size limit: the largest accepted batch is computed correctly and one token more
    is refused with QWB_ERR_LIMIT.
It is collected last (file name) so a failing run that stops at the first failure has run
every other test first."""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle as O
import _data as D

pytestmark = pytest.mark.gpu
TOL = 1e-4
QWB_ERR_LIMIT = 9


@pytest.fixture(scope="module")
def qwb():
    import questwend_b200 as q
    q.lib()
    return q


def _noalloc(q, W, b, ids, out):
    from questwend_b200 import _lib as L
    ad, bd, idd, od = q.ops.desc(W), q.ops.desc(b), q.ops.desc(ids), q.ops.desc(out)
    return L.lib().qwb_mul_mat_id_noalloc(C.byref(ad), C.byref(bd), C.byref(idd), C.byref(od),
                                         q.ops.status_block().data_ptr(),
                                         C.c_void_p(torch.cuda.current_stream().cuda_stream))


def _workspace_size(q, W, b, ids):
    from questwend_b200 import _lib as L
    return L.lib().qwb_mul_mat_id_workspace_size(C.byref(q.ops.desc(W)), C.byref(q.ops.desc(b)),
                                                 C.byref(q.ops.desc(ids)))


def _ids(T, n_as, n_used, seed):
    return torch.from_numpy(np.stack([D.rng(seed + i).choice(n_as, n_used, replace=False)
                                      for i in range(T)]).astype(np.int32)).cuda()


def test_noalloc_matches_workspace_entry_point_twice(qwb):
    t, K, M, n_as = O.Q4_K, 2048, 768, 32
    W = qwb.QTensor.from_bytes(D.weights(t, n_as, M, K, seed=77), t, (K, M, n_as))
    qwb.read_status()
    # the larger call first: the second call reads scratch bytes the first one left
    for call, (T, n_used) in enumerate(((64, 8), (3, 6))):
        b = torch.from_numpy(D.acts((T, 1, K), seed=100 + call)).cuda()
        ids = _ids(T, n_as, n_used, 200 + call * 100)
        want = qwb.mul_mat_id(W, b, ids).clone()
        got = torch.full_like(want, float("nan"))
        assert _noalloc(qwb, W, b, ids, got) == 0
        torch.cuda.synchronize()
        e = O.nrmse(got.cpu().numpy(), want.cpu().numpy())
        assert e <= TOL, (call, e)
    assert qwb.read_status()[0] == 0


def test_noalloc_accepts_tensor_core_sized_batch_within_gemv_plan(qwb):
    from questwend_b200 import _lib as L
    # 8 experts, every token selects all 8: 128 pairs per expert, the tensor-core size for
    # qwb_mul_mat_id, whose fp16 B tiles alone (~9.4 MB) are over the scratch size
    t, K, M, n_as, n_used, T = O.Q4_K, 4096, 256, 8, 8, 128
    w = D.weights(t, n_as, M, K, seed=31)
    W = qwb.QTensor.from_bytes(w, t, (K, M, n_as))
    x = D.acts((T, 1, K), seed=32)
    b = torch.from_numpy(x).cuda()
    ids_np = np.stack([D.rng(33 + i).permutation(n_as) for i in range(T)]).astype(np.int32)
    ids = torch.from_numpy(ids_np).cuda()
    assert _workspace_size(qwb, W, b, ids) > L.NOALLOC_SCRATCH_BYTES
    got = torch.full((T, n_used, M), float("nan"), device="cuda")
    assert _noalloc(qwb, W, b, ids, got) == 0
    torch.cuda.synchronize()
    want, rc = O.mul_mat_id(t, w, K, M, n_as, x, ids_np)
    assert rc == 0
    e = O.nrmse(got.cpu().numpy(), want)
    assert e <= TOL, e


def test_noalloc_limit_boundary(qwb):
    from questwend_b200 import _lib as L
    t, K, M, n_as, n_used = O.Q8_0, 4096, 64, 8, 8
    W = qwb.QTensor.from_bytes(D.weights(t, n_as, M, K, seed=5), t, (K, M, n_as))

    def call(T, b=None, ids=None, out=None):
        b = torch.zeros((T, 1, K), device="cuda") if b is None else b
        ids = torch.zeros((T, n_used), dtype=torch.int32, device="cuda") if ids is None else ids
        out = torch.empty((T, n_used, M), device="cuda") if out is None else out
        return _noalloc(qwb, W, b, ids, out)

    # the largest accepted token count (accepted sizes form a prefix: the plan grows with T)
    lo, hi = 1, 4096
    assert call(lo) == 0 and call(hi) == QWB_ERR_LIMIT
    while hi - lo > 1:
        mid = (lo + hi) // 2
        rc = call(mid)
        assert rc in (0, QWB_ERR_LIMIT), rc
        lo, hi = (mid, hi) if rc == 0 else (lo, mid)
    torch.cuda.synchronize()
    T = lo
    # one token more is refused, and the public query agrees it does not fit
    b1 = torch.zeros((T + 1, 1, K), device="cuda")
    ids1 = torch.zeros((T + 1, n_used), dtype=torch.int32, device="cuda")
    assert _workspace_size(qwb, W, b1, ids1) > L.NOALLOC_SCRATCH_BYTES
    assert call(T + 1, b1, ids1) == QWB_ERR_LIMIT
    # the largest accepted batch fills the scratch and is computed correctly
    b = torch.from_numpy(D.acts((T, 1, K), seed=41)).cuda()
    ids = _ids(T, n_as, n_used, 4000)
    want = qwb.mul_mat_id(W, b, ids).clone()
    got = torch.full_like(want, float("nan"))
    assert call(T, b, ids, got) == 0
    torch.cuda.synchronize()
    e = O.nrmse(got.cpu().numpy(), want.cpu().numpy())
    assert e <= TOL, e
    assert qwb.read_status()[0] == 0
