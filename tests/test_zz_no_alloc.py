"""qwb_mul_mat_id_noalloc: MUL_MAT_ID for callers that cannot allocate device memory.

Callers such as a ggml backend's graph_compute, code running under someone else's CUDA
graph capture, or a host whose device memory is fully committed to its expert pool can
neither allocate nor hand over a workspace; this entry point runs from scratch space the
library carries in its own device image.  The test drives it through the C ABI and
compares it with qwb_mul_mat_id (which takes a caller workspace) on two calls in a row,
with different inputs, at the tolerance the other MUL_MAT_ID tests use; it also checks
that a problem larger than the scratch is refused.  It is collected last (file name) so a
failing run that stops at the first failure has run every other test first."""
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


def _noalloc(q, W, b, ids, out):
    from questwend_b200 import _lib as L
    ad, bd, idd, od = q.ops.desc(W), q.ops.desc(b), q.ops.desc(ids), q.ops.desc(out)
    return L.lib().qwb_mul_mat_id_noalloc(C.byref(ad), C.byref(bd), C.byref(idd), C.byref(od),
                                         q.ops.status_block().data_ptr(),
                                         C.c_void_p(torch.cuda.current_stream().cuda_stream))


def test_noalloc_matches_workspace_entry_point_twice(qwb):
    t, K, M, n_as, n_used = O.Q4_K, 2048, 768, 32, 8
    W = qwb.QTensor.from_bytes(D.weights(t, n_as, M, K, seed=77), t, (K, M, n_as))
    qwb.read_status()
    for call, T in enumerate((4, 9)):
        b = torch.from_numpy(D.acts((T, 1, K), seed=100 + call)).cuda()
        ids = torch.from_numpy(np.stack([D.rng(200 + call * 50 + i).choice(n_as, n_used, replace=False)
                                         for i in range(T)]).astype(np.int32)).cuda()
        want = qwb.mul_mat_id(W, b, ids).clone()
        got = torch.full_like(want, float("nan"))
        assert _noalloc(qwb, W, b, ids, got) == 0
        torch.cuda.synchronize()
        e = O.nrmse(got.cpu().numpy(), want.cpu().numpy())
        assert e <= TOL, (call, e)
    assert qwb.read_status()[0] == 0


def test_noalloc_rejects_problems_beyond_scratch(qwb):
    from questwend_b200 import _lib as L
    t, K, M, n_as, n_used, T = O.Q8_0, 4096, 64, 8, 8, 2048  # ~9.5 MB of quantized rows
    W = qwb.QTensor.from_bytes(D.weights(t, n_as, M, K, seed=5), t, (K, M, n_as))
    b = torch.zeros((T, 1, K), device="cuda")
    ids = torch.zeros((T, n_used), dtype=torch.int32, device="cuda")
    out = torch.empty((T, n_used, M), device="cuda")
    need = L.lib().qwb_mul_mat_id_workspace_size(C.byref(qwb.ops.desc(W)), C.byref(qwb.ops.desc(b)),
                                                 C.byref(qwb.ops.desc(ids)))
    assert need > L.NOALLOC_SCRATCH_BYTES
    assert _noalloc(qwb, W, b, ids, out) == 9  # QWB_ERR_LIMIT
