"""GPU parity: quantized MUL_MAT (qwb_mul_mat), the shared-expert / dense-FFN / output-head
form of the expert kernels (one expert that every token selects), against the reference's
own ggml_mul_mat on its CPU backend (oracle/_ref; the restatement when that build is
absent).  Bar: nRMS <= 1e-4, max abs-rel error in the message.  Also through the ggml
backend library (ggml_backend_load -> graph_compute on a MUL_MAT node)."""
import os

import numpy as np
import pytest
import torch

import oracle as O
import _data as D

pytestmark = pytest.mark.gpu
TOL = 1e-4
SHIM = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "questwend_b200", "libggml-qwb.so")


@pytest.fixture(scope="module")
def qwb():
    import questwend_b200 as q
    q.lib()
    return q


def _want(t, w, K, M, b):
    if O.ref_available():
        return O.mul_mat(t, w, K, M, b, impl="ref")[0]
    dst, rc = O.mul_mat(t, w, K, M, b)
    assert rc == 0
    return dst


@pytest.mark.parametrize("t,K,M,T", [
    (O.Q4_K, 2048, 300, 1),     # shared expert / dense FFN, decode
    (O.Q4_K, 2048, 768, 5),
    (O.Q4_K, 1024, 256, 64),    # many tokens: tensor-core grouped GEMM
    (O.Q6_K, 2048, 4096, 1),    # output-head rows (Q6_K), decode
    (O.Q6_K, 768, 2048, 12),    # 8-31 tokens: int8 tensor cores, 8-token tiles
    (O.Q6_K, 2048, 4096, 8),    # output-head rows at 8 tokens
    (O.Q8_0, 1024, 300, 20),
    (O.Q8_0, 2048, 200, 3),
    (O.Q8_0, 512, 96, 40),
])
def test_matches_reference_mul_mat(qwb, t, K, M, T):
    w = D.weights(t, 1, M, K, seed=K + M + T)
    b = D.acts((T, K), seed=T + 11)
    A = qwb.QTensor.from_bytes(w, t, (K, M))
    got = qwb.mul_mat(A, torch.from_numpy(b).cuda()).cpu().numpy()
    flags, _, _ = qwb.read_status()
    assert flags == 0
    want = _want(t, w, K, M, b)
    e = O.nrmse(got, want)
    assert e <= TOL, (e, O.max_abs_rel(got, want))


def test_column_view_of_activations(qwb):
    # b as rows of a wider buffer (nb1 > K*4): ggml views of a larger activation tensor
    t, K, M, T = O.Q4_K, 1024, 128, 4
    w = D.weights(t, 1, M, K, seed=3)
    wide = D.acts((T, K + 256), seed=4)
    A = qwb.QTensor.from_bytes(w, t, (K, M))
    got = qwb.mul_mat(A, torch.from_numpy(wide).cuda()[:, :K]).cpu().numpy()
    want = _want(t, w, K, M, np.ascontiguousarray(wide[:, :K]))
    assert O.nrmse(got, want) <= TOL


@pytest.mark.parametrize("t,K,M,T", [(O.Q4_K, 2048, 512, 2), (O.Q6_K, 2048, 1024, 1), (O.Q8_0, 1024, 256, 40)])
def test_through_ggml_backend_library(t, K, M, T):
    if not os.path.exists(SHIM) or not O.ref_available():
        pytest.skip("backend library or reference ggml not built")
    w = D.weights(t, 1, M, K, seed=21 + T)
    b = D.acts((T, K), seed=22)
    got, rc = O.backend_mul_mat(SHIM, t, w, K, M, b)
    assert rc == 0, rc
    want = _want(t, w, K, M, b)
    e = O.nrmse(got, want)
    assert e <= TOL, (e, O.max_abs_rel(got, want))
