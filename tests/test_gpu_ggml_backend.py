"""Drop-in check on a B200: the reference's own ggml loads questwend_b200/libggml-qwb.so
with ggml_backend_load, allocates the tensors in its buffer type (weights in a buffer
marked as weights, as the model loader marks them), and computes graphs with
ggml_backend_graph_compute and with ggml_backend_sched, where the scheduler sends
MUL_MAT_ID to this backend and a following ggml_scale to the CPU backend.
Bars: MUL_MAT_ID within 1e-4 normalized RMS of the oracle (max abs-rel in the message);
GET_ROWS bit-exact."""
import os

import numpy as np
import pytest

import oracle as O
import _data as D

pytestmark = pytest.mark.gpu
SHIM = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "questwend_b200", "libggml-qwb.so")
TOL = 1e-4


@pytest.fixture(scope="module")
def ready():
    if not os.path.exists(SHIM):
        pytest.skip("libggml-qwb.so not built")
    if not O.ref_available():
        pytest.skip("the reference ggml (oracle/_ref) is not built")


@pytest.mark.parametrize("t,K,M,n_as,T,n_used,n_b,width", [
    (O.Q4_K, 2048, 768, 32, 3, 8, 1, 32),     # decode-like; ids a strided view (argsort row)
    (O.Q6_K, 768, 2048, 16, 4, 8, 8, 8),      # down shape, one b row per slot
    (O.Q8_0, 1024, 256, 8, 5, 4, 1, 8),
    (O.Q4_K, 1024, 256, 8, 256, 8, 1, 8),     # many tokens per expert: tensor-core path
])
def test_graph_compute_matches_oracle(ready, t, K, M, n_as, T, n_used, n_b, width):
    w = D.weights(t, n_as, M, K, seed=K + M + T)
    b = D.acts((T, n_b, K), seed=T + 3)
    ids = np.stack([D.rng(100 + i).permutation(n_as)[:width] if width <= n_as
                    else D.rng(100 + i).integers(0, n_as, width) for i in range(T)]).astype(np.int32)
    got, rc = O.backend_mul_mat_id(SHIM, t, w, K, M, n_as, b, ids, n_used=n_used)
    assert rc == 0, rc
    want, rc = O.mul_mat_id(t, w, K, M, n_as, b, ids[:, :n_used].copy())
    assert rc == 0
    e = O.nrmse(got, want)
    assert e <= TOL, (e, O.max_abs_rel(got, want))


@pytest.mark.parametrize("t", [O.Q4_K, O.Q6_K, O.Q8_0, O.F16, O.F32])
def test_get_rows_bit_exact(ready, t):
    ne0, nrows, n = 512, 64, 37
    src = D.weights(t, 1, nrows, ne0, seed=5) if t in (O.Q4_K, O.Q6_K, O.Q8_0) else None
    if t == O.F16:
        src = D.rng(6).standard_normal((nrows, ne0)).astype(np.float16).view(np.uint8).reshape(-1)
    elif t == O.F32:
        src = D.rng(6).standard_normal((nrows, ne0)).astype(np.float32).view(np.uint8).reshape(-1)
    idx = D.rng(7).integers(0, nrows, n).astype(np.int32)
    got, rc = O.backend_get_rows(SHIM, t, src, ne0, nrows, idx)
    assert rc == 0, rc
    want, rc = O.get_rows(t, src, ne0, nrows, idx)
    assert rc == 0
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_scheduler_places_mul_mat_id_on_this_backend(ready):
    t, K, M, n_as, T, n_used = O.Q4_K, 2048, 512, 16, 6, 4
    w = D.weights(t, n_as, M, K, seed=7)
    b = D.acts((T, 1, K), seed=8)
    ids = np.stack([D.rng(200 + i).permutation(n_as)[:n_used] for i in range(T)]).astype(np.int32)
    got, rc, n_splits, on_shim = O.backend_sched_mul_mat_id(SHIM, t, w, K, M, n_as, b, ids, 2.0)
    assert rc == 0, rc
    assert on_shim and n_splits >= 2, (on_shim, n_splits)
    want, _ = O.mul_mat_id(t, w, K, M, n_as, b, ids)
    e = O.nrmse(got, 2.0 * want)
    assert e <= TOL, (e, O.max_abs_rel(got, 2.0 * want))
