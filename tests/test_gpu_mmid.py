"""GPU parity: MUL_MAT_ID on Q4_K / Q6_K / Q8_0 against the reference's arithmetic.

Bar: normalized RMS error <= 1e-4 against the CPU oracle on the same inputs (the
integer sub-block dots are exact; only the fp32 summation order differs, so the
measured error is ~1e-7); max abs-rel error is reported in the assertion message."""
import os

import numpy as np
import pytest
import torch

import oracle as O
import _data as D

pytestmark = pytest.mark.gpu
G = os.path.join(os.path.dirname(__file__), "golden")
TOL = 1e-4


@pytest.fixture(scope="module")
def qwb():
    import questwend_b200 as q
    q.lib()
    return q


def cu(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("name,t", [("q4K", O.Q4_K), ("q6K", O.Q6_K), ("q80", O.Q8_0)])
def test_golden(qwb, name, t):
    g = np.load(os.path.join(G, "mul_mat_id.npz"))
    K, M, n_as = 512, 64, 8
    w = D.weights(t, n_as, M, K, seed=21 + t)
    assert D.sha(w) == str(g[f"{name}_wsha"])
    W = qwb.QTensor.from_bytes(w, t, (K, M, n_as))
    for n_b in (1, 3):
        got = qwb.mul_mat_id(W, cu(g[f"b{n_b}"]), cu(g["ids"])).cpu().numpy()
        want = g[f"{name}_nb{n_b}"]
        e = O.nrmse(got, want)
        assert e <= TOL, (name, n_b, e, O.max_abs_rel(got, want))


CASES = [
    # type, K, M, n_as, T, n_used, n_b
    (O.Q4_K, 2048, 768, 128, 1, 8, 1),     # config-1 gate/up shape, decode
    (O.Q6_K, 768, 2048, 32, 1, 8, 8),      # down shape, decode (b = act per slot)
    (O.Q8_0, 4096, 256, 16, 3, 8, 1),
    (O.Q4_K, 4096, 256, 16, 9, 8, 1),      # several tokens per expert (NT > 1)
    (O.Q6_K, 1024, 128, 8, 33, 4, 4),
    (O.Q8_0, 512, 96, 8, 64, 8, 8),
    (O.Q4_K, 768, 2048, 8, 64, 8, 8),
    # weight-streaming kernel edges
    (O.Q6_K, 768, 2048, 4, 40, 2, 1),      # 20 tokens per expert: three token passes
    (O.Q8_0, 2048, 300, 16, 7, 4, 2),      # rows not a multiple of the stage rows
    (O.Q8_0, 96, 40, 3, 5, 2, 1),          # 3 blocks per row: a partial lane group
    (O.Q4_K, 256, 33, 5, 3, 5, 1),         # one superblock per row: 32 rows per stage
    (O.Q4_K, 256, 8, 2, 1, 2, 1),          # 16 rows in total: most CTAs idle
    (O.Q4_K, 16384, 64, 4, 2, 2, 1),       # long rows: fewer consumer warps
]


@pytest.mark.parametrize("t,K,M,n_as,T,n_used,n_b", CASES)
def test_random(qwb, t, K, M, n_as, T, n_used, n_b):
    w = D.weights(t, n_as, M, K, seed=K + M + T)
    b = D.acts((T, n_b, K), seed=T)
    r = D.rng(T + 1)
    ids = np.stack([r.choice(n_as, n_used, replace=n_used > n_as) for _ in range(T)]).astype(np.int32)
    W = qwb.QTensor.from_bytes(w, t, (K, M, n_as))
    got = qwb.mul_mat_id(W, cu(b), cu(ids)).cpu().numpy()
    want, rc = O.mul_mat_id(t, w, K, M, n_as, b, ids)
    assert rc == 0
    e = O.nrmse(got, want)
    assert e <= TOL, (e, O.max_abs_rel(got, want))


def test_strided_ids_view_and_pool(qwb):
    # ids as a strided view (argsort_top_k keeps the full argsort row: nb1 = E*4), weights
    # as a slot pool larger than the experts referenced
    t, K, M, n_slots, T, n_used, E = O.Q4_K, 1024, 128, 24, 6, 4, 16
    w = D.weights(t, n_slots, M, K, seed=5)
    b = D.acts((T, 1, K), seed=6)
    full = np.stack([D.rng(40 + i).permutation(E) for i in range(T)]).astype(np.int32)
    ids_view = cu(full)[:, :n_used]
    assert ids_view.stride(0) == E
    W = qwb.QTensor.from_bytes(w, t, (K, M, n_slots))
    got = qwb.mul_mat_id(W, cu(b), ids_view).cpu().numpy()
    want, _ = O.mul_mat_id(t, w, K, M, n_slots, b, np.ascontiguousarray(full[:, :n_used]))
    assert O.nrmse(got, want) <= TOL


def test_bad_ids_reported_not_faulting(qwb):
    qwb.read_status()
    t, K, M, n_as = O.Q8_0, 256, 64, 4
    w = D.weights(t, n_as, M, K, seed=8)
    b = D.acts((2, 1, K), seed=9)
    ids = np.array([[0, 9], [-3, 2]], dtype=np.int32)
    W = qwb.QTensor.from_bytes(w, t, (K, M, n_as))
    got = qwb.mul_mat_id(W, cu(b), cu(ids)).cpu().numpy()
    flags, bad, count = qwb.read_status()
    assert flags & 1 and count == 2 and bad in (9, -3)
    assert not got[0, 1].any() and not got[1, 0].any()
    ok_ids = np.array([[0, 0], [2, 2]], dtype=np.int32)
    want, _ = O.mul_mat_id(t, w, K, M, n_as, b, ok_ids)
    assert O.nrmse(got[0, 0], want[0, 0]) <= TOL and O.nrmse(got[1, 1], want[1, 1]) <= TOL


def test_repeat_calls_identical(qwb):
    t, K, M, n_as, T = O.Q4_K, 2048, 512, 32, 4
    w = D.weights(t, n_as, M, K, seed=12)
    W = qwb.QTensor.from_bytes(w, t, (K, M, n_as))
    b, ids = cu(D.acts((T, 1, K), seed=13)), cu(np.tile(np.arange(8, dtype=np.int32), (T, 1)))
    a1 = qwb.mul_mat_id(W, b, ids).clone()
    a2 = qwb.mul_mat_id(W, b, ids)
    assert torch.equal(a1, a2)


# One token (T == 1, Q4_K / Q6_K, K / 256 in {3, 6, 8, 16}): the kernel without an expert
# index (mmid_one.cu), each CTA's slice of the selected experts' rows copied while the
# activation row is quantized.  Shapes: the large-model decode MUL_MAT_IDs (hidden 4096,
# expert FFN 1536: gate/up [4096 -> 1536] with one activation row, down [1536 -> 4096]
# with one per slot), Q6_K rows (2-byte aligned segments), ranges that split experts.
ONE_TOKEN = [
    # type, K, M, n_as, n_used, n_b
    (O.Q4_K, 4096, 1536, 128, 8, 1),
    (O.Q4_K, 1536, 4096, 64, 8, 8),
    (O.Q6_K, 1536, 512, 16, 4, 4),
    (O.Q6_K, 2048, 300, 8, 6, 2),
    (O.Q4_K, 4096, 100, 8, 8, 1),
]


@pytest.mark.parametrize("t,K,M,n_as,n_used,n_b", ONE_TOKEN)
def test_one_token(qwb, t, K, M, n_as, n_used, n_b):
    qwb.read_status()
    w = D.weights(t, n_as, M, K, seed=K + M + 3)
    b = D.acts((1, n_b, K), seed=K + 4)
    ids = D.rng(K + 5).choice(n_as, n_used, replace=False).astype(np.int32)[None, :]
    W = qwb.QTensor.from_bytes(w, t, (K, M, n_as))
    got = qwb.mul_mat_id(W, cu(b), cu(ids)).cpu().numpy()
    want, rc = O.mul_mat_id(t, w, K, M, n_as, b, ids)
    assert rc == 0
    e = O.nrmse(got, want)
    assert e <= TOL, (e, O.max_abs_rel(got, want))
    assert qwb.read_status()[0] == 0


def test_one_token_bad_id_and_strided_view(qwb):
    """An id outside the pool gives a zero output row and a QWB_DEVERR_ID_RANGE record; the
    ids may be a strided view (the argsort row of all experts)."""
    qwb.read_status()
    t, K, M, n_as, n_used, E = O.Q4_K, 2048, 384, 16, 4, 16
    w = D.weights(t, n_as, M, K, seed=71)
    b = D.acts((1, 1, K), seed=72)
    full = D.rng(73).permutation(E).astype(np.int32)[None, :]
    full[0, 2] = n_as + 7
    view = cu(full)[:, :n_used]
    W = qwb.QTensor.from_bytes(w, t, (K, M, n_as))
    got = qwb.mul_mat_id(W, cu(b), view).cpu().numpy()
    flags, bad, count = qwb.read_status()
    assert flags & 1 and bad == n_as + 7 and count == 1
    assert not got[0, 2].any()
    ok = np.ascontiguousarray(full[:, :n_used]).copy()
    ok[0, 2] = 0
    want, _ = O.mul_mat_id(t, w, K, M, n_as, b, ok)
    for j in (0, 1, 3):
        assert O.nrmse(got[0, j], want[0, j]) <= TOL
