"""GPU parity: MUL_MAT_ID on Q8_0 and Q6_K experts with many tokens per expert, the
integer tensor-core kernels:
  * mma.sync s8 x s8 -> s32 (prefill_i8.cu, fewer pairs per expert): one m16n8k32 per
    Q8_0 block with fp32 block scaling in block order; one m16n8k16 per Q6_K sub-block with
    its int8 scale in int32 and fp32 scaling per superblock;
  * tcgen05.mma kind::i8 (prefill_tc8.cu, Q6_K from 96 and Q8_0 from 256 pairs per
    expert): Q6_K with the sub-block scales folded into two int8 weight planes and fp32
    scaling per superblock; Q8_0 with one s32 tensor-memory accumulator region per
    32-element block and fp32 scaling per block;
against the oracle's dots (activations quantized as the CPU backend does: Q8_0 CPU
variant / Q8_K), against the reference's own ggml CPU backend under skewed routing, and
against the weight-streaming path on the same inputs.  Bar: nRMS <= 1e-4 (max abs-rel
error in the message)."""
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


def _run(q, W, b, ids, profile=False):
    from questwend_b200 import _lib as L
    lib = L.lib()
    if profile:
        L.check("qwb_profile_enable", lib.qwb_profile_enable(8))
        lib.qwb_profile_reset()
    out = q.mul_mat_id(W, b, ids)
    torch.cuda.synchronize()
    tags = []
    if profile:
        n = lib.qwb_profile_count() - 1
        ms = (C.c_float * max(n, 1))()
        tg = (C.c_int32 * max(n, 1))()
        L.check("qwb_profile_read", lib.qwb_profile_read(ms, tg, n))
        tags = list(tg[:n])
        L.check("qwb_profile_enable", lib.qwb_profile_enable(0))
    return out, tags


def _stream(q, W, b, ids):
    # qwb_mul_mat_id_noalloc never takes a tensor-core path: the weight-streaming kernel
    from questwend_b200 import _lib as L
    T, n_used, M = ids.shape[0], ids.shape[1], W.ne[1]
    out = torch.empty((T, n_used, M), dtype=torch.float32, device="cuda")
    ad, bd, idd, od = q.ops.desc(W), q.ops.desc(b), q.ops.desc(ids), q.ops.desc(out)
    rc = L.lib().qwb_mul_mat_id_noalloc(C.byref(ad), C.byref(bd), C.byref(idd), C.byref(od),
                                       q.ops.status_block().data_ptr(),
                                       C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    return out


CASES = [
    # type, K, M, n_as, T, n_used, n_b
    (O.Q8_0, 1024, 300, 8, 256, 4, 1),      # rows not a multiple of 128, partial token tiles
    (O.Q8_0, 2048, 768, 16, 512, 8, 1),     # gate/up-like
    (O.Q8_0, 512, 2048, 8, 128, 4, 4),      # down-like: one activation row per (token, slot)
    (O.Q8_0, 4096, 128, 8, 64, 8, 8),       # long K, one activation row per (token, slot)
    (O.Q6_K, 768, 2048, 8, 128, 4, 4),      # config-2 down shape
    (O.Q6_K, 1024, 300, 8, 256, 4, 1),
    (O.Q6_K, 2048, 128, 8, 64, 8, 8),
    # Q6_K at >= 96 pairs per used expert: the tcgen05 kernel (128-token tiles)
    (O.Q6_K, 768, 2048, 8, 256, 4, 4),      # 128 per expert, config-2 down shape
    (O.Q6_K, 2048, 300, 8, 512, 8, 8),      # 512 per expert, rows not a multiple of 128
    (O.Q6_K, 1536, 256, 4, 100, 4, 1),      # 100 per expert: one full and one 28-pair tile each
    # Q8_0 at >= 256 pairs per used expert: the tcgen05 kernel (one TMEM region per 32-block)
    (O.Q8_0, 4096, 256, 8, 256, 8, 8),      # 256 per expert, one activation row per (token, slot)
    (O.Q8_0, 1536, 300, 4, 300, 4, 1),      # 300 per expert: two full and one 44-pair tile each,
                                            # rows not a multiple of 128
    # 8 to 31 pairs per used expert: 8-token tiles (16-row warps, one 8-token MMA column)
    (O.Q8_0, 1024, 300, 16, 40, 4, 1),      # 10 per expert, partial tiles and row blocks
    (O.Q8_0, 4096, 128, 8, 12, 8, 8),       # 12 per expert, one activation row per pair
    (O.Q6_K, 768, 2048, 16, 64, 4, 4),      # 16 per expert, config-2 down shape
    (O.Q6_K, 2048, 300, 8, 16, 4, 1),       # exactly 8 per expert
]


@pytest.mark.parametrize("t,K,M,n_as,T,n_used,n_b", CASES)
def test_uniform_routing(qwb, t, K, M, n_as, T, n_used, n_b):
    w = D.weights(t, n_as, M, K, seed=K + M + T)
    b = D.acts((T, n_b, K), seed=T + 5)
    ids = np.stack([D.rng(200 + i).permutation(n_as)[:n_used] for i in range(T)]).astype(np.int32)
    W = qwb.QTensor.from_bytes(w, t, (K, M, n_as))
    got, tags = _run(qwb, W, cu(b), cu(ids), profile=True)
    assert 5 in tags  # the tensor-core kernel ran (QWB_KERNEL_GROUPED_GEMM)
    flags, _, _ = qwb.read_status()
    assert flags == 0
    want, rc = O.mul_mat_id(t, w, K, M, n_as, b, ids)
    assert rc == 0
    got = got.cpu().numpy()
    e = O.nrmse(got, want)
    assert e <= TOL, (e, O.max_abs_rel(got, want))


@pytest.mark.parametrize("t,T", [(O.Q8_0, 512), (O.Q8_0, 2048), (O.Q6_K, 512), (O.Q6_K, 1024)])
def test_zipf_routing_against_reference_build(qwb, t, T):
    K, M, n_as, n_used = 1024, 256, 64, 8
    w = D.weights(t, n_as, M, K, seed=31)
    b = D.acts((T, 1, K), seed=32)
    ids = D.zipf_ids(T, n_as, n_used, seed=33)
    W = qwb.QTensor.from_bytes(w, t, (K, M, n_as))
    got = _run(qwb, W, cu(b), cu(ids))[0].cpu().numpy()
    if O.ref_available():
        O.set_ref_threads(8)
        want, _ = O.mul_mat_id(t, w, K, M, n_as, b, ids, impl="ref")
    else:
        want, _ = O.mul_mat_id(t, w, K, M, n_as, b, ids)
    e = O.nrmse(got, want)
    assert e <= TOL, (e, O.max_abs_rel(got, want))


@pytest.mark.parametrize("t,T", [(O.Q8_0, 160), (O.Q8_0, 320), (O.Q6_K, 160), (O.Q8_0, 12), (O.Q6_K, 12)])
def test_matches_streaming_path(qwb, t, T):
    K, M, n_as, n_used = 1024, 384, 8, 8
    w = D.weights(t, n_as, M, K, seed=51)
    b = cu(D.acts((T, 1, K), seed=52))
    ids = cu(np.stack([D.rng(53 + i).permutation(n_as)[:n_used] for i in range(T)]).astype(np.int32))
    W = qwb.QTensor.from_bytes(w, t, (K, M, n_as))
    tc = _run(qwb, W, b, ids)[0]
    st = _stream(qwb, W, b, ids)
    # the same per-block fp32 products; only the summation order of blocks vs passes differs
    assert O.nrmse(tc.cpu().numpy(), st.cpu().numpy()) <= 1e-5
