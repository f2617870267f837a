"""GPU parity: decode batches on the pair kernels and the shared expert.

* The pair path (router clusters, then gate/up and down over the list of (token, expert)
  pairs, decode.cu): decode batches of up to 16 pairs through qwb_moe_ffn, with ffn_norm,
  the residual and expert-slot pools, against the oracle's build_moe layer.
* The shared expert of core/runtime.cpp:2825-2833 (sh = down_sh(silu(gate_sh x) *
  up_sh x), times sigmoid(gate_inp_sh . x) when the model has that gate, added to the
  routed sum) through qwb_moe_ffn, against the reference's own graph on its ggml CPU
  backend (oracle/_ref): inside the pair kernels (F_sh == F, up to 8 tokens) and on its
  own GEMV kernels otherwise (F_sh != F, more tokens, Q8_0 experts).
Bars: the same selection; layer output nRMS <= 3e-4 (the chained bar of the other layer
tests: act values one fp32 ulp apart can cross a Q8_K rounding boundary), max abs-rel in
the message."""
import os

import numpy as np
import pytest
import torch

import oracle as O
import _data as D

pytestmark = pytest.mark.gpu
CHAIN = 3e-4


@pytest.fixture(scope="module")
def qwb():
    import questwend_b200 as q
    q.lib()
    return q


def cu(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _layer(tgu, td, H, F, E, seed):
    r = D.rng(seed)
    rw = (r.standard_normal((E, H), dtype=np.float32) * 0.02).astype(np.float32)
    nw = (1.0 + 0.1 * r.standard_normal(H, dtype=np.float32)).astype(np.float32)
    return (rw, nw, D.weights(tgu, E, F, H, seed=seed + 1), D.weights(tgu, E, F, H, seed=seed + 2),
            D.weights(td, E, H, F, seed=seed + 3))


@pytest.mark.parametrize("T,k", [(2, 8), (4, 4), (8, 2)])
def test_pair_path_decode_batches(qwb, T, k):
    # up to 16 (token, expert) pairs: the pair kernels
    H, F, E = 2048, 768, 32
    rw, nw, g, u, d = _layer(O.Q4_K, O.Q6_K, H, F, E, seed=10 + T)
    x = D.acts((T, H), seed=20 + T) * np.float32(3.0)
    Wg = qwb.QTensor.from_bytes(g, O.Q4_K, (H, F, E))
    Wu = qwb.QTensor.from_bytes(u, O.Q4_K, (H, F, E))
    Wd = qwb.QTensor.from_bytes(d, O.Q6_K, (F, H, E))
    qwb.read_status()
    out, sel, w = qwb.moe_ffn(cu(x), cu(rw), Wg, Wu, Wd, k, residual=cu(x), norm_w=cu(nw), norm_eps=1e-6)
    assert qwb.read_status()[0] == 0
    r = O.moe_layer(x, rw, O.Q4_K, g, u, O.Q6_K, d, F, E, k, norm_w=nw, norm_eps=1e-6)
    assert np.array_equal(sel.cpu().numpy(), r["selected"])
    assert O.nrmse(w.cpu().numpy(), r["weights"]) < 1e-5  # f32 logit / softmax summation order
    got = out.cpu().numpy() - x
    e = O.nrmse(got, r["out"])
    assert e <= CHAIN, (e, O.max_abs_rel(got, r["out"]))
    # the generic batched path (taken when the act output is requested) agrees
    act = torch.empty((T, k, F), device="cuda")
    out2, _, _ = qwb.moe_ffn(cu(x), cu(rw), Wg, Wu, Wd, k, residual=cu(x), norm_w=cu(nw), norm_eps=1e-6, act=act)
    assert O.nrmse(out2.cpu().numpy() - x, got) <= CHAIN


def test_pair_path_slot_pools(qwb):
    # expert-slot pools with per-role g2s tables (the expert cache's in-graph remap)
    H, F, E, k, T, n_slots = 2048, 768, 32, 4, 4, 40
    rng = D.rng(30)
    rw, nw, g, u, d = _layer(O.Q4_K, O.Q4_K, H, F, E, seed=31)
    g2s = np.stack([rng.permutation(n_slots)[:E] for _ in range(3)]).astype(np.int32)
    pools, host = [], []
    for role, (wt, t, rows, K) in enumerate(((g, O.Q4_K, F, H), (u, O.Q4_K, F, H), (d, O.Q4_K, H, F))):
        rs = O.row_size(t, K) * rows
        p = np.zeros(n_slots * rs, np.uint8)
        for e in range(E):
            p[g2s[role, e] * rs:(g2s[role, e] + 1) * rs] = wt[e * rs:(e + 1) * rs]
        host.append(p)
        pools.append(qwb.QTensor.from_bytes(p, t, (K, rows, n_slots)))
    x = D.acts((T, H), seed=32)
    out, sel, _ = qwb.moe_ffn(cu(x), cu(rw), *pools, k, g2s=cu(g2s), residual=cu(x), norm_w=cu(nw))
    r = O.moe_layer(x, rw, O.Q4_K, host[0], host[1], O.Q4_K, host[2], F, n_slots, k, g2s=g2s, norm_w=nw)
    assert np.array_equal(sel.cpu().numpy(), r["selected"])
    assert O.nrmse(out.cpu().numpy() - x, r["out"]) <= CHAIN
    assert qwb.read_status()[0] == 0


needs_ref = pytest.mark.skipif(not O.ref_available(), reason="reference CPU build (oracle/_ref) missing")


@needs_ref
@pytest.mark.parametrize("tgu,td,T,Fs,gate", [
    (O.Q4_K, O.Q6_K, 1, 768, True),    # batch-1 decode: the shared expert in the pair kernels
    (O.Q4_K, O.Q6_K, 1, 768, False),   # no sigmoid gate (a model without ffn_gate_inp_shexp)
    (O.Q4_K, O.Q4_K, 2, 768, True),    # decode batch of 16 pairs: pair kernels
    (O.Q4_K, O.Q4_K, 6, 768, True),    # 48 pairs: streaming GEMVs, weighted-sum epilogue
    (O.Q4_K, O.Q6_K, 1, 512, True),    # F_sh != F: its own GEMVs, added in the decode down kernel
    (O.Q4_K, O.Q6_K, 12, 512, True),   # batched path (fused router), weighted-sum epilogue
    (O.Q4_K, O.Q6_K, 40, 768, True),   # batched path (separate rms-norm / router kernels)
    (O.Q8_0, O.Q8_0, 3, 768, True),    # Q8_0 experts
])
def test_shared_expert_against_reference_graph(qwb, tgu, td, T, Fs, gate):
    H, F, E, k = 2048, 768, 32, 8
    rw, nw, g, u, d = _layer(tgu, td, H, F, E, seed=40 + T + Fs)
    r = D.rng(41)
    sg = D.weights(tgu, 1, Fs, H, seed=42)
    su = D.weights(tgu, 1, Fs, H, seed=43)
    sd = D.weights(td, 1, H, Fs, seed=44)
    gi = (r.standard_normal(H, dtype=np.float32) * 0.05).astype(np.float32) if gate else None
    x = D.acts((T, H), seed=45 + T) * np.float32(3.0)
    Wg = qwb.QTensor.from_bytes(g, tgu, (H, F, E))
    Wu = qwb.QTensor.from_bytes(u, tgu, (H, F, E))
    Wd = qwb.QTensor.from_bytes(d, td, (F, H, E))
    sh = (qwb.QTensor.from_bytes(sg, tgu, (H, Fs)), qwb.QTensor.from_bytes(su, tgu, (H, Fs)),
          qwb.QTensor.from_bytes(sd, td, (Fs, H)), cu(gi) if gate else None)
    qwb.read_status()
    out, sel, _ = qwb.moe_ffn(cu(x), cu(rw), Wg, Wu, Wd, k, residual=cu(x), norm_w=cu(nw), norm_eps=1e-6, shexp=sh)
    assert qwb.read_status()[0] == 0
    O.set_ref_threads(max(1, len(os.sched_getaffinity(0))))
    want = O.moe_layer_shexp(x, rw, tgu, g, u, td, d, F, E, k, sg, su, sd, Fs, gi, norm_w=nw, norm_eps=1e-6)
    assert np.array_equal(sel.cpu().numpy(), want["selected"])
    got = out.cpu().numpy() - x
    e = O.nrmse(got, want["out"])
    print(f"shared expert T={T} Fs={Fs} gate={gate} types {tgu}/{td}: nrmse {e:.3e}")
    assert e <= CHAIN, (e, O.max_abs_rel(got, want["out"]))
