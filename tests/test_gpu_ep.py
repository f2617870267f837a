"""GPU parity: the expert-parallel MoE layer's device steps (qwb_moe_ep_prepare,
qwb_moe_ep_experts) on one B200, with N ranks emulated by running every rank's expert
shard in turn and summing the partial outputs (what the reduce-scatter does across GPUs).

Bars: the routing equals qwb_moe_ffn's (same ids, weights to 1e-5: the two router paths sum the
logits and the softmax in different f32 orders); the summed layer output
matches qwb_moe_ffn within 1e-5 normalized RMS (only the f32 order of the weighted expert
sum differs) and the CPU oracle's build_moe layer within 1e-4; max abs-rel error in the
message."""
import numpy as np
import pytest
import torch

import oracle as O
import _data as D

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def qwb():
    import questwend_b200 as q
    q.lib()
    return q


def cu(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _layer(t_gu, t_d, H, F, E, seed):
    r = D.rng(seed)
    router_w = (r.standard_normal((E, H), dtype=np.float32) * 0.02).astype(np.float32)
    norm_w = (1.0 + 0.1 * r.standard_normal(H)).astype(np.float32)
    gate = D.weights(t_gu, E, F, H, seed=seed + 1)
    up = D.weights(t_gu, E, F, H, seed=seed + 2)
    down = D.weights(t_d, E, H, F, seed=seed + 3)
    return router_w, norm_w, gate, up, down


def _shard(q, W, t, K, M, lo, n):
    mat = O.row_size(t, K) * M
    return q.QTensor(W.data[lo * mat:(lo + n) * mat], t, (K, M, n, 1))


@pytest.mark.parametrize("t_gu,t_d,T,world", [
    (O.Q4_K, O.Q6_K, 1, 2),     # decode token, 2 ranks
    (O.Q4_K, O.Q6_K, 16, 4),    # 4 ranks x 4 tokens
    (O.Q8_0, O.Q8_0, 8, 2),     # Q8_0 experts: Q8_0 (CPU variant) activations
])
def test_shards_sum_to_fused_layer(qwb, t_gu, t_d, T, world):
    from questwend_b200.expert_parallel import shard_range
    H, F, E, K = 2048, 768, 32, 8
    router_w, norm_w, gate, up, down = _layer(t_gu, t_d, H, F, E, seed=50 + T)
    x = D.acts((T, H), seed=60 + T)
    G = qwb.QTensor.from_bytes(gate, t_gu, (H, F, E))
    U = qwb.QTensor.from_bytes(up, t_gu, (H, F, E))
    Dn = qwb.QTensor.from_bytes(down, t_d, (F, H, E))
    xc, rw, nw = cu(x), cu(router_w), cu(norm_w)
    fused, fsel, fw = qwb.moe_ffn(xc, rw, G, U, Dn, K, residual=xc, norm_w=nw)

    act_type = O.Q8_K if t_gu != O.Q8_0 else O.Q8_0
    xq, sel, w = qwb.ops.moe_ep_prepare(xc, rw, K, norm_w=nw, act_type=act_type)
    assert (sel == fsel).all()
    assert torch.allclose(w, fw, rtol=1e-5, atol=0), float(((w - fw).abs() / fw.abs()).max())
    total = torch.zeros((T, H), device="cuda")
    for r in range(world):
        lo, n = shard_range(E, world, r)
        part = qwb.ops.moe_ep_experts(xq, sel, w, _shard(qwb, G, t_gu, H, F, lo, n), _shard(qwb, U, t_gu, H, F, lo, n),
                                      _shard(qwb, Dn, t_d, F, H, lo, n), lo, E)
        total += part
    flags, bad, cnt = qwb.read_status()
    assert flags == 0, (flags, bad, cnt)
    out = (total + xc).cpu().numpy()
    e = O.nrmse(out, fused.cpu().numpy())
    assert e <= 1e-5, (e, O.max_abs_rel(out, fused.cpu().numpy()))
    want = O.moe_layer(x, router_w, t_gu, gate, up, t_d, down, F, E, K, norm_w=norm_w)
    assert (want["selected"] == sel.cpu().numpy()).all()
    e = O.nrmse(out - x, want["out"])
    assert e <= 1e-4, (e, O.max_abs_rel(out - x, want["out"]))


def test_prepare_packs_reference_q8K_rows(qwb):
    # the gathered bytes are the reference quantizer's Q8_K rows of rms_norm(x) * ffn_norm
    H, E, K, T = 2048, 32, 8, 4
    r = D.rng(70)
    router_w = (r.standard_normal((E, H), dtype=np.float32) * 0.02).astype(np.float32)
    norm_w = (1.0 + 0.1 * r.standard_normal(H)).astype(np.float32)
    x = D.acts((T, H), seed=71)
    xq, _, _ = qwb.ops.moe_ep_prepare(cu(x), cu(router_w), K, norm_w=cu(norm_w))
    want = O.quantize_act(O.Q8_K, O.rms_norm_mul(x, norm_w, 1e-6))
    got = xq.cpu().numpy().reshape(-1)
    assert got.size == want.size
    assert (got == want.reshape(-1)).mean() > 0.999


def test_foreign_ids_are_skipped_not_reported(qwb):
    # a shard whose experts nobody selected returns zeros and raises no device error
    H, F, E, K, T = 2048, 768, 32, 8, 2
    router_w, norm_w, gate, up, down = _layer(O.Q4_K, O.Q6_K, H, F, E, seed=80)
    G = qwb.QTensor.from_bytes(gate, O.Q4_K, (H, F, E))
    U = qwb.QTensor.from_bytes(up, O.Q4_K, (H, F, E))
    Dn = qwb.QTensor.from_bytes(down, O.Q6_K, (F, H, E))
    x = cu(D.acts((T, H), seed=81))
    xq, sel, w = qwb.ops.moe_ep_prepare(x, cu(router_w), K, norm_w=cu(norm_w))
    sel = torch.zeros_like(sel)  # every slot routed to expert 0
    qwb.read_status()
    part = qwb.ops.moe_ep_experts(xq, sel, w, _shard(qwb, G, O.Q4_K, H, F, 16, 16),
                                  _shard(qwb, U, O.Q4_K, H, F, 16, 16), _shard(qwb, Dn, O.Q6_K, F, H, 16, 16), 16, E)
    flags, _, _ = qwb.read_status()
    assert flags == 0
    assert not part.any()
