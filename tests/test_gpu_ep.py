"""GPU parity: the expert-parallel MoE layer's device step (qwb_moe_ep_layer) on one
B200, with N ranks emulated by running every rank's expert shard in turn (residual on
rank 0 only) and summing the partial outputs, which is what the all-reduce does across
GPUs.

Bars: the routing of every shard equals qwb_moe_ffn's (same ids, weights to 1e-5: at one
token the two entry points use routers that sum in different f32 orders); the summed layer output matches qwb_moe_ffn within 1e-5 normalized RMS
(only the f32 order of the weighted expert sum differs) and the CPU oracle's build_moe
layer within 1e-4; max abs-rel error in the message.  Shapes: the 30B-A3B layer (hidden
2048, F 768) and the 235B-A22B expert-parallel layer (hidden 4096, F 1536, 128 experts,
top-8) at T = 1, 8 and 64 tokens over 2, 4 and 8 shards."""
import os

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


_BLK = {O.Q4_K: (144, 0), O.Q6_K: (210, 208), O.Q8_0: (34, 0)}


def expert_pool(t, n_exp, rows, K, seed, n_base=4):
    """n_exp distinct expert images: ggml-quantized base matrix e % n_base with every block
    scale d times (1 + e/256) (quantizing 128 full-size experts would take minutes)."""
    base = D.weights(t, n_base, rows, K, seed=seed)
    nbytes, off = _BLK[t]
    per = base.size // n_base
    b = base.reshape(n_base, per // nbytes, nbytes)
    out = np.empty((n_exp, per // nbytes, nbytes), dtype=np.uint8)
    for i in range(n_exp):
        blk = b[i % n_base].copy()
        d = blk[:, off:off + 2].copy().view(np.float16).astype(np.float32)
        blk[:, off:off + 2] = (d * np.float32(1.0 + i / 256.0)).astype(np.float16).view(np.uint8)
        out[i] = blk
    return out.reshape(-1)


def _layer(t_gu, t_d, H, F, E, seed):
    r = D.rng(seed)
    router_w = (r.standard_normal((E, H), dtype=np.float32) * 0.02).astype(np.float32)
    norm_w = (1.0 + 0.1 * r.standard_normal(H)).astype(np.float32)
    gate = expert_pool(t_gu, E, F, H, seed=seed + 1)
    up = expert_pool(t_gu, E, F, H, seed=seed + 2)
    down = expert_pool(t_d, E, H, F, seed=seed + 3)
    return router_w, norm_w, gate, up, down


def _shard(q, W, t, K, M, lo, n):
    mat = O.row_size(t, K) * M
    return q.QTensor(W.data[lo * mat:(lo + n) * mat], t, (K, M, n, 1))


@pytest.mark.parametrize("t_gu,t_d,H,F,E,T,world", [
    (O.Q4_K, O.Q6_K, 2048, 768, 32, 1, 2),     # decode token, 2 ranks
    (O.Q4_K, O.Q6_K, 2048, 768, 32, 16, 4),    # 16 tokens, 4 ranks
    (O.Q8_0, O.Q8_0, 2048, 768, 32, 8, 2),     # Q8_0 experts: Q8_0 (CPU variant) activations
    (O.Q4_K, O.Q6_K, 4096, 1536, 128, 1, 8),   # the 235B-A22B layer: T = 1, 8, 64
    (O.Q4_K, O.Q6_K, 4096, 1536, 128, 8, 8),
    (O.Q4_K, O.Q6_K, 4096, 1536, 128, 64, 4),
    (O.Q4_K, O.Q6_K, 4096, 1536, 128, 64, 2),
])
def test_shards_sum_to_fused_layer(qwb, t_gu, t_d, H, F, E, T, world):
    from questwend_b200.expert_parallel import shard_range
    K = 8
    router_w, norm_w, gate, up, down = _layer(t_gu, t_d, H, F, E, seed=50 + T + H)
    x = D.acts((T, H), seed=60 + T)
    G = qwb.QTensor.from_bytes(gate, t_gu, (H, F, E))
    U = qwb.QTensor.from_bytes(up, t_gu, (H, F, E))
    Dn = qwb.QTensor.from_bytes(down, t_d, (F, H, E))
    xc, rw, nw = cu(x), cu(router_w), cu(norm_w)
    fused, fsel, fw = qwb.moe_ffn(xc, rw, G, U, Dn, K, residual=xc, norm_w=nw)
    fused = fused.clone()

    total = torch.zeros((T, H), device="cuda")
    for r in range(world):
        lo, n = shard_range(E, world, r)
        part, sel, w = qwb.ops.moe_ep_layer(xc, rw, _shard(qwb, G, t_gu, H, F, lo, n), _shard(qwb, U, t_gu, H, F, lo, n),
                                            _shard(qwb, Dn, t_d, F, H, lo, n), lo, K,
                                            residual=xc if r == 0 else None, norm_w=nw)
        assert (sel == fsel).all()
        # T = 1: qwb_moe_ffn routes with the batch-1 decode router, which sums the logits
        # and the softmax in another f32 order than the batched router used here
        assert torch.allclose(w, fw, rtol=1e-5, atol=0), float(((w - fw).abs() / fw.abs()).max())
        total += part
    flags, bad, cnt = qwb.read_status()
    assert flags == 0, (flags, bad, cnt)
    out = total.cpu().numpy()
    e = O.nrmse(out, fused.cpu().numpy())
    assert e <= 1e-5, (e, O.max_abs_rel(out, fused.cpu().numpy()))
    if H == 4096 and O.ref_available():
        # the reference's own CPU backend (multi-threaded) for the large layer
        O.set_ref_threads(max(1, len(os.sched_getaffinity(0))))
        want = O.moe_layer(x, router_w, t_gu, gate, up, t_d, down, F, E, K, norm_w=norm_w, impl="ref")
    else:
        want = O.moe_layer(x, router_w, t_gu, gate, up, t_d, down, F, E, K, norm_w=norm_w)
    assert (want["selected"] == fsel.cpu().numpy()).all()
    e = O.nrmse(out - x, want["out"])
    print(f"EP H={H} T={T} world={world}: nrmse vs oracle {e:.3e}")
    assert e <= 1e-4, (e, O.max_abs_rel(out - x, want["out"]))


def test_unselected_shard_gives_zeros_and_no_error(qwb):
    # a shard whose experts no token selected returns exactly its residual input (zero
    # without one) and raises no device error
    H, F, E, K, T = 2048, 768, 32, 8, 2
    router_w, norm_w, gate, up, down = _layer(O.Q4_K, O.Q6_K, H, F, E, seed=80)
    G = qwb.QTensor.from_bytes(gate, O.Q4_K, (H, F, E))
    U = qwb.QTensor.from_bytes(up, O.Q4_K, (H, F, E))
    Dn = qwb.QTensor.from_bytes(down, O.Q6_K, (F, H, E))
    x = cu(D.acts((T, H), seed=81))
    # a mask that leaves only experts 0..7 selectable: shard [16, 32) gets no pair
    mask = torch.full((T, E), float("-inf"), device="cuda")
    mask[:, :8] = 0.0
    qwb.read_status()
    part, sel, _ = qwb.ops.moe_ep_layer(x, cu(router_w), _shard(qwb, G, O.Q4_K, H, F, 16, 16),
                                        _shard(qwb, U, O.Q4_K, H, F, 16, 16), _shard(qwb, Dn, O.Q6_K, F, H, 16, 16),
                                        16, K, norm_w=cu(norm_w), mask=mask)
    flags, _, _ = qwb.read_status()
    assert flags == 0
    assert (sel < 8).all()
    assert not part.any()
    part, _, _ = qwb.ops.moe_ep_layer(x, cu(router_w), _shard(qwb, G, O.Q4_K, H, F, 16, 16),
                                      _shard(qwb, U, O.Q4_K, H, F, 16, 16), _shard(qwb, Dn, O.Q6_K, F, H, 16, 16),
                                      16, K, residual=x, norm_w=cu(norm_w), mask=mask)
    assert torch.equal(part, x)


@pytest.mark.parametrize("T,world", [(1, 2), (8, 4), (24, 2)])
def test_shared_expert_on_one_shard(qwb, T, world):
    # the shared expert given to rank 0 only (with the residual): the shards' sum equals
    # the fused layer with the shared expert (pair kernels up to 8 tokens, GEMVs beyond)
    from questwend_b200.expert_parallel import shard_range
    H, F, E, K = 2048, 768, 32, 8
    router_w, norm_w, gate, up, down = _layer(O.Q4_K, O.Q6_K, H, F, E, seed=120 + T)
    r = D.rng(121)
    sh_np = (D.weights(O.Q4_K, 1, F, H, seed=122), D.weights(O.Q4_K, 1, F, H, seed=123),
             D.weights(O.Q6_K, 1, H, F, seed=124))
    gi = cu((r.standard_normal(H, dtype=np.float32) * 0.05).astype(np.float32))
    sh = (qwb.QTensor.from_bytes(sh_np[0], O.Q4_K, (H, F)), qwb.QTensor.from_bytes(sh_np[1], O.Q4_K, (H, F)),
          qwb.QTensor.from_bytes(sh_np[2], O.Q6_K, (F, H)), gi)
    x = D.acts((T, H), seed=125 + T)
    G = qwb.QTensor.from_bytes(gate, O.Q4_K, (H, F, E))
    U = qwb.QTensor.from_bytes(up, O.Q4_K, (H, F, E))
    Dn = qwb.QTensor.from_bytes(down, O.Q6_K, (F, H, E))
    xc, rw, nw = cu(x), cu(router_w), cu(norm_w)
    fused, _, _ = qwb.moe_ffn(xc, rw, G, U, Dn, K, residual=xc, norm_w=nw, shexp=sh)
    fused = fused.clone()
    total = torch.zeros((T, H), device="cuda")
    for rk in range(world):
        lo, n = shard_range(E, world, rk)
        part, _, _ = qwb.ops.moe_ep_layer(xc, rw, _shard(qwb, G, O.Q4_K, H, F, lo, n),
                                          _shard(qwb, U, O.Q4_K, H, F, lo, n), _shard(qwb, Dn, O.Q6_K, F, H, lo, n),
                                          lo, K, residual=xc if rk == 0 else None, norm_w=nw,
                                          shexp=sh if rk == 0 else None)
        total += part
    assert qwb.read_status()[0] == 0
    e = O.nrmse(total.cpu().numpy(), fused.cpu().numpy())
    assert e <= 1e-5, (e, O.max_abs_rel(total.cpu().numpy(), fused.cpu().numpy()))
