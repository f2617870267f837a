"""GPU parity at the workloads' own shapes (not scaled-down stand-ins).

* Prefill sweep shape: hidden 4096, expert FFN 1536, 128 experts, top-8, T = 2048 tokens,
  routing from Gumbel-perturbed Zipf(1.1) popularity.  MUL_MAT_ID for the Q4_K gate/up
  shape (one activation row per token), the Q4_K and Q6_K down shapes (one row per
  (token, slot)) and the Q8_0 gate/up shape, each against the reference's own ggml CPU
  backend compiled from its sources (oracle/_ref; experts with >= 8 rows take its tiled
  path).  Bar: nRMS <= 1e-4; the max abs-rel error is in the message.
* Single MoE layer, hidden 2048, 128 experts, top-8, expert FFN 768, through the fused
  layer (qwb_moe_ffn: router, top-k, gate/up, SwiGLU, down, weighted sum) against the
  reference's build_moe graph on its CPU backend: Q4_K down (the single-layer workload)
  and Q6_K down (the Q4_K_M mix).  Selection identical, nRMS <= 1e-4.
* GET_ROWS on the full 151936 x 4096 embedding table in Q4_K / Q6_K / Q8_0 with an
  8192-index stream (uniform, 50 % repeats, rows 0 and 151935 included): bit-exact
  against the oracle's dequantisation.

Expert and table bytes: generating 128 distinct full-size quantized experts per case
would take minutes of CPU quantisation, so expert e is ggml-quantized N(0, 0.02) base
matrix e mod n_base with every block's fp16 scale d multiplied by (1 + e/256): every
expert (and every table row, with its own factor) is a different, valid block matrix, so
an expert or row mix-up changes the result."""
import os

import numpy as np
import pytest
import torch

import oracle as O
import _data as D

pytestmark = pytest.mark.gpu
TOL = 1e-4

# bytes per block and offset of the fp16 scale d inside it (ggml-common.h)
_BLK = {O.Q4_K: (144, 0), O.Q6_K: (210, 208), O.Q8_0: (34, 0)}


def scaled_copies(base: np.ndarray, t: int, n_base: int, n_out: int, factor) -> np.ndarray:
    """n_out matrices: copy i is base matrix i % n_base with d scaled by factor(i)."""
    nbytes, off = _BLK[t]
    per = base.size // n_base
    b = base.reshape(n_base, per // nbytes, nbytes)
    out = np.empty((n_out, per // nbytes, nbytes), dtype=np.uint8)
    for i in range(n_out):
        blk = b[i % n_base].copy()
        d = blk[:, off:off + 2].copy().view(np.float16).astype(np.float32)
        blk[:, off:off + 2] = (d * np.float32(factor(i))).astype(np.float16).view(np.uint8)
        out[i] = blk
    return out.reshape(-1)


def expert_pool(t, n_exp, rows, K, seed, n_base=4):
    base = D.weights(t, n_base, rows, K, seed=seed)
    return scaled_copies(base, t, n_base, n_exp, lambda e: 1.0 + e / 256.0)


def _threads():
    return max(1, len(os.sched_getaffinity(0)))


@pytest.fixture(scope="module")
def qwb():
    import questwend_b200 as q
    q.lib()
    return q


def cu(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


needs_ref = pytest.mark.skipif(not O.ref_available(), reason="reference CPU build (oracle/_ref) missing")

PF_H, PF_F, E, K_USED, PF_T = 4096, 1536, 128, 8, 2048


@needs_ref
@pytest.mark.parametrize("t,shape", [(O.Q4_K, "gate_up"), (O.Q4_K, "down"), (O.Q8_0, "gate_up"),
                                     (O.Q6_K, "down")])
def test_prefill_shape_against_reference_build(qwb, t, shape):
    K, M, n_b = (PF_H, PF_F, 1) if shape == "gate_up" else (PF_F, PF_H, K_USED)
    w = expert_pool(t, E, M, K, seed=1000 + t * 10 + n_b)
    b = D.acts((PF_T, n_b, K), seed=2000 + n_b)
    ids = D.zipf_ids(PF_T, E, K_USED, seed=3000)
    W = qwb.QTensor.from_bytes(w, t, (K, M, E))
    got = qwb.mul_mat_id(W, cu(b), cu(ids)).cpu().numpy()
    flags, _, _ = qwb.read_status()
    assert flags == 0
    del W
    torch.cuda.empty_cache()
    O.set_ref_threads(_threads())
    want, _ = O.mul_mat_id(t, w, K, M, E, b, ids, impl="ref")
    e, mar = O.nrmse(got, want), O.max_abs_rel(got, want)
    print(f"prefill {shape} type {t} T={PF_T}: nrmse {e:.3e} max_abs_rel {mar:.3e}")
    assert e <= TOL, (e, mar)


@needs_ref
@pytest.mark.parametrize("down_t", [O.Q4_K, O.Q6_K])
@pytest.mark.parametrize("T", [1, 8])
def test_moe_layer_128_experts_against_reference_build(qwb, down_t, T):
    H, F = 2048, 768
    rng = D.rng(40 + T)
    rw = (rng.standard_normal((E, H), dtype=np.float32) * 0.02).astype(np.float32)
    nw = (1.0 + 0.1 * rng.standard_normal(H, dtype=np.float32)).astype(np.float32)
    x = D.acts((T, H), seed=41 + T)
    g = expert_pool(O.Q4_K, E, F, H, seed=50)
    u = expert_pool(O.Q4_K, E, F, H, seed=51)
    d = expert_pool(down_t, E, H, F, seed=52)
    Wg = qwb.QTensor.from_bytes(g, O.Q4_K, (H, F, E))
    Wu = qwb.QTensor.from_bytes(u, O.Q4_K, (H, F, E))
    Wd = qwb.QTensor.from_bytes(d, down_t, (F, H, E))
    out, sel, wts = qwb.moe_ffn(cu(x), cu(rw), Wg, Wu, Wd, K_USED, norm_w=cu(nw), norm_eps=1e-6)
    torch.cuda.synchronize()
    flags, _, _ = qwb.read_status()
    assert flags == 0
    O.set_ref_threads(_threads())
    ref = O.moe_layer(x, rw, O.Q4_K, g, u, down_t, d, F, E, K_USED, impl="ref", norm_w=nw, norm_eps=1e-6)
    assert np.array_equal(sel.cpu().numpy(), ref["selected"])
    assert O.nrmse(wts.cpu().numpy(), ref["weights"]) <= 1e-6
    got = out.cpu().numpy()
    e, mar = O.nrmse(got, ref["out"]), O.max_abs_rel(got, ref["out"])
    print(f"moe layer E=128 T={T} down {down_t}: nrmse {e:.3e} max_abs_rel {mar:.3e}")
    assert e <= TOL, (e, mar)


VOCAB, EMB = 151936, 4096


@pytest.mark.parametrize("t", [O.Q4_K, O.Q6_K, O.Q8_0])
def test_get_rows_full_table(qwb, t):
    n_base = 256
    base = D.weights(t, 1, n_base, EMB, seed=60 + t)
    # row r = base row r % 256 with its scales times 1 + (r % 997) / 1024
    nbytes, off = _BLK[t]
    rb = base.size // n_base
    tab = np.tile(base.reshape(n_base, rb), (-(-VOCAB // n_base), 1))[:VOCAB]
    blocks = tab.reshape(VOCAB, rb // nbytes, nbytes)
    fac = (1.0 + (np.arange(VOCAB) % 997) / 1024.0).astype(np.float32)
    d = blocks[:, :, off:off + 2].copy().view(np.float16).astype(np.float32)
    blocks[:, :, off:off + 2] = (d * fac[:, None, None]).astype(np.float16).view(np.uint8)
    tab = tab.reshape(-1)
    r = D.rng(70 + t)
    uniq = r.integers(0, VOCAB, 4094)
    idx = np.concatenate([[0, VOCAB - 1], uniq, r.choice(uniq, 8192 - 4096)])
    idx = r.permutation(idx).astype(np.int32)
    src = qwb.QTensor.from_bytes(tab, t, (EMB, VOCAB))
    got = qwb.get_rows(src, cu(idx)).cpu().numpy().reshape(idx.size, EMB)
    want, rc = O.get_rows(t, tab, EMB, VOCAB, idx)
    assert rc == 0
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
