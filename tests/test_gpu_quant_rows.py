"""GPU parity: activation quantizers and GET_ROWS are bit-exact with the reference."""
import os

import numpy as np
import pytest
import torch

import oracle as O
import _data as D

pytestmark = pytest.mark.gpu
G = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def qwb():
    import questwend_b200 as q
    q.lib()
    return q


def cu(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_q8K_golden(qwb):
    g = np.load(os.path.join(G, "act_quant.npz"))
    got = qwb.quantize_q8_K(cu(g["act_x"])).cpu().numpy().reshape(-1)
    assert np.array_equal(got, g["act_q8K"])


def test_q80_golden(qwb):
    g = np.load(os.path.join(G, "act_quant.npz"))
    got = qwb.quantize_q8_0(cu(g["act_x"])).cpu().numpy().reshape(-1)
    assert np.array_equal(got, g["act_q80"])


@pytest.mark.parametrize("rows,k", [(1, 256), (7, 2048), (64, 4096), (3, 768)])
def test_quantizers_random(qwb, rows, k):
    x = D.acts((rows, k), seed=rows * 1000 + k) * np.float32(3.0)
    x[0, :17] = 0.0
    xc = cu(x)
    assert np.array_equal(qwb.quantize_q8_K(xc).cpu().numpy().reshape(-1), O.quantize_act(O.Q8_K, x))
    for v in (O.Q8_0_CPU, O.Q8_0_REF):
        got = qwb.quantize_q8_0(xc, variant=v).cpu().numpy().reshape(-1)
        assert np.array_equal(got, O.quantize_act(O.Q8_0, x, variant=v)), v


def test_q80_row_not_multiple_of_256(qwb):
    x = D.acts((5, 96), seed=9)
    assert np.array_equal(qwb.quantize_q8_0(cu(x)).cpu().numpy().reshape(-1), O.quantize_act(O.Q8_0, x))


@pytest.mark.parametrize("name,t", [("q4K", O.Q4_K), ("q6K", O.Q6_K), ("q80", O.Q8_0)])
def test_get_rows_golden_quant(qwb, name, t):
    g = np.load(os.path.join(G, "get_rows.npz"))
    src = qwb.QTensor.from_bytes(g[f"{name}_tab"], t, (512, 16))
    out = qwb.get_rows(src, cu(g["idx"]))
    assert np.array_equal(out.cpu().numpy().reshape(-1, 512).view(np.uint32), g[f"{name}_out"].view(np.uint32))


def test_get_rows_golden_f32_i32(qwb):
    g = np.load(os.path.join(G, "get_rows.npz"))
    out = qwb.get_rows(cu(g["f32_tab"]), cu(g["idx"]))
    assert np.array_equal(out.cpu().numpy().reshape(-1, 64).view(np.uint32), g["f32_out"].view(np.uint32))
    out = qwb.get_rows(cu(g["i32_tab"]), cu(g["idx"]))
    assert np.array_equal(out.cpu().numpy().reshape(-1), g["i32_out"].reshape(-1))


@pytest.mark.parametrize("t", [O.Q4_K, O.Q6_K, O.Q8_0, O.F16])
def test_get_rows_random_large(qwb, t):
    nrows, ne0, n = 1000, 4096, 512
    rng = D.rng(t)
    idx = rng.integers(0, nrows, n).astype(np.int32)
    idx[n // 2:] = idx[:n // 2]  # 50 % repeats
    idx[0], idx[1] = 0, nrows - 1
    if t == O.F16:
        tab = rng.standard_normal((nrows, ne0)).astype(np.float16)
        src = cu(tab)
        want, _ = O.get_rows(O.F16, tab.view(np.uint16), ne0, nrows, idx)
    else:
        raw = D.weights(t, 1, nrows, ne0, seed=t, scale=1.0)
        src = qwb.QTensor.from_bytes(raw, t, (ne0, nrows))
        want, _ = O.get_rows(t, raw, ne0, nrows, idx)
    got = qwb.get_rows(src, cu(idx)).cpu().numpy().reshape(n, ne0)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_get_rows_slot_table_3d(qwb):
    # in-graph slot remap: get_rows(g2s [1, E], selected [n_used, T]) and the 3D form
    E, k, T = 128, 8, 3
    g2s = D.rng(1).permutation(E).astype(np.int32).reshape(E, 1)
    sel = np.stack([D.rng(10 + t).choice(E, k, replace=False) for t in range(1)]).astype(np.int32)
    out = qwb.get_rows(cu(g2s), cu(sel.reshape(k)))
    assert np.array_equal(out.cpu().numpy().reshape(-1), g2s[sel.reshape(-1), 0])
    # probs3 [1, E, T] gathered by selected [k, T] -> [1, k, T]
    probs = D.acts((T, E, 1), seed=4)
    selT = np.stack([D.rng(20 + t).choice(E, k, replace=False) for t in range(T)]).astype(np.int32)
    out = qwb.get_rows(cu(probs), cu(selT)).cpu().numpy().reshape(T, k)
    want = np.take_along_axis(probs[:, :, 0], selT, axis=1)
    assert np.array_equal(out.view(np.uint32), want.view(np.uint32))


def test_get_rows_bad_index_reports(qwb):
    qwb.read_status()
    tab = D.acts((16, 256), seed=2)
    idx = np.array([1, 16, -1, 3], dtype=np.int32)
    out = qwb.get_rows(cu(tab), cu(idx)).cpu().numpy().reshape(4, 256)
    flags, bad, count = qwb.read_status()
    assert flags & 2 and count == 2 and bad in (16, -1)
    assert np.array_equal(out[0], tab[1]) and np.array_equal(out[3], tab[3])
    assert not out[1].any() and not out[2].any()
