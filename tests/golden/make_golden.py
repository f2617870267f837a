"""Generate the golden fixtures in this directory from the REFERENCE ggml CPU backend.

Run in a container where the reference sources are present and oracle/_ref was built
(``make -C oracle``):

    python tests/golden/make_golden.py

Each fixture stores small inputs (or the seed and shapes that regenerate them through
tests/_data.py) and the outputs of the reference's own ggml CPU backend
(oracle/_ref/libqwbref.so: ggml_quantize_chunk, the CPU backend's from_float,
ggml_get_rows / ggml_mul_mat_id / the build_moe graph).  The tests compare the C
restatement (oracle/) and the CUDA path against them; the reference is not needed at
test time.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

import oracle as O  # noqa: E402
import _data as D  # noqa: E402


def special_rows(k):
    r = D.rng(7)
    rows = [
        r.standard_normal(k).astype(np.float32),                 # plain
        np.zeros(k, np.float32),                                 # all-zero blocks
        r.standard_normal(k).astype(np.float32),                 # |max| tie, opposite signs
        (np.arange(k, dtype=np.float32) % 255 - 127) / 127.0,    # exact grid values
        r.standard_normal(k).astype(np.float32) * 1e-30,         # tiny / subnormal products
        r.standard_normal(k).astype(np.float32) * 1e30,          # huge
        np.full(k, -2.5, np.float32),                            # constant negative
        r.uniform(-1, 1, k).astype(np.float32),
    ]
    rows[2][5] = -3.0
    rows[2][77] = 3.0
    rows[2][300 % k] = 3.0
    rows[3][::7] *= 0.5  # half-way products
    return np.stack(rows)


def main():
    assert O.ref_available(), "build oracle/_ref first (make -C oracle)"
    O.set_ref_threads(4)
    out = {}

    # activation quantizers: the CPU backend's from_float (Q8_K, Q8_0 x86 variant)
    x = special_rows(512)
    out["act_x"] = x
    out["act_q8K"] = O.quantize_act(O.Q8_K, x, impl="ref")
    out["act_q80"] = O.quantize_act(O.Q8_0, x, impl="ref")
    np.savez_compressed(os.path.join(HERE, "act_quant.npz"), **out)

    # weight quantizers (ggml_quantize_chunk, no imatrix)
    wx = (D.rng(11).standard_normal((4, 512)) * 0.02).astype(np.float32)
    wx[1, :256] = 0.0  # an all-zero superblock
    np.savez_compressed(os.path.join(HERE, "weights_quant.npz"), x=wx,
                        q4K=O.quantize_weights(O.Q4_K, wx, impl="ref"),
                        q6K=O.quantize_weights(O.Q6_K, wx, impl="ref"),
                        q80=O.quantize_weights(O.Q8_0, wx, impl="ref"))

    # mul_mat_id: K=512, M=64, n_as=8, T=5, n_used=3; b broadcast (n_b=1) and per-slot (n_b=3)
    mm = {}
    K, M, n_as, T, n_used = 512, 64, 8, 5, 3
    ids = np.stack([D.rng(100 + t).choice(n_as, n_used, replace=False) for t in range(T)]).astype(np.int32)
    ids[4] = [7, 7, 0]  # duplicate expert within a token
    mm["ids"] = ids
    for name, t in (("q4K", O.Q4_K), ("q6K", O.Q6_K), ("q80", O.Q8_0)):
        w = D.weights(t, n_as, M, K, seed=21 + t)
        w_ref = O.quantize_weights(t, (D.rng(21 + t).standard_normal((n_as * M, K), dtype=np.float32) * 0.02)
                                   .astype(np.float32), impl="ref")
        assert D.sha(w) == D.sha(w_ref), "restated weight quantizer drifted from the reference"
        mm[f"{name}_wsha"] = np.array(D.sha(w_ref))
        for n_b in (1, n_used):
            b = D.acts((T, n_b, K), seed=31 + n_b)
            mm[f"b{n_b}"] = b
            dst, _ = O.mul_mat_id(t, w_ref, K, M, n_as, b, ids, impl="ref")
            mm[f"{name}_nb{n_b}"] = dst
    np.savez_compressed(os.path.join(HERE, "mul_mat_id.npz"), **mm)

    # get_rows: 16-row tables of 512, duplicate / first / last / repeated indices
    gr = {}
    idx = np.array([3, 0, 15, 3, 7, 7, 15, 1], dtype=np.int32)
    gr["idx"] = idx
    for name, t in (("q4K", O.Q4_K), ("q6K", O.Q6_K), ("q80", O.Q8_0)):
        tab = D.weights(t, 1, 16, 512, seed=41 + t, scale=1.0)
        gr[f"{name}_tab"] = tab
        gr[f"{name}_out"], _ = O.get_rows(t, tab, 512, 16, idx, impl="ref")
    f32 = D.acts((16, 64), seed=5)
    f32.view(np.uint32)[0, :6] = [0x7fc00001, 0xffc12345, 0x80000000, 0x7f800000, 0xff800000, 0x00000001]
    gr["f32_tab"] = f32
    gr["f32_out"], _ = O.get_rows(O.F32, f32, 64, 16, idx, impl="ref")
    i32 = D.rng(6).integers(-2**31, 2**31 - 1, size=(16, 1), dtype=np.int64).astype(np.int32)
    gr["i32_tab"] = i32
    gr["i32_out"], _ = O.get_rows(O.I32, i32, 1, 16, idx, impl="ref")
    np.savez_compressed(os.path.join(HERE, "get_rows.npz"), **gr)

    # full MoE layer (build_moe graph): H=1024, F=256, E=8, k=4, Q4_K gate/up, Q6_K down
    ml = {}
    H, F, E, k = 1024, 256, 8, 4
    rw = (D.rng(51).standard_normal((E, H)) * 0.02).astype(np.float32)
    g = D.weights(O.Q4_K, E, F, H, seed=52)
    u = D.weights(O.Q4_K, E, F, H, seed=53)
    dn = D.weights(O.Q6_K, E, H, F, seed=54)
    ml["router_w"] = rw
    ml["wsha"] = np.array(D.sha(g) + D.sha(u) + D.sha(dn))
    for T in (1, 5):
        x = D.acts((T, H), seed=60 + T)
        r = O.moe_layer(x, rw, O.Q4_K, g, u, O.Q6_K, dn, F, E, k, impl="ref")
        ml[f"x{T}"] = x
        for key in ("out", "selected", "weights"):
            ml[f"{key}{T}"] = r[key]
    # slot-remap branch: experts live in a 12-slot pool, g2s tables per role
    n_slots = 12
    perm = D.rng(70).permutation(n_slots)[:E].astype(np.int32)
    g2s = np.stack([perm, np.roll(perm, 1), np.roll(perm, 2)]).astype(np.int32)
    pool = {}
    for role, (wt, rows, K) in enumerate(((g, F, H), (u, F, H), (dn, H, F))):
        t = O.Q6_K if role == 2 else O.Q4_K
        rs = O.row_size(t, K) * rows
        p = np.zeros(n_slots * rs, np.uint8)
        for e in range(E):
            p[g2s[role, e] * rs:(g2s[role, e] + 1) * rs] = wt[e * rs:(e + 1) * rs]
        pool[role] = p
    x = D.acts((1, H), seed=61)
    r = O.moe_layer(x, rw, O.Q4_K, pool[0], pool[1], O.Q6_K, pool[2], F, n_slots, k, g2s=g2s, impl="ref")
    ml["g2s"] = g2s
    ml["out_remap"] = r["out"]
    np.savez_compressed(os.path.join(HERE, "moe_layer.npz"), **ml)
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
