"""The drop-in: libggml-qwb.so as the "cuda" backend of an unchanged ggml host.

The library is installed the way a QuestWend deployment would install it: in one
directory as libggml-cuda-qwb.so beside the stock ggml-cuda backend (the reference's own
ggml-cuda compiled for sm_100a, oracle/_ref/cuda/libggml-cuda.so) under its usual name
libggml-cuda.so.  The host is the reference's own ggml (oracle/_ref), which
  * discovers backends with ggml_backend_load_all_from_path and takes the first GPU device
    that initialises, as core/runtime.cpp:996-1010 does: it must be QWB0, wrapping
    ggml-cuda's device;
  * builds a stack of QuestWend MoE FFN blocks (rms_norm * ffn_norm, build_moe of
    core/runtime.cpp:2743-2816, residual add; an identity scale between blocks stands in
    for attention) with ggml's graph allocator and calls
    ggml_backend_graph_compute on the whole graph, as runtime.cpp:6177-6178 does.
Every node the library does not compute goes to the wrapped ggml-cuda backend; each
build_moe subgraph runs as one qwb_moe_ffn call.

Checks: GGML_STATUS_SUCCESS, the fused-layer / delegated-node counters, and every layer
of the stack against the reference's CPU backend on the same input: the GPU's output
after l layers is compared with the CPU's layer l applied to the GPU's output after l-1
layers (nRMS <= 1e-4, max abs-rel in the message).  Whole stacks are not compared end to
end at that bar: an activation value one fp32 ulp away from a Q8_K rounding boundary
flips one code, and the reference's own layer output moves by ~1e-3 for such a flip, so
two correct computations drift apart after a few layers.  Also covered: the expert-cache
branch (in-graph slot remap; each layer's selection record read back), the per-node path
with fusion off (ggml-cuda computes SwiGLU and the weighting there, so its act values
differ from the CPU's in the last bits and cross Q8_K boundaries: the chained bar 3e-4),
and the stock ggml-cuda backend on the same graph (the GPU baseline, checked loosely: it
quantizes activations to Q8_1, not the CPU backend's Q8_K)."""
import os
import shutil
import subprocess
import sys

import numpy as np
import pytest

import oracle as O
import _data as D

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
QWB_LIB = os.path.join(ROOT, "questwend_b200", "libggml-qwb.so")
LIBQWB = os.path.join(ROOT, "questwend_b200", "libqwb.so")
CUDA_LIB = os.path.join(ROOT, "oracle", "_ref", "cuda", "libggml-cuda.so")
TOL = 1e-4

needs = pytest.mark.skipif(not (O.ref_available() and os.path.exists(CUDA_LIB) and os.path.exists(QWB_LIB)),
                           reason="reference ggml, its ggml-cuda build or libggml-qwb.so missing")

_BLK = {O.Q4_K: (144, 0), O.Q6_K: (210, 208), O.Q8_0: (34, 0)}


def scaled_images(t, n, rows, K, seed, n_base=4):
    """n distinct expert byte images: base image i % n_base with its block scales d times
    (1 + i/64)."""
    base = D.weights(t, n_base, rows, K, seed=seed)
    nbytes, off = _BLK[t]
    per = base.size // n_base
    b = base.reshape(n_base, per // nbytes, nbytes)
    out = np.empty((n, per // nbytes, nbytes), dtype=np.uint8)
    for i in range(n):
        blk = b[i % n_base].copy()
        d = blk[:, off:off + 2].copy().view(np.float16).astype(np.float32)
        blk[:, off:off + 2] = (d * np.float32(1.0 + i / 64.0)).astype(np.float16).view(np.uint8)
        out[i] = blk
    return out.reshape(-1)


@pytest.fixture(scope="module")
def install(tmp_path_factory):
    """The deployment layout: <dir>/libggml-cuda-qwb.so + <dir>/libggml-cuda.so."""
    d = tmp_path_factory.mktemp("ggml_backends")
    shutil.copy(QWB_LIB, d / "libggml-cuda-qwb.so")
    os.symlink(CUDA_LIB, d / "libggml-cuda.so")
    os.symlink(LIBQWB, d / "libqwb.so")  # resolved through the copy's $ORIGIN run path
    return str(d)


@pytest.fixture(scope="module")
def model():
    H, F, E, n_used, L = 2048, 768, 32, 8, 3
    rng = D.rng(5)
    m = dict(H=H, F=F, E=E, n_used=n_used, L=L,
             g=scaled_images(O.Q4_K, E, F, H, seed=11), u=scaled_images(O.Q4_K, E, F, H, seed=12),
             d=scaled_images(O.Q6_K, E, H, F, seed=13),
             rw=(rng.standard_normal((L, E, H), dtype=np.float32) * 0.02).astype(np.float32),
             nw=(1.0 + 0.1 * rng.standard_normal((L, H), dtype=np.float32)).astype(np.float32))
    O.set_ref_threads(max(1, len(os.sched_getaffinity(0))))
    return m


def stack(path, m, T, x, L=None, k0=0, g2s=None, n_slots=0, params=None, iters=0):
    """The MoE stack of layers k0 .. k0+L-1 of the model (expert images rotated so the
    stack's layer 0 is the model's layer k0)."""
    L = m["L"] - k0 if L is None else L
    E = m["E"]

    def rot(a):
        per = a.size // E
        return np.concatenate([a[((e + k0) % E) * per:((e + k0) % E + 1) * per] for e in range(E)])
    return O.backend_moe_stack(path, L, m["H"], m["F"], E, m["n_used"], T, O.Q4_K, rot(m["g"]), rot(m["u"]),
                               O.Q6_K, rot(m["d"]), E, m["rw"][k0:k0 + L], m["nw"][k0:k0 + L], x,
                               g2s=None if g2s is None else g2s[k0:k0 + L], n_slots=n_slots, iters=iters,
                               params=params)


def layerwise(path, m, T, x, tol, g2s=None, n_slots=0, params=None):
    """GPU stacks of 1 .. L layers; layer l checked against the CPU's layer l on the GPU's
    output after l - 1 layers.  Returns the last GPU run."""
    prev, got = x, None
    for l in range(1, m["L"] + 1):
        got = stack(path, m, T, x, L=l, g2s=g2s, n_slots=n_slots, params=params)
        assert got["rc"] == 0, got["rc"]
        want = stack(None, m, T, prev, L=1, k0=l - 1, g2s=g2s, n_slots=n_slots)
        assert want["rc"] == 0
        e, mar = O.nrmse(got["out"], want["out"]), O.max_abs_rel(got["out"], want["out"])
        print(f"layer {l} T={T} {params}: nrmse {e:.3e} max_abs_rel {mar:.3e} stats {got['stats']}")
        assert e <= tol, (l, e, mar)
        if g2s is not None:
            assert np.array_equal(got["selected"][l - 1], want["selected"][0]), l
        prev = got["out"]
    return got


@needs
def test_first_gpu_device_is_qwb(install):
    # a fresh process: the host registry must hold only what this directory provides
    code = ("import sys; sys.path.insert(0, %r); import oracle as O; print(O.dropin_first_gpu(%r))"
            % (ROOT, install))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip().splitlines()[-1] == "QWB0", r.stdout + r.stderr[-2000:]


@needs
@pytest.mark.parametrize("T", [1, 8])
def test_stack_fused_layerwise_against_cpu(install, model, T):
    x = D.acts((T, model["H"]), seed=20 + T)
    got = layerwise(os.path.join(install, "libggml-cuda-qwb.so"), model, T, x, TOL)
    fused, own, inner_nodes, inner_runs, delegating = got["stats"]
    assert delegating == 1
    # every block fused (ffn_norm, routing, experts, weighted sum, residual); the scale
    # standing in for attention between blocks runs on ggml-cuda
    assert fused == model["L"] and own == 0 and inner_nodes >= model["L"] and inner_runs >= model["L"], got["stats"]
    # repeated computes of the same graph give the same result
    again = stack(os.path.join(install, "libggml-cuda-qwb.so"), model, T, x, iters=2)
    assert again["stats"][0] == 3 * model["L"]
    assert np.array_equal(again["out"], got["out"])


@needs
def test_stack_per_node_path(install, model):
    T = 4
    x = D.acts((T, model["H"]), seed=30)
    got = layerwise(os.path.join(install, "libggml-cuda-qwb.so"), model, T, x, 3e-4, params="fuse=0")
    fused, own, inner_nodes, inner_runs, _ = got["stats"]
    assert fused == 0 and own == 3 * model["L"] and inner_runs >= model["L"], got["stats"]


@needs
def test_stack_expert_cache_branch(install, model):
    E, L = model["E"], model["L"]
    r = D.rng(40)
    # every expert resident in a pool slot of its own (same permutation for all roles)
    perms = [r.permutation(E).astype(np.int32) for _ in range(L)]
    g2s = np.stack([np.stack([p, p, p]) for p in perms])  # [L][3][E]
    x = D.acts((1, model["H"]), seed=41)
    got = layerwise(os.path.join(install, "libggml-cuda-qwb.so"), model, 1, x, TOL, g2s=g2s, n_slots=E)
    assert got["stats"][0] == L, got["stats"]
    # the slot-remap graph computes what the resident graph computes
    res = stack(os.path.join(install, "libggml-cuda-qwb.so"), model, 1, x)
    assert O.nrmse(res["out"], got["out"]) <= 1e-6


@needs
def test_stock_ggml_cuda_baseline_runs(model):
    T = 1
    x = D.acts((T, model["H"]), seed=50)
    want = stack(None, model, T, x, L=1)
    got = stack(CUDA_LIB, model, T, x, L=1)
    assert got["rc"] == 0
    e = O.nrmse(got["out"], want["out"])
    print(f"stock ggml-cuda, one layer: nrmse {e:.3e} (Q8_1 activations)")
    assert e <= 2e-2, e


@needs
@pytest.mark.parametrize("T,gate", [(1, True), (4, False)])
def test_stack_shared_expert_fused_layerwise(install, model, T, gate):
    # blocks with a shared expert (runtime.cpp:2825-2833): the shared expert's nodes join
    # the fused qwb_moe_ffn call (its shexp operands), still one call per block
    H, F, L = model["H"], model["F"], model["L"]
    r = D.rng(60)
    sg = D.weights(O.Q4_K, 1, F, H, seed=61)
    su = D.weights(O.Q4_K, 1, F, H, seed=62)
    sd = D.weights(O.Q6_K, 1, H, F, seed=63)
    # one gate row for every layer: the CPU check of layer l runs a 1-layer stack
    gi = np.tile((r.standard_normal(H, dtype=np.float32) * 0.05).astype(np.float32), (L, 1)) if gate else None
    O.stack_set_shexp(sg, su, sd, F, gi)
    try:
        x = D.acts((T, H), seed=64 + T)
        got = layerwise(os.path.join(install, "libggml-cuda-qwb.so"), model, T, x, TOL)
        fused, own, _, _, _ = got["stats"]
        assert fused == L and own == 0, got["stats"]
    finally:
        O.stack_set_shexp()
