"""CPU checkers for the quantized MoE hot path -- TEST INFRASTRUCTURE ONLY.

Two backends, both plain C/C++ on the host:

* ``port`` -- ``liboracle.so``, this project's C restatement of the reference's
  ggml arithmetic (``qwb_oracle.c``; every function cites the reference file:line it
  restates).
* ``ref``  -- ``_ref/<isa>/libqwbref.so``, the reference's own ggml CPU backend
  compiled from the reference sources by ``oracle/Makefile`` and driven by
  ``ref_harness.cpp`` (graphs mirroring ``core/runtime.cpp:2693-2816``).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs import this
package, and only as the checker or the timed CPU baseline; the product path
(``questwend_b200``) never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

# ggml enum ggml_type values
F32, F16, Q8_0, Q4_K, Q6_K, Q8_K, I32 = 0, 1, 8, 12, 14, 15, 26
Q8_0_CPU, Q8_0_REF = 0, 1

_BLOCK = {F32: (1, 4), F16: (1, 2), I32: (1, 4), Q8_0: (32, 34), Q4_K: (256, 144),
          Q6_K: (256, 210), Q8_K: (256, 292)}


def row_size(t: int, n: int) -> int:
    blk, nbytes = _BLOCK[t]
    assert n % blk == 0, (t, n)
    return n // blk * nbytes


def vec_dot_type(t: int) -> int:
    return Q8_0 if t == Q8_0 else Q8_K


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


_port = None
_ref = None


def _build_port():
    so = os.path.join(HERE, "liboracle.so")
    src = os.path.join(HERE, "qwb_oracle.c")
    if not os.path.exists(so) or os.path.getmtime(so) < os.path.getmtime(src):
        subprocess.check_call(["make", "-s", "-C", HERE, "oracle"])
    return so


def port():
    """ctypes handle on the C restatement (built on first use when gcc is present)."""
    global _port
    if _port is None:
        lib = C.CDLL(_build_port())
        vp, i64, i32, f32 = C.c_void_p, C.c_int64, C.c_int, C.c_float
        lib.qo_row_size.restype = C.c_size_t
        lib.qo_row_size.argtypes = [i32, i64]
        lib.qo_quantize_weights.argtypes = [i32, vp, vp, i64, i64]
        lib.qo_quantize_row_q8_K.argtypes = [vp, vp, i64]
        lib.qo_quantize_row_q8_0.argtypes = [vp, vp, i64, i32]
        lib.qo_to_float.argtypes = [i32, vp, vp, i64, i64]
        lib.qo_vec_dot.restype = f32
        lib.qo_vec_dot.argtypes = [i32, i64, vp, vp]
        lib.qo_mul_mat_id.argtypes = [i32, vp, i64, i64, i64, vp, i64, i64, vp, i64, i64, vp, i32]
        lib.qo_get_rows.argtypes = [i32, vp, i64, i64, vp, i64, vp]
        lib.qo_route.argtypes = [vp, i64, i64, i64, i32, f32, vp, vp, vp]
        lib.qo_swiglu.argtypes = [vp, vp, vp, i64]
        lib.qo_moe_layer.argtypes = [vp, i64, i64, vp, i64, i64, i32, vp, vp, i32, vp, i64, i64,
                                     vp, vp, vp, vp, vp, vp]
        lib.qo_rms_norm_mul.argtypes = [vp, vp, f32, i64, i64, vp]
        lib.qo_fp32_to_fp16.restype = C.c_uint16
        lib.qo_fp32_to_fp16.argtypes = [f32]
        lib.qo_fnv1a64.restype = C.c_uint64
        lib.qo_fnv1a64.argtypes = [vp, C.c_size_t]
        lib.qo_slab_audit.argtypes = [vp, vp, C.c_size_t] + [vp] * 6
        _port = lib
    return _port


def _host_isa() -> str:
    try:
        flags = open("/proc/cpuinfo").read()
    except OSError:
        return "x86-64-v3"
    need = ("avx512f", "avx512bw", "avx512vl", "avx512dq", "avx512_vnni")
    return "x86-64-v4" if all(f in flags for f in need) else "x86-64-v3"


def ref_path() -> str:
    return os.path.join(HERE, "_ref", _host_isa(), "libqwbref.so")


def ref_available() -> bool:
    return os.path.exists(ref_path())


def ref():
    """ctypes handle on the reference's ggml CPU backend (oracle/_ref), or None."""
    global _ref
    if _ref is None:
        if not ref_available():
            return None
        # global symbols: a ggml backend library loaded through ggml_backend_load resolves
        # its ggml calls against this copy of ggml
        lib = C.CDLL(ref_path(), mode=C.RTLD_GLOBAL)
        vp, i64, i32, f32, f64 = C.c_void_p, C.c_int64, C.c_int, C.c_float, C.c_double
        cp, ip = C.c_char_p, C.POINTER(C.c_int)
        lib.qref_set_threads.argtypes = [i32]
        lib.qref_last_times.restype = i32
        lib.qref_last_times.argtypes = [vp, i32]
        lib.qref_quantize.restype = C.c_size_t
        lib.qref_quantize.argtypes = [i32, vp, vp, i64, i64]
        lib.qref_from_float.argtypes = [i32, vp, vp, i64, i64]
        lib.qref_to_float.argtypes = [i32, vp, vp, i64, i64]
        lib.qref_mul_mat_id.restype = f64
        lib.qref_mul_mat_id.argtypes = [i32, vp, i64, i64, i64, vp, i64, i64, vp, i64, i64, vp, i32]
        lib.qref_get_rows.restype = f64
        lib.qref_get_rows.argtypes = [i32, vp, i64, i64, vp, i64, vp, i32]
        lib.qref_route.restype = f64
        lib.qref_route.argtypes = [vp, i64, i64, i64, i32, f32, vp, vp, vp, i32]
        lib.qref_moe_layer.restype = f64
        lib.qref_moe_layer.argtypes = [vp, i64, i64, vp, i64, i64, i32, vp, vp, i32, vp, i64, i64,
                                       vp, vp, vp, vp, vp, vp, i32, vp, f32]
        lib.qref_moe_layer_shexp.restype = f64
        lib.qref_moe_layer_shexp.argtypes = [vp, i64, i64, vp, i64, i64, i32, vp, vp, i32, vp, i64, i64, vp, f32,
                                             vp, vp, vp, i64, vp, vp, vp, vp]
        lib.qref_backend_mul_mat_id.argtypes = [cp, i32, vp, i64, i64, i64, vp, i64, i64, vp, i64, i64, vp]
        lib.qref_backend_get_rows.argtypes = [cp, i32, vp, i64, i64, vp, i64, vp]
        lib.qref_mul_mat.restype = f64
        lib.qref_mul_mat.argtypes = [i32, vp, i64, i64, vp, i64, vp, i32]
        lib.qref_backend_mul_mat.argtypes = [cp, i32, vp, i64, i64, vp, i64, vp]
        lib.qref_backend_sched_mul_mat_id.argtypes = [cp, i32, vp, i64, i64, i64, vp, i64, vp, i64, f32, vp, ip, ip]
        lib.qref_backend_moe_stack.argtypes = [cp, cp, i32, i64, i64, i64, i64, i64, i32, vp, vp, i32, vp, i64,
                                               vp, vp, vp, vp, i64, vp, vp, i32, C.POINTER(C.c_double),
                                               C.POINTER(C.c_uint64)]
        lib.qref_dropin_first_gpu.argtypes = [cp, C.c_char_p, i32]
        lib.qref_stack_set_shexp.argtypes = [vp, vp, vp, i64, vp]
        _ref = lib
    return _ref


# ------------------------------------------------------------------ port wrappers
def quantize_weights(t: int, x: np.ndarray, impl: str = "port") -> np.ndarray:
    """Quantize f32 rows [..., n_per_row] to type t (ggml_quantize_chunk, no imatrix)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.shape[-1]
    nrow = x.size // n
    out = np.zeros(nrow * row_size(t, n), dtype=np.uint8)
    if impl == "ref":
        ref().qref_quantize(t, _p(x), _p(out), nrow, n)
    else:
        rc = port().qo_quantize_weights(t, _p(x), _p(out), nrow, n)
        assert rc == 0
    return out


def quantize_act(t: int, x: np.ndarray, variant: int = Q8_0_CPU, impl: str = "port") -> np.ndarray:
    """CPU-backend activation quantizer (from_float) for t in {Q8_K, Q8_0}."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    k = x.shape[-1]
    nrow = x.size // k
    out = np.zeros(nrow * row_size(t, k), dtype=np.uint8)
    if impl == "ref":
        assert variant == Q8_0_CPU or t == Q8_K
        assert ref().qref_from_float(t, _p(x), _p(out), nrow, k) == 0
        return out
    lib = port()
    rs = row_size(t, k)
    for r in range(nrow):
        src = x.reshape(nrow, k)[r]
        dst = out[r * rs:(r + 1) * rs]
        if t == Q8_K:
            lib.qo_quantize_row_q8_K(_p(src), _p(dst), k)
        else:
            lib.qo_quantize_row_q8_0(_p(src), _p(dst), k, variant)
    return out


def dequantize(t: int, data: np.ndarray, nrow: int, k: int, impl: str = "port") -> np.ndarray:
    out = np.zeros((nrow, k), dtype=np.float32)
    if impl == "ref":
        assert ref().qref_to_float(t, _p(data), _p(out), nrow, k) == 0
    else:
        assert port().qo_to_float(t, _p(data), _p(out), nrow, k) == 0
    return out


def mul_mat_id(t: int, w: np.ndarray, K: int, M: int, n_as: int, b: np.ndarray,
               ids: np.ndarray, impl: str = "port", q8_0_variant: int = Q8_0_CPU,
               iters: int = 0):
    """dst[T, n_used, M] = ggml_mul_mat_id(as[n_as, M, K], b[T, n_b, K], ids[T, n_used]).

    Returns (dst, rc) for the port, (dst, ms_per_iter) for the reference."""
    b = np.ascontiguousarray(b, dtype=np.float32)
    T, n_b = b.shape[0], b.shape[1]
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    n_used = ids.shape[1]
    ids_stride = ids.strides[0] // 4
    dst = np.zeros((T, n_used, M), dtype=np.float32)
    if impl == "ref":
        ms = ref().qref_mul_mat_id(t, _p(w), K, M, n_as, _p(b), n_b, T, _p(ids), n_used,
                                   ids_stride, _p(dst), iters)
        return dst, ms
    rc = port().qo_mul_mat_id(t, _p(w), K, M, n_as, _p(b), n_b, T, _p(ids), n_used,
                              ids_stride, _p(dst), q8_0_variant)
    return dst, rc


def mul_mat(t: int, w: np.ndarray, K: int, M: int, b: np.ndarray, impl: str = "port", iters: int = 0):
    """dst[T, M] = ggml_mul_mat(a[M, K] quantized, b[T, K]).  impl="ref": the reference's
    ggml CPU backend (returns (dst, ms_per_iter)); "port": the restatement's mul_mat_id
    with one expert that every token selects (the same dots; returns (dst, rc))."""
    b = np.ascontiguousarray(b, dtype=np.float32).reshape(-1, K)
    T = b.shape[0]
    if impl == "ref":
        dst = np.zeros((T, M), dtype=np.float32)
        ms = ref().qref_mul_mat(t, _p(w), K, M, _p(b), T, _p(dst), iters)
        return dst, ms
    dst, rc = mul_mat_id(t, w, K, M, 1, b.reshape(T, 1, K), np.zeros((T, 1), dtype=np.int32))
    return dst.reshape(T, M), rc


def get_rows(t: int, src: np.ndarray, ne0: int, nrows: int, idx: np.ndarray,
             impl: str = "port", iters: int = 0):
    idx = np.ascontiguousarray(idx, dtype=np.int32)
    dt = np.int32 if t == I32 else np.float32
    dst = np.zeros((idx.size, ne0), dtype=dt)
    if impl == "ref":
        ms = ref().qref_get_rows(t, _p(src), ne0, nrows, _p(idx), idx.size, _p(dst), iters)
        return dst, ms
    rc = port().qo_get_rows(t, _p(src), ne0, nrows, _p(idx), idx.size, _p(dst))
    return dst, rc


# ------------------------------------------------- a ggml backend loaded by ggml itself
def backend_mul_mat_id(path: str, t: int, w: np.ndarray, K: int, M: int, n_as: int, b: np.ndarray,
                       ids: np.ndarray, n_used: int | None = None):
    """mul_mat_id computed by the ggml backend library at `path`, loaded with the
    reference ggml's own ggml_backend_load and driven through ggml_backend_graph_compute.
    ids [T, W]: the op uses its first n_used columns (a strided view when n_used < W).
    Returns (dst [T, n_used, M], rc); rc 0 on success."""
    b = np.ascontiguousarray(b, dtype=np.float32)
    T, n_b = b.shape[0], b.shape[1]
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    n_used = ids.shape[1] if n_used is None else n_used
    dst = np.zeros((T, n_used, M), dtype=np.float32)
    rc = ref().qref_backend_mul_mat_id(path.encode(), t, _p(w), K, M, n_as, _p(b), n_b, T, _p(ids), n_used,
                                       ids.shape[1], _p(dst))
    return dst, rc


def backend_get_rows(path: str, t: int, src: np.ndarray, ne0: int, nrows: int, idx: np.ndarray):
    """get_rows computed by the ggml backend library at `path`.  Returns (dst, rc)."""
    idx = np.ascontiguousarray(idx, dtype=np.int32)
    dst = np.zeros((idx.size, ne0), dtype=np.int32 if t == I32 else np.float32)
    rc = ref().qref_backend_get_rows(path.encode(), t, _p(src), ne0, nrows, _p(idx), idx.size, _p(dst))
    return dst, rc


def backend_mul_mat(path: str, t: int, w: np.ndarray, K: int, M: int, b: np.ndarray):
    """mul_mat computed by the ggml backend library at `path`.  Returns (dst [T, M], rc)."""
    b = np.ascontiguousarray(b, dtype=np.float32).reshape(-1, K)
    dst = np.zeros((b.shape[0], M), dtype=np.float32)
    rc = ref().qref_backend_mul_mat(path.encode(), t, _p(w), K, M, _p(b), b.shape[0], _p(dst))
    return dst, rc


def backend_sched_mul_mat_id(path: str, t: int, w: np.ndarray, K: int, M: int, n_as: int, b: np.ndarray,
                             ids: np.ndarray, scale: float):
    """scale * mul_mat_id through ggml_backend_sched over [the backend at `path`, CPU], the
    weights in the loaded backend's weight buffer.  Returns (dst, rc, n_splits,
    mul_mat_id placed on the loaded backend)."""
    b = np.ascontiguousarray(b, dtype=np.float32).reshape(b.shape[0], 1, K)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    T, n_used = ids.shape
    dst = np.zeros((T, n_used, M), dtype=np.float32)
    n_splits, on_backend = C.c_int(0), C.c_int(0)
    rc = ref().qref_backend_sched_mul_mat_id(path.encode(), t, _p(w), K, M, n_as, _p(b), T, _p(ids), n_used,
                                             scale, _p(dst), C.byref(n_splits), C.byref(on_backend))
    return dst, rc, n_splits.value, bool(on_backend.value)


def backend_moe_stack(path, L, H, F, E, n_used, T, type_gu, gate_u, up_u, type_d, down_u, n_unique,
                      router_w, norm_w, x, g2s=None, n_slots=0, iters=0, params=None):
    """A stack of L QuestWend MoE FFN blocks (ffn_norm, build_moe, residual) computed by
    the ggml backend library at `path` (None: the reference's CPU backend).  Expert e of
    layer l is image (e + l) % n_unique of gate_u / up_u / down_u.  g2s [L][3][E] selects
    the expert-cache branch (slot pools of n_slots, T = 1).  Returns dict(rc, out [T, H],
    selected [L, n_used] (cache branch), ms per run, stats: fused layers, nodes run one at
    a time on libqwb.so, nodes delegated, delegated runs, delegating mode)."""
    out = np.zeros((T, H), dtype=np.float32)
    sel = np.zeros((L, n_used), dtype=np.int32)
    ms = C.c_double(0.0)
    st = (C.c_uint64 * 5)()
    g = None if g2s is None else np.ascontiguousarray(g2s, dtype=np.int32)
    rw = np.ascontiguousarray(router_w, dtype=np.float32)
    nw = np.ascontiguousarray(norm_w, dtype=np.float32)
    xx = np.ascontiguousarray(x, dtype=np.float32)
    rc = ref().qref_backend_moe_stack(None if path is None else path.encode(),
                                      None if params is None else params.encode(), L, H, F, E, n_used, T,
                                      type_gu, _p(gate_u), _p(up_u), type_d, _p(down_u), n_unique, _p(rw), _p(nw),
                                      _p(xx), _p(g), n_slots, _p(out), _p(sel), iters, C.byref(ms), st)
    return dict(rc=rc, out=out, selected=sel, ms=ms.value, stats=list(st))


_stack_sh_keep = None


def stack_set_shexp(gate=None, up=None, down=None, Fs=0, gate_inp=None):
    """Give every block of backend_moe_stack the shared expert of core/runtime.cpp:2825-2833
    (byte images gate/up [H, Fs] and down [Fs, H], the same for every layer; gate_inp
    [L][H] f32 sigmoid gate weights or None); stack_set_shexp() removes it."""
    global _stack_sh_keep
    gi = None if gate_inp is None else np.ascontiguousarray(gate_inp, dtype=np.float32)
    g, u, d = (None if a is None else np.ascontiguousarray(a) for a in (gate, up, down))
    _stack_sh_keep = (g, u, d, gi)  # the library keeps the pointers
    ref().qref_stack_set_shexp(_p(g), _p(u), _p(d), Fs, _p(gi))


def dropin_first_gpu(directory: str) -> str:
    """ggml_backend_load_all_from_path(directory), then the name of the first GPU device
    that initialises: the device QuestWend's runtime takes (core/runtime.cpp:996-1010)."""
    buf = C.create_string_buffer(256)
    rc = ref().qref_dropin_first_gpu(directory.encode(), buf, 256)
    return buf.value.decode() if rc == 0 else f"<error {rc}>"


def route(logits: np.ndarray, n_used: int, norm: bool = True, scale: float = 0.0,
          mask: np.ndarray | None = None, impl: str = "port", iters: int = 0):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    T, E = logits.shape
    sel = np.zeros((T, n_used), dtype=np.int32)
    w = np.zeros((T, n_used), dtype=np.float32)
    m = None if mask is None else np.ascontiguousarray(mask, dtype=np.float32)
    if impl == "ref":
        ref().qref_route(_p(logits), E, T, n_used, int(norm), scale, _p(m), _p(sel), _p(w), iters)
    else:
        port().qo_route(_p(logits), E, T, n_used, int(norm), scale, _p(m), _p(sel), _p(w))
    return sel, w


def rms_norm_mul(x, w, eps):
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    y = np.zeros_like(x)
    port().qo_rms_norm_mul(_p(x), _p(w), eps, x.shape[0], x.shape[1], _p(y))
    return y


def moe_layer_shexp(x, router_w, type_gu, gate, up, type_d, down, F, n_mat, n_used, sh_gate, sh_up, sh_down, Fs,
                    sh_gate_inp=None, norm_w=None, norm_eps: float = 1e-6):
    """One build_moe layer plus the shared expert of core/runtime.cpp:2825-2833 (gate/up of
    type_gu [H, Fs], down of type_d [Fs, H], optional sigmoid gate [H]) on the reference's
    own ggml CPU backend (oracle/_ref).  Returns dict(out, selected, weights)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    router_w = np.ascontiguousarray(router_w, dtype=np.float32)
    nw = None if norm_w is None else np.ascontiguousarray(norm_w, dtype=np.float32)
    gi = None if sh_gate_inp is None else np.ascontiguousarray(sh_gate_inp, dtype=np.float32)
    T, H = x.shape
    E = router_w.shape[0]
    out = np.zeros((T, H), dtype=np.float32)
    sel = np.zeros((T, n_used), dtype=np.int32)
    w = np.zeros((T, n_used), dtype=np.float32)
    ref().qref_moe_layer_shexp(_p(x), H, T, _p(router_w), E, n_used, type_gu, _p(gate), _p(up), type_d, _p(down), F,
                               n_mat, _p(nw), norm_eps, _p(sh_gate), _p(sh_up), _p(sh_down), Fs, _p(gi), _p(out),
                               _p(sel), _p(w))
    return dict(out=out, selected=sel, weights=w)


def moe_layer(x, router_w, type_gu, gate, up, type_d, down, F, n_mat, n_used,
              g2s=None, mask=None, impl: str = "port", iters: int = 0, want_act=False,
              norm_w=None, norm_eps: float = 1e-6):
    """One build_moe layer.  x [T, H], router_w [E, H]; with norm_w the layer input is
    rms_norm(x) * norm_w (the ffn_norm).  Returns dict(out, selected, weights, act, ms)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    nw = None if norm_w is None else np.ascontiguousarray(norm_w, dtype=np.float32)
    if nw is not None and impl != "ref":
        x = rms_norm_mul(x, nw, norm_eps)
    router_w = np.ascontiguousarray(router_w, dtype=np.float32)
    T, H = x.shape
    E = router_w.shape[0]
    out = np.zeros((T, H), dtype=np.float32)
    sel = np.zeros((T, n_used), dtype=np.int32)
    w = np.zeros((T, n_used), dtype=np.float32)
    act = np.zeros((T, n_used, F), dtype=np.float32) if want_act else None
    g2 = None if g2s is None else np.ascontiguousarray(g2s, dtype=np.int32)
    m = None if mask is None else np.ascontiguousarray(mask, dtype=np.float32)
    ms = 0.0
    if impl == "ref":
        ms = ref().qref_moe_layer(_p(x), H, T, _p(router_w), E, n_used, type_gu, _p(gate), _p(up),
                                  type_d, _p(down), F, n_mat, _p(g2), _p(m), _p(out), _p(sel),
                                  _p(w), _p(act), iters, _p(nw), norm_eps)
    else:
        rc = port().qo_moe_layer(_p(x), H, T, _p(router_w), E, n_used, type_gu, _p(gate), _p(up),
                                 type_d, _p(down), F, n_mat, _p(g2), _p(m), _p(out), _p(sel),
                                 _p(w), _p(act))
        assert rc == 0, rc
    return dict(out=out, selected=sel, weights=w, act=act, ms=ms)


def set_ref_threads(n: int):
    ref().qref_set_threads(n)


def ref_last_times() -> np.ndarray:
    """ms of each timed evaluation of the last reference call that was given iters > 0."""
    n = ref().qref_last_times(None, 0)
    out = np.zeros(max(n, 1), dtype=np.float64)
    ref().qref_last_times(_p(out), n)
    return out[:n]


def nrmse(got: np.ndarray, want: np.ndarray) -> float:
    """Normalized RMS error: ||got - want||_2 / ||want||_2."""
    got = np.asarray(got, dtype=np.float64).ravel()
    want = np.asarray(want, dtype=np.float64).ravel()
    den = np.sqrt(np.mean(want * want))
    return float(np.sqrt(np.mean((got - want) ** 2)) / (den if den > 0 else 1.0))


def max_abs_rel(got: np.ndarray, want: np.ndarray) -> float:
    """max |got - want| / max |want|."""
    got = np.asarray(got, dtype=np.float64).ravel()
    want = np.asarray(want, dtype=np.float64).ravel()
    den = np.max(np.abs(want)) if want.size else 1.0
    return float(np.max(np.abs(got - want)) / (den if den > 0 else 1.0)) if want.size else 0.0


def fnv1a64(data: bytes | np.ndarray) -> int:
    """FNV-1a 64 of a byte string (core/expert_weight_audit.h:83-87), C restatement."""
    a = np.frombuffer(bytes(data), dtype=np.uint8) if not isinstance(data, np.ndarray) else np.ascontiguousarray(data, dtype=np.uint8)
    return int(port().qo_fnv1a64(_p(a) if a.size else None, a.size))


def slab_audit(expected: np.ndarray, actual: np.ndarray) -> dict:
    """The byte audit record of ExpertWeightAudit::compare (core/expert_weight_audit.h:
    106-125) for one slab, C restatement."""
    e = np.ascontiguousarray(expected, dtype=np.uint8)
    a = np.ascontiguousarray(actual, dtype=np.uint8)
    assert e.size == a.size
    eq, fd, eb, ab, fe, fa = (C.c_int32(), C.c_uint64(), C.c_uint32(), C.c_uint32(), C.c_uint64(), C.c_uint64())
    port().qo_slab_audit(_p(e), _p(a), e.size, C.byref(eq), C.byref(fd), C.byref(eb), C.byref(ab),
                         C.byref(fe), C.byref(fa))
    return {"equal": eq.value, "first_difference": fd.value, "expected_byte": eb.value,
            "actual_byte": ab.value, "expected_fnv1a64": fe.value, "actual_fnv1a64": fa.value}
