"""Host-side mirror of the ggml operators this library implements on B200.

Each function mirrors a ggml graph op (same argument meaning, ggml's dimension order
expressed as torch shapes, same result) and calls the C ABI of libqwb.so on the
current CUDA stream with device tensors:

    get_rows(src, idx)                 GGML_OP_GET_ROWS        (ggml.c:3975)
    mul_mat_id(as_, b, ids)            GGML_OP_MUL_MAT_ID      (ggml.c:3413)
    quantize_q8_K / quantize_q8_0      the CPU backend's from_float for src1
    moe_route(logits, k)               route_experts subgraph  (core/runtime.cpp:2693)
    swiglu(gate, up)                   ggml_swiglu_split       (ggml.c:3082)
    moe_weighted_sum(experts, w)       weighted reduce         (core/runtime.cpp:2796)
    moe_ffn(...)                       build_moe               (core/runtime.cpp:2743)

Torch shapes are ggml's ne reversed: a ggml tensor [ne0, ne1, ne2] is a torch tensor of
shape (ne2, ne1, ne0).  Quantized tensors are ``QTensor`` (raw ggml block bytes in a
uint8 device buffer plus the ggml type and ne).  Data-dependent errors (ids out of
range) are recorded in a device status block; ``read_status()`` returns and clears it.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib as L
from ._lib import F16, F32, I32, Q4_K, Q6_K, Q8_0, Q8_K, Q8_0_CPU, Q8_0_REF  # noqa: F401

_BLOCK = {F32: (1, 4), F16: (1, 2), I32: (1, 4), Q8_0: (32, 34), Q4_K: (256, 144),
          Q6_K: (256, 210), Q8_K: (256, 292)}


def row_size(t: int, n: int) -> int:
    blk, nb = _BLOCK[t]
    if n % blk:
        raise ValueError(f"row of {n} not a multiple of the block size {blk}")
    return n // blk * nb


@dataclass
class QTensor:
    """A ggml tensor of block-quantized rows in device memory (contiguous)."""
    data: torch.Tensor  # uint8, cuda
    type: int
    ne: tuple  # (ne0, ne1, ne2, ne3)

    @staticmethod
    def from_bytes(raw, t: int, ne, device="cuda") -> "QTensor":
        ne = tuple(ne) + (1,) * (4 - len(ne))
        if isinstance(raw, torch.Tensor):
            src = raw.to(device=device, dtype=torch.uint8).reshape(-1)
        else:
            src = torch.from_numpy(raw.reshape(-1).view("uint8")).to(device)
        need = row_size(t, ne[0]) * ne[1] * ne[2] * ne[3]
        if src.numel() != need:
            raise ValueError(f"{src.numel()} bytes for a {ne} tensor of type {t} (need {need})")
        # the kernels read weight spans widened to 16-byte boundaries: keep 16 readable
        # bytes after the last row, as ggml's padded backend buffers do
        buf = torch.zeros(need + 16, dtype=torch.uint8, device=device)
        buf[:need].copy_(src)
        return QTensor(buf[:need], t, ne)

    @property
    def nb(self):
        rs = row_size(self.type, self.ne[0])
        return (_BLOCK[self.type][1], rs, rs * self.ne[1], rs * self.ne[1] * self.ne[2])

    def desc(self) -> L.Tensor:
        d = L.Tensor()
        d.data = self.data.data_ptr()
        d.type = self.type
        for i in range(4):
            d.ne[i] = self.ne[i]
            d.nb[i] = self.nb[i]
        return d


_DT = {torch.float32: F32, torch.float16: F16, torch.int32: I32}


def desc(t) -> L.Tensor:
    """qwb_tensor describing a torch tensor (ggml order: ne0 = last torch dim)."""
    if isinstance(t, QTensor):
        return t.desc()
    if t.dim() > 4:
        raise ValueError("at most 4 dims")
    d = L.Tensor()
    d.data = t.data_ptr()
    d.type = _DT[t.dtype]
    shape = list(reversed(t.shape)) + [1] * (4 - t.dim())
    strides = list(reversed(t.stride())) + [0] * (4 - t.dim())
    es = t.element_size()
    for i in range(4):
        d.ne[i] = shape[i]
        d.nb[i] = strides[i] * es if i < t.dim() else (d.nb[i - 1] * d.ne[i - 1] if i else es)
    return d


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


_ws = {}
_status = {}


def workspace(nbytes: int, device=None) -> torch.Tensor:
    """Per-device scratch buffer, grown on demand; its first 256 bytes (the control
    block the fused kernels keep at zero between calls) are zeroed on allocation."""
    dev = torch.device(device or torch.cuda.current_device())
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    buf = _ws.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(nbytes, 1 << 20) + 256, dtype=torch.uint8, device=f"cuda:{key}")
        _ws[key] = buf
    return buf


def status_block(device=None) -> torch.Tensor:
    key = torch.cuda.current_device() if device is None else torch.device(device).index
    sb = _status.get(key)
    if sb is None:
        sb = torch.zeros(4, dtype=torch.int32, device=f"cuda:{key}")
        _status[key] = sb
    return sb


def read_status(reset: bool = True, device=None):
    """(flags, first bad value, count) of the device status block; clears it."""
    sb = status_block(device)
    out = L.StatusBlock()
    L.check("qwb_status_block_read", L.lib().qwb_status_block_read(sb.data_ptr(), C.byref(out), int(reset), _stream()))
    return out.flags, out.bad_value, out.count


def _ws_ptr(ws: torch.Tensor) -> int:
    p = ws.data_ptr()
    assert p % 256 == 0
    return p


# ------------------------------------------------------------------ quantizers
def quantize_q8_K(x: torch.Tensor) -> torch.Tensor:
    """Rows of x [..., K] f32 -> packed block_q8_K bytes [..., K/256*292]."""
    K = x.shape[-1]
    x2 = x.reshape(-1, K)
    y = torch.empty((x2.shape[0], row_size(Q8_K, K)), dtype=torch.uint8, device=x.device)
    L.check("qwb_quantize_row_q8_K", L.lib().qwb_quantize_row_q8_K(
        x2.data_ptr(), y.data_ptr(), x2.shape[0], K, x2.stride(0), _stream()))
    return y.reshape(*x.shape[:-1], -1)


def quantize_q8_0(x: torch.Tensor, variant: int = Q8_0_CPU) -> torch.Tensor:
    K = x.shape[-1]
    x2 = x.reshape(-1, K)
    y = torch.empty((x2.shape[0], row_size(Q8_0, K)), dtype=torch.uint8, device=x.device)
    L.check("qwb_quantize_row_q8_0", L.lib().qwb_quantize_row_q8_0(
        x2.data_ptr(), y.data_ptr(), x2.shape[0], K, x2.stride(0), variant, _stream()))
    return y.reshape(*x.shape[:-1], -1)


# ------------------------------------------------------------------ GET_ROWS
def get_rows(src, idx: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """ggml_get_rows(src [ne0, ne01, ne02, ne03], idx [n, ne02, ne03]) -> [ne0, n, ne02, ne03]."""
    sd = desc(src)
    idx_d = desc(idx)
    ne0 = sd.ne[0]
    shape = (idx_d.ne[2], idx_d.ne[1], idx_d.ne[0], ne0)
    odt = torch.int32 if sd.type == I32 else torch.float32
    if out is None:
        out = torch.empty(shape, dtype=odt, device=idx.device)
    od = desc(out.reshape(shape))
    L.check("qwb_get_rows", L.lib().qwb_get_rows(C.byref(sd), C.byref(idx_d), C.byref(od),
                                                 status_block().data_ptr(), _stream()))
    return out


# ------------------------------------------------------------------ MUL_MAT_ID
def mul_mat_id(as_: QTensor, b: torch.Tensor, ids: torch.Tensor, out: torch.Tensor | None = None):
    """ggml_mul_mat_id(as [K, M, n_as], b [K, n_b, T], ids [n_used, T]) -> [M, n_used, T].

    Torch shapes: b (T, n_b, K) f32, ids (T, n_used) int32 (may be a column slice),
    result (T, n_used, M) f32."""
    ad, bd, idd = desc(as_), desc(b), desc(ids)
    T, n_used, M = ids.shape[0], ids.shape[1], as_.ne[1]
    if out is None:
        out = torch.empty((T, n_used, M), dtype=torch.float32, device=b.device)
    od = desc(out)
    lib = L.lib()
    need = lib.qwb_mul_mat_id_workspace_size(C.byref(ad), C.byref(bd), C.byref(idd))
    if need == 0 and T * n_used > 0:
        raise L.QwbError("qwb_mul_mat_id_workspace_size", 3)
    ws = workspace(need)
    L.check("qwb_mul_mat_id", lib.qwb_mul_mat_id(C.byref(ad), C.byref(bd), C.byref(idd), C.byref(od),
                                                 _ws_ptr(ws), ws.numel(), status_block().data_ptr(), _stream()))
    return out


# ------------------------------------------------------------------ MUL_MAT
def mul_mat(a: QTensor, b: torch.Tensor, out: torch.Tensor | None = None):
    """ggml_mul_mat(a [K, M] quantized, b [K, T] f32) -> [M, T] (dense FFN / shared expert /
    output head).  Torch shapes: b (T, K) f32, result (T, M) f32."""
    T, M = b.shape[0], a.ne[1]
    if out is None:
        out = torch.empty((T, M), dtype=torch.float32, device=b.device)
    ad, bd, od = desc(a), desc(b), desc(out)
    lib = L.lib()
    need = lib.qwb_mul_mat_workspace_size(C.byref(ad), C.byref(bd))
    if need == 0 and T > 0:
        raise L.QwbError("qwb_mul_mat_workspace_size", 3)
    ws = workspace(need)
    L.check("qwb_mul_mat", lib.qwb_mul_mat(C.byref(ad), C.byref(bd), C.byref(od), _ws_ptr(ws), ws.numel(),
                                           status_block().data_ptr(), _stream()))
    return out


# ------------------------------------------------------------------ small MoE ops
def moe_route(logits: torch.Tensor, n_used: int, norm: bool = True, scale: float = 0.0,
              mask: torch.Tensor | None = None):
    T, E = logits.shape
    sel = torch.empty((T, n_used), dtype=torch.int32, device=logits.device)
    w = torch.empty((T, n_used), dtype=torch.float32, device=logits.device)
    L.check("qwb_moe_route", L.lib().qwb_moe_route(
        logits.data_ptr(), mask.data_ptr() if mask is not None else None, E, T, n_used, int(norm), scale,
        sel.data_ptr(), w.data_ptr(), _stream()))
    return sel, w


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    out = torch.empty_like(gate)
    L.check("qwb_swiglu", L.lib().qwb_swiglu(gate.data_ptr(), up.data_ptr(), out.data_ptr(), gate.numel(),
                                             _stream()))
    return out


def moe_weighted_sum(experts: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
    """experts (T, n_used, H), weights (T, n_used) -> (T, H)."""
    T, n_used, H = experts.shape
    out = torch.empty((T, H), dtype=torch.float32, device=experts.device)
    L.check("qwb_moe_weighted_sum", L.lib().qwb_moe_weighted_sum(
        experts.data_ptr(), weights.data_ptr(), out.data_ptr(), H, n_used, T, _stream()))
    return out


def _set_shexp(d, shexp):
    """shexp: None or (gate QTensor [H, F_sh], up QTensor, down QTensor [F_sh, H], gate_inp (H,) f32 or None)."""
    if shexp is None:
        return
    g, u, dn, gi = shexp
    d.shexp_gate, d.shexp_up, d.shexp_down = g.desc(), u.desc(), dn.desc()
    d.shexp_gate_inp = gi.data_ptr() if gi is not None else None


def moe_ffn_desc(x, router_w, gate: QTensor, up: QTensor, down: QTensor, n_used: int, out,
                 g2s=None, mask=None, residual=None, selected=None, weights=None, act=None,
                 norm_w=None, norm_eps: float = 1e-6, shexp=None) -> L.MoeFfnDesc:
    T, H = x.shape
    d = L.MoeFfnDesc()
    d.x = x.data_ptr()
    d.router_w = router_w.data_ptr()
    d.mask = mask.data_ptr() if mask is not None else None
    d.g2s = g2s.data_ptr() if g2s is not None else None
    d.gate, d.up, d.down = gate.desc(), up.desc(), down.desc()
    d.H, d.F, d.E, d.n_used, d.T = H, gate.ne[1], router_w.shape[0], n_used, T
    d.residual = residual.data_ptr() if residual is not None else None
    d.out = out.data_ptr()
    d.selected = selected.data_ptr() if selected is not None else None
    d.weights = weights.data_ptr() if weights is not None else None
    d.act = act.data_ptr() if act is not None else None
    d.norm_w = norm_w.data_ptr() if norm_w is not None else None
    d.norm_eps = norm_eps
    _set_shexp(d, shexp)
    return d


def moe_ffn(x, router_w, gate: QTensor, up: QTensor, down: QTensor, n_used: int,
            g2s=None, mask=None, residual=None, out=None, act=None, norm_w=None, norm_eps: float = 1e-6,
            shexp=None):
    """One MoE FFN layer (build_moe).  x (T, H) f32, router_w (E, H) f32, gate/up ggml
    [H, F, n_mat], down [F, H, n_mat]; g2s (3, E) int32 expert->slot tables (gate, up,
    down) or None; act: optional (T, n_used, F) f32 tensor receiving swiglu(gate, up);
    norm_w: optional ffn_norm weight (H,): the layer then runs on rms_norm(x) * norm_w;
    shexp: optional shared expert (gate [H, F_sh], up, down [F_sh, H] QTensors, gate_inp
    (H,) f32 or None), added to the routed experts' sum (core/runtime.cpp:2825-2833).
    Returns (out (T, H), selected (T, n_used), weights (T, n_used))."""
    T, H = x.shape
    if out is None:
        out = torch.empty((T, H), dtype=torch.float32, device=x.device)
    sel = torch.empty((T, n_used), dtype=torch.int32, device=x.device)
    w = torch.empty((T, n_used), dtype=torch.float32, device=x.device)
    d = moe_ffn_desc(x, router_w, gate, up, down, n_used, out, g2s, mask, residual, sel, w, act, norm_w, norm_eps,
                     shexp)
    lib = L.lib()
    need = lib.qwb_moe_ffn_workspace_size(C.byref(d))
    if need == 0:
        raise L.QwbError("qwb_moe_ffn_workspace_size", 3)
    ws = workspace(need)
    L.check("qwb_moe_ffn", lib.qwb_moe_ffn(C.byref(d), _ws_ptr(ws), ws.numel(), status_block().data_ptr(),
                                           _stream()))
    return out, sel, w


# ------------------------------------------------------------------ expert parallelism
def moe_ep_layer_desc(x, router_w, gate: QTensor, up: QTensor, down: QTensor, expert_lo: int, n_used: int, out,
                      residual=None, selected=None, weights=None, norm_w=None, norm_eps: float = 1e-6,
                      mask=None, shexp=None) -> L.MoeEpLayerDesc:
    T, H = x.shape
    d = L.MoeEpLayerDesc()
    d.x, d.router_w = x.data_ptr(), router_w.data_ptr()
    d.norm_w = norm_w.data_ptr() if norm_w is not None else None
    d.norm_eps = norm_eps
    d.mask = mask.data_ptr() if mask is not None else None
    d.gate, d.up, d.down = gate.desc(), up.desc(), down.desc()
    d.expert_lo = expert_lo
    d.H, d.F, d.E, d.n_used, d.T = H, gate.ne[1], router_w.shape[0], n_used, T
    d.residual = residual.data_ptr() if residual is not None else None
    d.out = out.data_ptr()
    d.selected = selected.data_ptr() if selected is not None else None
    d.weights = weights.data_ptr() if weights is not None else None
    _set_shexp(d, shexp)
    return d


def moe_ep_layer(x, router_w, gate: QTensor, up: QTensor, down: QTensor, expert_lo: int, n_used: int,
                 residual=None, norm_w=None, norm_eps: float = 1e-6, mask=None, out=None, shexp=None):
    """One GPU's share of an expert-parallel MoE layer.  x (T, H) f32: all tokens' rows (the
    same on every GPU); gate/up [H, F, n_local], down [F, H, n_local]: global experts
    [expert_lo, expert_lo + n_local).  Routes all tokens (replicated router) and returns
    (out (T, H), selected (T, n_used), weights (T, n_used)): out[t] = the weighted sum of
    this GPU's experts' outputs for token t (+ the shared expert `shexp`, as in moe_ffn,
    when given) (+ residual[t] when given).  Summing out over the GPUs (all-reduce) gives
    the layer's output: pass residual and shexp to one GPU only."""
    T, H = x.shape
    if out is None:
        out = torch.empty((T, H), dtype=torch.float32, device=x.device)
    sel = torch.empty((T, n_used), dtype=torch.int32, device=x.device)
    w = torch.empty((T, n_used), dtype=torch.float32, device=x.device)
    d = moe_ep_layer_desc(x, router_w, gate, up, down, expert_lo, n_used, out, residual, sel, w, norm_w, norm_eps,
                          mask, shexp)
    lib = L.lib()
    need = lib.qwb_moe_ep_layer_workspace_size(C.byref(d))
    if need == 0:
        raise L.QwbError("qwb_moe_ep_layer_workspace_size", 3)
    ws = workspace(need)
    L.check("qwb_moe_ep_layer", lib.qwb_moe_ep_layer(C.byref(d), _ws_ptr(ws), ws.numel(), status_block().data_ptr(),
                                                     _stream()))
    return out, sel, w


# ------------------------------------------------------------------ expert pool writes
def _slab_ptr(x) -> int:
    if isinstance(x, torch.Tensor):
        if not x.is_contiguous():
            raise ValueError("slab sources must be contiguous")
        return x.data_ptr()
    return int(x)


def _slab_copies(srcs, slots):
    if len(srcs) != len(slots):
        raise ValueError("one slot per slab")
    arr = (L.SlabCopy * max(len(srcs), 1))()
    for i, (src, slot) in enumerate(zip(srcs, slots)):
        arr[i].src = _slab_ptr(src)
        arr[i].slot = int(slot)
    return arr


def pool_write_slabs(pool: QTensor, srcs, slots, src_slab_bytes: int | None = None):
    """Copy expert slabs into pool slots on the current stream, like the expert cache's
    ``ggml_backend_tensor_set_async(pool, src, slot * nb2, nb2)`` per (role, expert)
    (core/expert_cache.cpp:637-723, :1357-1377).  ``srcs``: tensors (page-locked host
    memory for asynchronous copies, or device memory) or raw pointers of one slab each;
    ``slots``: their slots in ``pool`` (a [ne0, ne1, n_slots] QTensor)."""
    nb2 = pool.nb[2]
    for x in srcs:
        if isinstance(x, torch.Tensor) and x.numel() * x.element_size() != nb2:
            raise ValueError(f"slab of {x.numel() * x.element_size()} bytes, pool slot holds {nb2}")
    arr = _slab_copies(srcs, slots)
    d = pool.desc()
    L.check("qwb_pool_write_slabs", L.lib().qwb_pool_write_slabs(
        C.byref(d), nb2 if src_slab_bytes is None else src_slab_bytes, arr, len(srcs), _stream()))


def pool_audit_slabs(pool: QTensor, expected, slots, checksums: bool = True):
    """Byte audit of pool slots on the GPU (core/expert_weight_audit.h:56-66, :106-125):
    one record per slot (equal, first_difference, expected_byte, actual_byte,
    expected_fnv1a64, actual_fnv1a64) as a list of dicts.  ``expected``: the bytes each
    slot should hold, in device or page-locked host memory.  ``checksums=False`` skips the
    serial FNV-1a chains (both sums read 0) and only compares."""
    n = len(expected)
    res = torch.zeros((max(n, 1), C.sizeof(L.SlabAudit)), dtype=torch.uint8, device=pool.data.device)
    arr = _slab_copies(expected, slots)
    d = pool.desc()
    L.check("qwb_pool_audit_slabs", L.lib().qwb_pool_audit_slabs(C.byref(d), arr, n, int(checksums), res.data_ptr(),
                                                                 _stream()))
    host = res.cpu().numpy()
    out = []
    for i in range(n):
        r = L.SlabAudit.from_buffer_copy(host[i].tobytes())
        out.append({k: int(getattr(r, k)) for k, _ in L.SlabAudit._fields_ if k != "reserved"})
    return out
