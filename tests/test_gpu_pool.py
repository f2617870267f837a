"""Expert pool writes (qwb_pool_write_slabs) and the device byte audit
(qwb_pool_audit_slabs) on the GPU, through the C ABI: slot bytes after the writes are
bit-exact copies of their sources, and the audit records equal the reference's own
ExpertWeightAudit output (tests/golden/slab_audit.json) and the C restatement."""
import ctypes as C
import json
import os

import numpy as np
import pytest
import torch

import _data as D
import oracle as O
from questwend_b200 import _lib as L

pytestmark = pytest.mark.gpu
G = os.path.join(os.path.dirname(__file__), "golden", "slab_audit.json")


def _pool_desc(buf: torch.Tensor, slab: int, n_slots: int) -> L.Tensor:
    d = L.Tensor()
    d.data, d.type = buf.data_ptr(), L.I32
    ne = (slab, 1, n_slots, 1)
    nb = (1, slab, slab, slab * n_slots)
    for i in range(4):
        d.ne[i], d.nb[i] = ne[i], nb[i]
    return d


def _copies(entries):
    arr = (L.SlabCopy * max(len(entries), 1))()
    for i, (src, slot) in enumerate(entries):
        arr[i].src, arr[i].slot = src, slot
    return arr


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _audit(pool_desc, entries, checksums=1):
    n = len(entries)
    res = torch.zeros((n, C.sizeof(L.SlabAudit)), dtype=torch.uint8, device="cuda")
    rc = L.lib().qwb_pool_audit_slabs(C.byref(pool_desc), _copies(entries), n, checksums, res.data_ptr(),
                                      _stream())
    assert rc == 0, L.STATUS.get(rc, rc)
    host = res.cpu().numpy()
    out = []
    for i in range(n):
        r = L.SlabAudit.from_buffer_copy(host[i].tobytes())
        out.append({k: int(getattr(r, k)) for k, _ in L.SlabAudit._fields_ if k != "reserved"})
    return out


def _pinned(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(a).pin_memory()


def test_pool_write_round_trip():
    slab, n_slots = 884736, 6  # one C1 Q4_K expert matrix per slot
    pool = torch.zeros(slab * n_slots, dtype=torch.uint8, device="cuda")
    d = _pool_desc(pool, slab, n_slots)
    # a page-locked staging buffer of four slabs (as fetch_parallel stages a group),
    # one device-resident slab, and slot 0 named twice (the later source wins)
    stage = _pinned(np.concatenate([D.slab_bytes(slab, 20 + i) for i in range(4)]))
    dev_src = torch.from_numpy(D.slab_bytes(slab, 30)).cuda()
    first0 = _pinned(D.slab_bytes(slab, 31))
    base = stage.data_ptr()
    entries = [(first0.data_ptr(), 0), (base, 2), (base + slab, 3), (base + 2 * slab, 0),
               (base + 3 * slab, 5), (dev_src.data_ptr(), 1)]
    rc = L.lib().qwb_pool_write_slabs(C.byref(d), slab, _copies(entries), len(entries), _stream())
    assert rc == 0
    got = pool.view(n_slots, slab).cpu().numpy()
    want = {0: D.slab_bytes(slab, 22), 1: D.slab_bytes(slab, 30), 2: D.slab_bytes(slab, 20),
            3: D.slab_bytes(slab, 21), 5: D.slab_bytes(slab, 23)}
    for s, w in want.items():
        assert np.array_equal(got[s], w), s
    assert not got[4].any()  # untouched slot
    # an out-of-range slot anywhere in the group: error, nothing written
    before = pool.clone()
    bad = _copies([(base, 4), (base, 6)])
    assert L.lib().qwb_pool_write_slabs(C.byref(d), slab, bad, 2, _stream()) == 1
    torch.cuda.synchronize()
    assert torch.equal(pool, before)
    # slab size mismatch (pool vs source)
    assert L.lib().qwb_pool_write_slabs(C.byref(d), slab - 1, _copies([(base, 4)]), 1, _stream()) == 3


def test_pool_write_copy_engine_fallback():
    # sources the gather kernel cannot read (pageable host memory) or not 16-byte aligned
    # go through one copy per slab; slots named twice still end with the later source
    slab, n_slots = 65552, 5  # 64 KB + 16: the last chunk is partial
    pool = torch.zeros(slab * n_slots, dtype=torch.uint8, device="cuda")
    d = _pool_desc(pool, slab, n_slots)
    pageable = [D.slab_bytes(slab, 40 + i) for i in range(3)]
    entries = [(pageable[0].ctypes.data, 3), (pageable[1].ctypes.data, 0), (pageable[2].ctypes.data, 3)]
    assert L.lib().qwb_pool_write_slabs(C.byref(d), slab, _copies(entries), 3, _stream()) == 0
    # page-locked but misaligned by one byte
    raw = _pinned(np.concatenate([np.zeros(1, np.uint8), D.slab_bytes(slab, 50), D.slab_bytes(slab, 51)]))
    mis = [(raw.data_ptr() + 1, 1), (raw.data_ptr() + 1 + slab, 4)]
    assert L.lib().qwb_pool_write_slabs(C.byref(d), slab, _copies(mis), 2, _stream()) == 0
    got = pool.view(n_slots, slab).cpu().numpy()
    assert np.array_equal(got[3], pageable[2]) and np.array_equal(got[0], pageable[1])
    assert np.array_equal(got[1], D.slab_bytes(slab, 50)) and np.array_equal(got[4], D.slab_bytes(slab, 51))
    assert not got[2].any()


def test_pool_write_slot_to_slot_in_array_order():
    # sources inside the pool: copies run in array order, so slot 2 receives slot 0's bytes
    # from before entry 1 overwrote slot 0
    slab, n_slots = 4096, 4
    init = np.concatenate([D.slab_bytes(slab, 60 + i) for i in range(n_slots)])
    pool = torch.from_numpy(init).cuda()
    d = _pool_desc(pool, slab, n_slots)
    new0 = torch.from_numpy(D.slab_bytes(slab, 70)).cuda()
    entries = [(pool.data_ptr(), 2), (new0.data_ptr(), 0), (pool.data_ptr() + 3 * slab, 1)]
    assert L.lib().qwb_pool_write_slabs(C.byref(d), slab, _copies(entries), 3, _stream()) == 0
    got = pool.view(n_slots, slab).cpu().numpy()
    assert np.array_equal(got[2], D.slab_bytes(slab, 60))
    assert np.array_equal(got[0], D.slab_bytes(slab, 70))
    assert np.array_equal(got[1], D.slab_bytes(slab, 63))
    assert np.array_equal(got[3], D.slab_bytes(slab, 63))


def test_pool_write_gather_partial_chunks_and_duplicates():
    # the gather kernel: slab sizes that end inside a 64 KB chunk and inside a 4-load
    # group, many slots (more than one launch's table of 128), duplicates keep the last
    slab, n_slots = 16 * 1000 + 16, 300
    pool = torch.zeros(slab * n_slots, dtype=torch.uint8, device="cuda")
    d = _pool_desc(pool, slab, n_slots)
    src = torch.from_numpy(np.concatenate([D.slab_bytes(slab, 200 + i) for i in range(260)])).cuda()
    rng = np.random.default_rng(3)
    slots = rng.choice(n_slots, 250, replace=False).tolist() + [7, 7, 11]
    srcs = list(range(250)) + [250, 251, 252]
    slots[5] = 11  # slot 11 named earlier too: the last entry (source 252) wins
    entries = [(src.data_ptr() + i * slab, sl) for i, sl in zip(srcs, slots)]
    assert L.lib().qwb_pool_write_slabs(C.byref(d), slab, _copies(entries), len(entries), _stream()) == 0
    got = pool.view(n_slots, slab).cpu().numpy()
    final = {}
    for i, sl in zip(srcs, slots):
        final[sl] = i
    for sl, i in final.items():
        assert np.array_equal(got[sl], D.slab_bytes(slab, 200 + i)), (sl, i)
    untouched = [sl for sl in range(n_slots) if sl not in final]
    assert not got[untouched].any()


def _golden():
    with open(G) as f:
        return json.load(f)["cases"]


@pytest.mark.parametrize("where", ["device", "pinned"])
def test_pool_audit_matches_reference(where):
    for case in _golden():
        size = case["size"]
        exp, act = D.audit_pair(size, case["seed"], case["flips"])
        pool = torch.zeros(2 * size, dtype=torch.uint8, device="cuda")
        d = _pool_desc(pool, size, 2)
        # slot 0 <- the actual bytes, slot 1 <- the expected bytes, written from host memory
        pa, pe = _pinned(act), _pinned(exp)
        assert L.lib().qwb_pool_write_slabs(C.byref(d), size, _copies([(pa.data_ptr(), 0), (pe.data_ptr(), 1)]),
                                            2, _stream()) == 0
        src = torch.from_numpy(exp).cuda() if where == "device" else pe
        r_act, r_exp = _audit(d, [(src.data_ptr(), 0), (src.data_ptr(), 1)])
        want = {"equal": case["equal"], "first_difference": case["first_difference"],
                "expected_byte": case["expected_byte"], "actual_byte": case["actual_byte"],
                "expected_fnv1a64": int(case["expected_fnv1a64"], 16),
                "actual_fnv1a64": int(case["actual_fnv1a64"], 16)}
        assert r_act == want, (size, case["seed"])
        fe = int(case["expected_fnv1a64"], 16)
        assert r_exp == {"equal": 1, "first_difference": size, "expected_byte": 0, "actual_byte": 0,
                         "expected_fnv1a64": fe, "actual_fnv1a64": fe}
        # compare only: the same record without the checksums
        c_act, c_exp = _audit(d, [(src.data_ptr(), 0), (src.data_ptr(), 1)], checksums=0)
        assert c_act == dict(want, expected_fnv1a64=0, actual_fnv1a64=0)
        assert c_exp == {"equal": 1, "first_difference": size, "expected_byte": 0, "actual_byte": 0,
                         "expected_fnv1a64": 0, "actual_fnv1a64": 0}


def test_pool_audit_many_slots_against_oracle():
    # more slots than one launch's pointer table (128): two launches
    slab, n = 4096, 200
    rng = np.random.default_rng(5)
    exp = np.stack([D.slab_bytes(slab, 100 + i) for i in range(n)])
    act = exp.copy()
    bad = rng.choice(n, 17, replace=False)
    for s in bad:
        act[s, rng.integers(slab)] ^= np.uint8(rng.integers(1, 256))
    pool = torch.from_numpy(act.reshape(-1)).cuda()
    d = _pool_desc(pool, slab, n)
    e = torch.from_numpy(exp).cuda()
    got = _audit(d, [(e[i].data_ptr(), i) for i in range(n)])
    for i in range(n):
        assert got[i] == O.slab_audit(exp[i], act[i]), i
    assert sum(1 - g["equal"] for g in got) == len(bad)


def test_pool_audit_rejects_pageable_memory():
    slab = 4096
    pool = torch.zeros(slab, dtype=torch.uint8, device="cuda")
    d = _pool_desc(pool, slab, 1)
    pageable = np.zeros(slab, np.uint8)
    res = torch.zeros((1, C.sizeof(L.SlabAudit)), dtype=torch.uint8, device="cuda")
    rc = L.lib().qwb_pool_audit_slabs(C.byref(d), _copies([(pageable.ctypes.data, 0)]), 1, 1, res.data_ptr(),
                                      _stream())
    assert rc == 1
    assert not res.any()
