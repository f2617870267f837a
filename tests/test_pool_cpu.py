"""Expert pool writes and the byte audit, without a GPU: the C restatement of the audit
(oracle/) against the reference's own ExpertWeightAudit output (tests/golden/
slab_audit.json, from tests/golden/make_audit_golden.py) and the published FNV-1a 64
test vectors, and the host-side argument checks of qwb_pool_write_slabs /
qwb_pool_audit_slabs (which return before any CUDA call)."""
import ctypes as C
import json
import os

import pytest

import _data as D
import oracle as O
from questwend_b200 import _lib as L
from questwend_b200 import build as B

G = os.path.join(os.path.dirname(__file__), "golden", "slab_audit.json")


def golden_cases():
    with open(G) as f:
        return json.load(f)["cases"]


def test_fnv1a64_published_vectors():
    # test vectors of the FNV-1a 64 specification (Fowler / Noll / Vo)
    assert O.fnv1a64(b"") == 0xCBF29CE484222325
    assert O.fnv1a64(b"a") == 0xAF63DC4C8601EC8C
    assert O.fnv1a64(b"foobar") == 0x85944171F73967E8


def test_fixture_covers_the_cases():
    cases = golden_cases()
    assert [(c["size"], c["seed"], [tuple(f) for f in c["flips"]]) for c in cases] == \
        [(s, sd, list(fl)) for s, sd, fl in D.AUDIT_CASES]
    assert any(c["equal"] for c in cases) and any(not c["equal"] for c in cases)


@pytest.mark.parametrize("case", golden_cases(), ids=lambda c: f"{c['size']}-{c['seed']}")
def test_oracle_audit_matches_reference(case):
    exp, act = D.audit_pair(case["size"], case["seed"], case["flips"])
    got = O.slab_audit(exp, act)
    assert got["equal"] == case["equal"]
    assert got["first_difference"] == case["first_difference"]
    assert got["expected_byte"] == case["expected_byte"]
    assert got["actual_byte"] == case["actual_byte"]
    assert got["expected_fnv1a64"] == int(case["expected_fnv1a64"], 16)
    assert got["actual_fnv1a64"] == int(case["actual_fnv1a64"], 16)


@pytest.fixture(scope="module")
def lib():
    B.build()
    return L.lib()


def _pool(slots=4, slab=2304):
    d = L.Tensor()
    d.data, d.type = 0x100000, L.Q4_K
    ne = (512, 8, slots, 1)
    nb = (144, 288, slab, slab * slots)
    for i in range(4):
        d.ne[i], d.nb[i] = ne[i], nb[i]
    return d


def _copies(entries):
    arr = (L.SlabCopy * max(len(entries), 1))()
    for i, (src, slot) in enumerate(entries):
        arr[i].src, arr[i].slot = src, slot
    return arr


def test_pool_write_host_validation(lib):
    pool = _pool()
    ok = _copies([(0x2000, 0), (0x2000 + 2304, 1)])
    # slab size mismatch (pool vs source), the reference's fetch_slab check
    assert lib.qwb_pool_write_slabs(C.byref(pool), 2048, ok, 2, None) == 3
    # slot outside [0, n_slots) anywhere in the group: nothing is written
    assert lib.qwb_pool_write_slabs(C.byref(pool), 2304, _copies([(0x2000, 0), (0x3000, 4)]), 2, None) == 1
    assert lib.qwb_pool_write_slabs(C.byref(pool), 2304, _copies([(0x2000, -1)]), 1, None) == 1
    # null source, negative count, missing pool
    assert lib.qwb_pool_write_slabs(C.byref(pool), 2304, _copies([(None, 0)]), 1, None) == 1
    assert lib.qwb_pool_write_slabs(C.byref(pool), 2304, ok, -1, None) == 1
    assert lib.qwb_pool_write_slabs(None, 2304, ok, 2, None) == 1
    # nothing to copy
    assert lib.qwb_pool_write_slabs(C.byref(pool), 2304, None, 0, None) == 0


def test_pool_audit_host_validation(lib):
    pool = _pool()
    assert lib.qwb_pool_audit_slabs(C.byref(pool), _copies([(0x2000, 4)]), 1, 1, 0x5000, None) == 1
    assert lib.qwb_pool_audit_slabs(C.byref(pool), _copies([(0x2000, 0)]), 1, 1, None, None) == 1
    assert lib.qwb_pool_audit_slabs(C.byref(pool), _copies([(None, 0)]), 1, 1, 0x5000, None) == 1
    assert lib.qwb_pool_audit_slabs(C.byref(pool), None, 0, 1, None, None) == 0
    assert C.sizeof(L.SlabAudit) == 40 and C.sizeof(L.SlabCopy) == 16
