"""Generate tests/golden/slab_audit.json from the REFERENCE's own expert byte audit.

Run in a container where the reference sources are present and oracle/_ref/audit_harness
was built (``make -C oracle``):

    python tests/golden/make_audit_golden.py

For every case of tests/_data.py AUDIT_CASES (slab size, seed, bytes flipped in the
actual copy) the expected and actual bytes (tests/_data.py slab_bytes / audit_pair) are
written to files and handed to the reference's ExpertWeightAudit
(core/expert_weight_audit.h) through oracle/audit_harness.cpp; its log lines give the
fixture: equal flag, FNV-1a 64 of both byte strings, and for a mismatch the first
differing byte index and the two bytes there.  The tests compare the C restatement
(oracle/) and the GPU audit kernel against them; the reference is not needed at test
time.
"""
import json
import os
import re
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

import _data as D  # noqa: E402

HARNESS = os.path.join(ROOT, "oracle", "_ref", "audit_harness")
LINE = re.compile(r"expert-byte-audit selected-GPU .* bytes=(\d+) equal=(\d) "
                  r"expected_fnv1a64=([0-9a-f]{16}) actual_fnv1a64=([0-9a-f]{16})")
DIFF = re.compile(r"expert-byte-audit first_difference=(\d+) expected_byte=(\d+) actual_byte=(\d+)")


def run_case(size, seed, flips, tmp):
    exp, act = D.audit_pair(size, seed, flips)
    pe, pa = os.path.join(tmp, "expected.bin"), os.path.join(tmp, "actual.bin")
    exp.tofile(pe)
    act.tofile(pa)
    p = subprocess.run([HARNESS, pe, pa], capture_output=True, text=True)
    if p.returncode not in (0, 3):
        raise RuntimeError(f"audit harness failed: {p.stderr}")
    m = LINE.search(p.stderr)
    assert m and int(m.group(1)) == size, p.stderr
    rec = {"size": size, "seed": seed, "flips": [list(f) for f in flips], "equal": int(m.group(2)),
           "expected_fnv1a64": m.group(3), "actual_fnv1a64": m.group(4),
           "first_difference": size, "expected_byte": 0, "actual_byte": 0}
    d = DIFF.search(p.stderr)
    if d:
        rec["first_difference"], rec["expected_byte"], rec["actual_byte"] = (int(g) for g in d.groups())
    assert (p.returncode == 3) == (rec["equal"] == 0)
    return rec


def main():
    if not os.path.exists(HARNESS):
        raise SystemExit(f"{HARNESS} missing: run `make -C oracle` where the reference sources are present")
    with tempfile.TemporaryDirectory() as tmp:
        cases = [run_case(size, seed, flips, tmp) for size, seed, flips in D.AUDIT_CASES]
    out = os.path.join(HERE, "slab_audit.json")
    with open(out, "w") as f:
        json.dump({"source": "reference core/expert_weight_audit.h via oracle/audit_harness.cpp",
                   "cases": cases}, f, indent=1)
    print(f"wrote {out}: {len(cases)} cases")


if __name__ == "__main__":
    main()
