// audit_harness.cpp - runs the reference's own expert byte audit (ExpertWeightAudit,
// core/expert_weight_audit.h, header-only, compiled from the reference sources by
// oracle/Makefile into _ref/audit_harness) on one (expected, actual) pair of files.
// TEST INFRASTRUCTURE ONLY: tests/golden/make_audit_golden.py runs it to record the
// reference's audit lines (equal flag, first difference, FNV-1a 64 checksums) as
// fixtures.
//
// usage: audit_harness <expected file> <actual file>
// The audit's GPU-destination path (:62-66) is driven with a readback callback that
// returns the actual file's bytes; the reference compares them with the expected file
// (its "authoritative GGUF" span at offset 0) and logs to stderr.  Exit 0 when the
// reference accepted the bytes, 3 when it raised its mismatch error, 1 on usage errors.
#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <vector>

#include "expert_weight_audit.h"

int main(int argc, char **argv) {
    if (argc != 3) {
        std::fprintf(stderr, "usage: %s <expected file> <actual file>\n", argv[0]);
        return 1;
    }
    std::FILE *f = std::fopen(argv[2], "rb");
    if (!f) return 1;
    std::vector<unsigned char> actual;
    unsigned char buf[1 << 16];
    size_t got;
    while ((got = std::fread(buf, 1, sizeof(buf), f)) > 0) actual.insert(actual.end(), buf, buf + got);
    std::fclose(f);
    try {
        questwend::ExpertWeightAudit audit(0, 0, 1, true);
        if (!audit.begin(0, 1, 1)) return 1;
        audit.destination(argv[1], 0, actual.size(), 0, 0, 0, [&](void *dst, size_t n) {
            std::memcpy(dst, actual.data(), n);
        });
        audit.end();
    } catch (const std::runtime_error &e) {
        std::fprintf(stderr, "audit-harness error: %s\n", e.what());
        return 3;
    }
    return 0;
}
