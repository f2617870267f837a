"""Seeded synthetic inputs shared by the tests (weights N(0, 0.02) quantized with the
reference quantizer restatement, activations N(0, 1)), as the reference's benchmarks
specify.  numpy's PCG64 stream is stable across platforms and numpy versions."""
import hashlib

import numpy as np

import oracle as O


def rng(seed):
    return np.random.default_rng(seed)


def weights(t, n_mat, rows, K, seed, scale=0.02):
    """ggml tensor [K, rows, n_mat] of type t: n_mat*rows quantized rows of K."""
    x = (rng(seed).standard_normal((n_mat * rows, K), dtype=np.float32) * scale).astype(np.float32)
    return O.quantize_weights(t, x)


def acts(shape, seed):
    return rng(seed).standard_normal(shape, dtype=np.float32)


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).view(np.uint8).tobytes()).hexdigest()[:16]


def zipf_ids(T, E, n_used, seed, s=1.1):
    """Skewed routing: logits = log Zipf(s) popularity (expert ranks in seeded random
    order) + Gumbel noise, top-n_used per token -> int32 [T, n_used]."""
    r = rng(seed)
    pop = 1.0 / np.arange(1, E + 1, dtype=np.float64) ** s
    logits = np.log(pop[r.permutation(E)])[None, :] + r.gumbel(size=(T, E))
    return np.argsort(-logits, axis=1, kind="stable")[:, :n_used].astype(np.int32)


def slab_bytes(size: int, seed: int) -> np.ndarray:
    """Deterministic pseudo-random slab bytes (splitmix64 of the byte index), defined by
    this formula rather than by a library generator so fixtures never depend on numpy's
    stream versions."""
    with np.errstate(over="ignore"):
        z = np.arange(size, dtype=np.uint64) + np.uint64(seed) * np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    return (z & np.uint64(0xFF)).astype(np.uint8)


# Byte-audit cases: (slab bytes, seed, [(position, xor mask), ...] planted in the actual
# bytes).  Sizes cover one partial chunk, exact multiples and non-multiples of the
# device's 8 KB staging chunk and of 16 bytes, and a C1 Q4_K expert slab (884,736 B).
AUDIT_CASES = [
    (1, 1, []), (1, 2, [(0, 0x80)]), (15, 3, [(14, 1)]), (16, 4, []),
    (8191, 5, [(8190, 0xff)]), (8192, 6, [(0, 1), (100, 2)]), (8193, 7, [(8192, 4)]),
    (70001, 8, [(40000, 0x10), (40001, 0x10)]), (65536, 9, [(8191, 1), (8192, 1)]),
    (884736, 10, []), (884736, 11, [(884735, 0x01)]), (884736, 12, [(123457, 0x5a), (700000, 3)]),
]


def audit_pair(size, seed, flips):
    """(expected, actual) bytes of one audit case."""
    exp = slab_bytes(size, seed)
    act = exp.copy()
    for pos, mask in flips:
        act[pos] ^= mask
    return exp, act
