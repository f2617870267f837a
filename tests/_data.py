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
