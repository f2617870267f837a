"""The bench's synthetic quantized weights (bench.synth_blocks) are valid ggml blocks: the
C oracle dequantizes them to finite weights of the magnitude of a quantized N(0, 0.02)
matrix, as the bench's JSON line claims in its `data` field.  CPU only."""
import numpy as np
import pytest

import bench
import oracle as O


@pytest.mark.parametrize("t", [O.Q4_K, O.Q6_K, O.Q8_0])
def test_synthetic_blocks_dequantize_to_small_finite_weights(t):
    rows, K = 64, 512
    b = bench.synth_blocks(t, rows, K, np.random.default_rng(3))
    assert b.dtype == np.uint8 and b.size == rows * O.row_size(t, K)
    w = O.dequantize(t, b, rows, K)
    assert w.shape == (rows, K) and np.isfinite(w).all()
    assert np.abs(w).max() < 0.05
    assert 0.002 < float(np.sqrt(np.mean(w.astype(np.float64) ** 2))) < 0.03
    # not degenerate: most weights differ from each other row to row
    assert np.unique(w).size > K


def test_expert_sets_are_seeded():
    a = bench.quantized_experts(seed=0)
    b = bench.quantized_experts(seed=0)
    assert all(np.array_equal(x, y) for x, y in zip(a, b))
    assert [x.size for x in a] == [bench.UNIQUE * bench.F * O.row_size(O.Q4_K, bench.H)] * 2 + \
        [bench.UNIQUE * bench.H * O.row_size(O.Q6_K, bench.F)]
