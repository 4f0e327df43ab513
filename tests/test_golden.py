"""The oracle reproduces the committed golden fixtures (tests/golden/make_golden.py)."""

import os

import numpy as np

from oracle import bsa_oracle as orc

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _config1_inputs():
    rng = np.random.default_rng(0)
    return tuple(rng.standard_normal((1, 4, 4096, 128), dtype=np.float32) for _ in range(3))


def test_config1_routing_and_output():
    g = np.load(os.path.join(GOLD, "config1.npz"))
    q, k, v = _config1_inputs()
    shape, chunk = (1, 1, 4096), (1, 1, 64)
    qb = orc.mean_pool_blocks_3d(q, shape, chunk)
    kb = orc.mean_pool_blocks_3d(k, shape, chunk)
    assert np.array_equal(qb.astype(np.float64).sum(axis=(2, 3)), g["q_pooled_sum"])
    assert np.array_equal(kb.astype(np.float64).sum(axis=(2, 3)), g["k_pooled_sum"])
    idx, n = orc.topk_block_indices(orc.block_routing_scores(qb, kb), sparsity=0.9375)
    assert n == 4 and idx.shape == (1, 4, 64, 4)
    assert np.array_equal(idx, g["block_indices"])
    out = orc.bsa_sparse_attention(q, k, v, idx, shape, chunk, qblocks=[0, 63]).astype(np.float32)
    assert np.allclose(out, g["out_qblocks_0_63"], rtol=0, atol=1e-6)


def test_config1_matches_workload_generator():
    import sys

    sys.path.insert(0, os.path.join(os.path.dirname(GOLD), "..", "longcat-video-mlx_b200"))
    from longcat_video.workloads import make_config1_numpy

    for a, b in zip(make_config1_numpy(0), _config1_inputs()):
        assert np.array_equal(a, b)


def test_small_fixture():
    g = np.load(os.path.join(GOLD, "small.npz"))
    shape, chunk = (4, 8, 8), (4, 4, 4)
    qb = orc.mean_pool_blocks_3d(g["q"], shape, chunk)
    kb = orc.mean_pool_blocks_3d(g["k"], shape, chunk)
    assert qb.tobytes() == g["q_pooled"].tobytes() and kb.tobytes() == g["k_pooled"].tobytes()
    s = orc.block_routing_scores(qb, kb)
    assert s.tobytes() == g["scores"].tobytes()
    idx, n = orc.topk_block_indices(s, sparsity=0.5)
    assert n == 2 and np.array_equal(idx, g["block_indices"])
    out, _ = orc.bsa_attention(g["q"], g["k"], g["v"], shape, sparsity=0.5, chunk_thw=chunk)
    assert np.allclose(out, g["out"], rtol=0, atol=1e-6)
