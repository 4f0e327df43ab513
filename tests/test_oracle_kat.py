"""Pins the CPU oracle against the reference's own known-answer tests.

Each test restates one test of xocialize/longcat-video-mlx ``tests/smoke/test_bsa_tier_a_smoke.py``
(or the RoPE test of ``tests/smoke/test_blocks_smoke.py``) on ``oracle/bsa_oracle.py``, plus
cross-checks between the numpy and C restatements of the fixed summation / selection orders.
"""

import math

import numpy as np
import pytest

from oracle import bsa_oracle as orc


def test_mean_pool_known_pattern():
    # test_bsa_tier_a_smoke.py:47-65: 8x8x8 grid, block (0,0,0) = 1, others 0
    T = H = W = 8
    D = 4
    x = np.zeros((1, 2, T, H, W, D), dtype=np.float32)
    x[:, :, :4, :4, :4, :] = 1.0
    y = orc.mean_pool_blocks_3d(x.reshape(1, 2, T * H * W, D), (T, H, W), (4, 4, 4))
    assert y.shape == (1, 2, 8, D)
    assert np.allclose(y[:, :, 0], 1.0)
    assert np.allclose(y[:, :, 1:], 0.0)


def test_routing_scores_simple():
    # test_bsa_tier_a_smoke.py:68-75: ones . twos over D=8 = 16
    q = np.ones((1, 1, 4, 8), np.float32)
    k = np.ones((1, 1, 4, 8), np.float32) * 2
    s = orc.block_routing_scores(q, k)
    assert s.shape == (1, 1, 4, 4)
    assert s[0, 0, 0, 0] == pytest.approx(16.0)


def test_topk_indices_count():
    # test_bsa_tier_a_smoke.py:78-86: 8 blocks, sparsity 0.75 -> k = 2, ids in range
    score = np.random.default_rng(0).standard_normal((1, 2, 4, 8)).astype(np.float32)
    idx, n = orc.topk_block_indices(score, sparsity=0.75)
    assert idx.shape == (1, 2, 4, 2) and n == 2
    assert (idx >= 0).all() and (idx < 8).all()


def test_topk_indices_minimum_one():
    # test_bsa_tier_a_smoke.py:89-94: sparsity 0.99 on 4 blocks clamps to 1
    score = np.random.default_rng(1).standard_normal((1, 1, 2, 4)).astype(np.float32)
    _, n = orc.topk_block_indices(score, sparsity=0.99)
    assert n == 1


def test_num_selected_floor_rule():
    # block_sparse_attention.py:127 -- floor; the benchmark configs use ceil (85/169/338)
    assert orc.num_selected_blocks(64, 0.9375) == 4
    assert orc.num_selected_blocks(1350, 0.9375) == 84
    assert orc.num_selected_blocks(2700, 0.9375) == 168
    assert orc.num_selected_blocks(1350, 0.875) == 168
    assert orc.num_selected_blocks(1350, 0.75) == 337
    assert [math.ceil((1 - s) * n) for s, n in ((0.9375, 1350), (0.9375, 2700), (0.875, 1350), (0.75, 1350))] == \
        [85, 169, 169, 338]


def test_token_block_indices():
    # test_bsa_tier_a_smoke.py:97-111
    assert (orc.build_token_block_indices((4, 4, 4), (4, 4, 4)) == 0).all()
    t2 = orc.build_token_block_indices((8, 4, 4), (4, 4, 4))
    assert t2.shape == (128,)
    assert (t2[:64] == 0).all() and (t2[64:] == 1).all()


def test_token_pair_mask():
    # test_bsa_tier_a_smoke.py:114-138: q-block 0 picks {3,5}, q-block 1 picks {0,7}
    bi = np.array([[[[3, 5], [0, 7]]]], dtype=np.int32)
    mask = orc.build_token_pair_mask(bi, np.arange(8, dtype=np.int32), 8)
    assert mask.shape == (1, 1, 8, 8)
    assert mask[0, 0, 0, 3] and mask[0, 0, 0, 5] and not mask[0, 0, 0, 0]
    assert mask[0, 0, 1, 0] and mask[0, 0, 1, 7] and not mask[0, 0, 1, 3]


def _dense(q, k, v, scale):
    s = np.einsum("bhqd,bhkd->bhqk", q.astype(np.float64), k.astype(np.float64)) * scale
    s -= s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    return np.einsum("bhqk,bhkd->bhqd", p, v.astype(np.float64))


def test_sparsity_zero_matches_dense():
    # test_bsa_tier_a_smoke.py:141-162 (the L24 gate): sparsity 0 == dense, max_abs < 1e-4
    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal((1, 4, 64, 16)).astype(np.float32) for _ in range(3))
    out, _ = orc.bsa_attention(q, k, v, shape=(4, 4, 4), sparsity=0.0)
    assert np.abs(out - _dense(q, k, v, 1 / math.sqrt(16))).max() < 1e-4


def test_sparse_gather_equals_masked_dense():
    # the kernel-level semantics (per-block gather) equal Tier A's masked dense SDPA
    rng = np.random.default_rng(3)
    q, k, v = (rng.standard_normal((1, 2, 512, 32)).astype(np.float32) for _ in range(3))
    out_a, idx = orc.bsa_attention(q, k, v, shape=(8, 8, 8), sparsity=0.75)
    out_b = orc.bsa_sparse_attention(q, k, v, idx, (8, 8, 8), (4, 4, 4))
    assert np.abs(out_a - out_b).max() < 1e-10


def test_no_nan_at_target_shape():
    # test_bsa_tier_a_smoke.py:165-184
    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal((1, 2, 256, 32)).astype(np.float32) for _ in range(3))
    out, _ = orc.bsa_attention(q, k, v, shape=(4, 8, 8), sparsity=0.9375)
    assert out.shape == (1, 2, 256, 32) and np.isfinite(out).all()


def test_rejects_non_multiple_shape():
    # test_bsa_tier_a_smoke.py:187-196
    q = np.zeros((1, 1, 4 * 4 * 6, 8), np.float32)
    with pytest.raises(ValueError, match=r"multiple of"):
        orc.bsa_attention(q, q, q, shape=(4, 4, 6), sparsity=0.9)


def test_c_pool_matches_numpy_bitwise():
    rng = np.random.default_rng(5)
    x = rng.standard_normal((2, 3, 8 * 8 * 8, 24)).astype(np.float32)
    for shape, chunk in (((8, 8, 8), (4, 4, 4)), ((8, 8, 8), (2, 4, 8)), ((1, 1, 512), (1, 1, 64)),
                         ((8, 8, 8), (2, 2, 2))):
        a = orc.mean_pool_blocks_3d(x, shape, chunk)
        b = orc.oracle_pool_c(x, shape, chunk)
        assert a.tobytes() == b.tobytes(), chunk


def test_c_topk_matches_numpy_rule_with_ties():
    rng = np.random.default_rng(6)
    # heavy ties: few distinct values, plus signed zeros
    s = rng.integers(-3, 4, size=(64, 200)).astype(np.float32)
    s[:, ::7] = -0.0
    for k in (1, 5, 37, 200):
        a, _ = orc.topk_block_indices(s, topk=k)
        b = orc.topk_block_indices_numpy(s, k)
        assert np.array_equal(a, b), k


def test_topk_rule_is_score_desc_then_index_asc():
    s = np.array([[1.0, 3.0, 3.0, 2.0, 3.0]], np.float32)
    idx, _ = orc.topk_block_indices(s, topk=2)
    assert idx.tolist() == [[1, 2]]
    idx, _ = orc.topk_block_indices(s, topk=4)
    assert idx.tolist() == [[1, 2, 3, 4]]


def test_scores_fma_chain():
    rng = np.random.default_rng(7)
    q = rng.standard_normal((1, 1, 5, 16)).astype(np.float32)
    k = rng.standard_normal((1, 1, 6, 16)).astype(np.float32)
    s = orc.block_routing_scores(q, k)
    ref = q.astype(np.float64)[0, 0] @ k.astype(np.float64)[0, 0].T
    assert np.abs(s[0, 0] - ref).max() < 1e-4


def test_rotate_half_kat():
    # test_blocks_smoke.py:134-140
    assert orc.rotate_half(np.array([1.0, 2.0, 3.0, 4.0], np.float32)).tolist() == [-2.0, 1.0, -4.0, 3.0]


def test_rope_dims_and_tables():
    # rope_3d.py:60-62 and the 44/42/42 split of the 720p config
    assert orc.rope_axis_dims(128) == (44, 42, 42)
    cos, sin = orc.rope_full_tables((2, 3, 4), 128)
    assert cos.shape == (24, 128)
    # position 0 on every axis has angle 0
    assert np.allclose(cos[0], 1.0) and np.allclose(sin[0], 0.0)
    # rotation preserves the norm of every pair
    x = np.random.default_rng(0).standard_normal((1, 1, 24, 128)).astype(np.float32)
    y = orc.apply_rope(x, cos, sin, "fp32")
    assert np.allclose(np.linalg.norm(x, axis=-1), np.linalg.norm(y, axis=-1), rtol=1e-5)


def test_bf16_rounding_is_rne():
    x = np.array([1.0, 1.00390625, 1.005859375, -2.5e-3, 3.0e38], np.float32)
    y = orc.round_to_bf16(x)
    assert y[0] == 1.0
    assert y[1] == 1.0            # tie -> even
    assert y[2] == 1.0078125      # above the tie -> up
    assert abs(y[3] - (-2.5e-3)) < 2e-5
