"""Generate the committed golden fixtures from the CPU oracle (oracle/bsa_oracle.py).

    python tests/golden/make_golden.py

config1.npz : config 1 (H=4, S=4096 as 64 contiguous blocks, top-4 = floor(6.25% of 64), fp32,
              numpy default_rng(0) standard normals for q, k, v in that order): block indices
              [1,4,64,4], fp32 pooled Q/K checksums and the fp64 oracle output of q blocks 0 and 63.
small.npz   : a 4x8x8 latent with 4x4x4 voxel blocks, H=2, D=32, sparsity 0.5: inputs and every
              intermediate (pooled, scores, indices, output).
"""

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "longcat-video-mlx_b200"))

from oracle import bsa_oracle as orc  # noqa: E402


def config1_inputs(seed=0):
    rng = np.random.default_rng(seed)
    shape = (1, 4, 4096, 128)
    return tuple(rng.standard_normal(shape, dtype=np.float32) for _ in range(3))


def make_config1():
    q, k, v = config1_inputs(0)
    shape, chunk = (1, 1, 4096), (1, 1, 64)
    qb = orc.mean_pool_blocks_3d(q, shape, chunk)
    kb = orc.mean_pool_blocks_3d(k, shape, chunk)
    score = orc.block_routing_scores(qb, kb)
    idx, n = orc.topk_block_indices(score, sparsity=0.9375)
    assert n == 4
    out = orc.bsa_sparse_attention(q, k, v, idx, shape, chunk, qblocks=[0, 63]).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "config1.npz"), block_indices=idx,
                        q_pooled_sum=qb.astype(np.float64).sum(axis=(2, 3)),
                        k_pooled_sum=kb.astype(np.float64).sum(axis=(2, 3)), out_qblocks_0_63=out)


def make_small():
    rng = np.random.default_rng(1234)
    shape, chunk = (4, 8, 8), (4, 4, 4)
    q, k, v = (rng.standard_normal((1, 2, 256, 32), dtype=np.float32) for _ in range(3))
    qb = orc.mean_pool_blocks_3d(q, shape, chunk)
    kb = orc.mean_pool_blocks_3d(k, shape, chunk)
    score = orc.block_routing_scores(qb, kb)
    idx, n = orc.topk_block_indices(score, sparsity=0.5)
    out, idx2 = orc.bsa_attention(q, k, v, shape, sparsity=0.5, chunk_thw=chunk)
    assert np.array_equal(idx, idx2) and n == 2
    np.savez_compressed(os.path.join(HERE, "small.npz"), q=q, k=k, v=v, q_pooled=qb, k_pooled=kb, scores=score,
                        block_indices=idx, out=out.astype(np.float32))


if __name__ == "__main__":
    make_config1()
    make_small()
    for f in ("config1.npz", "small.npz"):
        print(f, os.path.getsize(os.path.join(HERE, f)), "bytes")
