"""GPU parity of the CUDA engine against the CPU oracle (oracle/bsa_oracle.py).

Contract (the engine's parity target): block indices bit-exact wherever the fp32 pooled scores are
computed identically (the engine and the oracle use the same fixed fp32 orders, so pooled means
and scores must match bit for bit); attention outputs within relative L2 <= 1e-2 and max-abs
<= 2e-2 of the fp32/fp64 oracle.
"""

import math

import numpy as np
import pytest
import torch

from oracle import bsa_oracle as orc

pytestmark = pytest.mark.gpu

REL_L2 = 1e-2
MAX_ABS = 2e-2


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def _rand(shape, dtype, seed, device, scale=1.0):
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(dtype).to(device)


def _close(out: np.ndarray, ref: np.ndarray):
    rel = np.linalg.norm(out - ref) / max(np.linalg.norm(ref), 1e-30)
    mx = np.abs(out - ref).max()
    assert rel <= REL_L2 and mx <= MAX_ABS, f"rel_l2={rel:.3e} max_abs={mx:.3e}"
    return rel, mx


GEOMS = [((4, 8, 8), (4, 4, 4)), ((1, 1, 1024), (1, 1, 64)), ((8, 4, 16), (2, 4, 8))]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("geom", GEOMS)
def test_pool_bitexact(cuda, dtype, geom):
    from longcat_video.models.block_sparse_attention import mean_pool_blocks_3d

    shape, chunk = geom
    S = shape[0] * shape[1] * shape[2]
    x = _rand((2, 3, S, 128), dtype, 1, cuda)
    got = mean_pool_blocks_3d(x, shape, chunk)
    ref = orc.mean_pool_blocks_3d(_np(x), shape, chunk)
    assert got.dtype == torch.float32
    assert _np(got).tobytes() == ref.tobytes()


def test_pool_strided_input_bitexact(cuda):
    # q/k/v as produced by the DiT: reshape(B, N, 3, H, D).permute(2, 0, 3, 1, 4)
    from longcat_video.models.block_sparse_attention import mean_pool_blocks_3d

    B, N, H, D = 1, 512, 4, 64
    qkv = _rand((B, N, 3, H, D), torch.bfloat16, 2, cuda).permute(2, 0, 3, 1, 4)
    q = qkv[0]
    assert not q.is_contiguous()
    got = mean_pool_blocks_3d(q, (8, 8, 8), (4, 4, 4))
    ref = orc.mean_pool_blocks_3d(_np(q), (8, 8, 8), (4, 4, 4))
    assert _np(got).tobytes() == ref.tobytes()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_pool_fused_rope_bitexact(cuda, dtype):
    from longcat_video import _native
    from longcat_video.models.rope_3d import RopeTables

    grid = (4, 6, 8)
    S = 192
    x = _rand((1, 2, S, 128), dtype, 3, cuda)
    rt = RopeTables(grid, 128, cuda)
    # product and oracle tables must be the same numbers
    tabs = orc.rope_axis_tables(grid, 128)
    assert np.array_equal(rt.host, np.concatenate([np.concatenate([c.ravel(), s.ravel()]) for c, s in tabs]))
    pooled, x_rot = _native.mean_pool(x, (1, 1, S), (1, 1, 64), rope=rt.native_args())
    cos, sin = orc.rope_full_tables(grid, 128)
    ref_rot = orc.apply_rope(_np(x), cos, sin, "bf16" if dtype == torch.bfloat16 else "fp16")
    assert _np(x_rot).tobytes() == ref_rot.tobytes()
    ref_pool = orc.mean_pool_blocks_3d(ref_rot, (1, 1, S), (1, 1, 64))
    assert _np(pooled).tobytes() == ref_pool.tobytes()


# nb up to 1536 keeps a row in 48 registers per lane, up to 3072 in 96, longer rows are re-read from memory
@pytest.mark.parametrize("nb,D,k", [(64, 128, 4), (130, 128, 9), (200, 64, 1), (96, 40, 96), (1350, 128, 85),
                                    (2000, 32, 130), (3200, 16, 50)])
def test_score_topk_bitexact(cuda, nb, D, k):
    from longcat_video import _native

    qp = _rand((1, 2, nb, D), torch.float32, 4, cuda)
    kp = _rand((1, 2, nb, D), torch.float32, 5, cuda)
    idx, scores = _native.score_topk(qp, kp, k, return_scores=True)
    ref_s = orc.block_routing_scores(_np(qp), _np(kp))
    assert _np(scores).tobytes() == ref_s.tobytes()
    ref_i, _ = orc.topk_block_indices(ref_s, topk=k)
    assert np.array_equal(idx.cpu().numpy(), ref_i)
    # the same indices without the score matrix (tensor-core keys + exact scores near the threshold)
    if nb <= 3072:
        fused, _ = _native.score_topk(qp, kp, k)
        assert _native.device_error(clear=True) == 0
        assert np.array_equal(fused.cpu().numpy(), ref_i)


def test_topk_from_scores_ties(cuda):
    from longcat_video.models.block_sparse_attention import topk_block_indices

    g = np.random.default_rng(9)
    s = g.integers(-2, 3, size=(1, 3, 50, 300)).astype(np.float32)
    s[..., ::11] = -0.0
    st = torch.from_numpy(s).to(cuda)
    for k in (1, 17, 150, 300):
        got, n = topk_block_indices(st, sparsity=0.0, topk=k)
        ref, _ = orc.topk_block_indices(s, topk=k)
        assert n == k and np.array_equal(got.cpu().numpy(), ref), k


def test_block_scores_rectangular(cuda):
    from longcat_video.models.block_sparse_attention import block_routing_scores

    q = _rand((1, 2, 7, 32), torch.float32, 6, cuda)
    k = _rand((1, 2, 13, 32), torch.float32, 7, cuda)
    got = block_routing_scores(q, k)
    ref = orc.block_routing_scores(_np(q), _np(k))
    assert _np(got).tobytes() == ref.tobytes()


def _random_indices(B, H, nb, k, seed):
    g = np.random.default_rng(seed)
    idx = np.stack([np.sort(g.choice(nb, size=k, replace=False)) for _ in range(B * H * nb)])
    return idx.reshape(B, H, nb, k).astype(np.int32)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [128, 64, 16])
@pytest.mark.parametrize("k", [1, 2, 5, 8])
def test_attention_indices_vs_oracle(cuda, dtype, D, k):
    from longcat_video.models.block_sparse_attention_cuda import bsa_attention_cuda

    shape, chunk = (8, 8, 8), (4, 4, 4)  # 8 voxel blocks, so k up to 8
    B, H, S = 1, 2, 512
    nb = S // 64
    q = _rand((B, H, S, D), dtype, 10 + D, cuda)
    kk = _rand((B, H, S, D), dtype, 20 + D, cuda)
    v = _rand((B, H, S, D), dtype, 30 + D, cuda)
    idx = _random_indices(B, H, nb, k, 40 + k)
    out = bsa_attention_cuda(q, kk, v, torch.from_numpy(idx).to(cuda), chunk_thw=chunk, shape=shape)
    torch.cuda.synchronize()
    ref = orc.bsa_sparse_attention(_np(q), _np(kk), _np(v), idx, shape, chunk)
    _close(_np(out), ref)


@pytest.mark.parametrize("geom", GEOMS)
def test_attention_geometries(cuda, geom):
    from longcat_video.models.block_sparse_attention_cuda import bsa_attention_cuda

    shape, chunk = geom
    if chunk[0] * chunk[1] * chunk[2] != 64:
        pytest.skip("kernel uses 64-token blocks")
    S = shape[0] * shape[1] * shape[2]
    nb = S // 64
    k = max(1, nb // 3)
    q, kk, v = (_rand((1, 2, S, 128), torch.bfloat16, s, cuda) for s in (50, 51, 52))
    idx = _random_indices(1, 2, nb, k, 53)
    out = bsa_attention_cuda(q, kk, v, torch.from_numpy(idx).to(cuda), chunk_thw=chunk, shape=shape)
    ref = orc.bsa_sparse_attention(_np(q), _np(kk), _np(v), idx, shape, chunk)
    _close(_np(out), ref)


def test_attention_single_block_equals_dense(cuda):
    # reference tests/smoke/test_bsa_tier_b_smoke.py:47-79: one block, top-1 == dense SDPA
    from longcat_video.models.block_sparse_attention_cuda import bsa_attention_cuda

    q, k, v = (_rand((1, 2, 64, 128), torch.bfloat16, s, cuda) for s in (60, 61, 62))
    out = bsa_attention_cuda(q, k, v, torch.zeros((1, 2, 1, 1), dtype=torch.int32, device=cuda),
                             chunk_thw=(4, 4, 4), shape=(4, 4, 4))
    dense = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float())
    _close(_np(out), _np(dense))


def test_attention_all_blocks_equals_dense(cuda):
    # reference tests/smoke/test_bsa_tier_b_smoke.py:82-117: every q block attends to every block
    from longcat_video.models.block_sparse_attention_cuda import bsa_attention_cuda

    S = 1024
    nb = S // 64
    q, k, v = (_rand((1, 2, S, 128), torch.bfloat16, s, cuda) for s in (63, 64, 65))
    idx = torch.arange(nb, dtype=torch.int32, device=cuda).expand(1, 2, nb, nb).contiguous()
    out = bsa_attention_cuda(q, k, v, idx, chunk_thw=(1, 1, 64), shape=(1, 1, S))
    dense = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float())
    _close(_np(out), _np(dense))


def test_batched_dit_views_run_sparse(cuda):
    """B > 1 DiT views (batch and head strides that do not merge) run the sparse path, not a shape error."""
    from longcat_video.models.block_sparse_attention import bsa_attention

    B, N, H, D = 2, 512, 3, 128
    qkv = _rand((B, N, 3, H, D), torch.bfloat16, 76, cuda).permute(2, 0, 3, 1, 4)
    q, k, v = qkv[0], qkv[1], qkv[2]
    a, ia = bsa_attention(q, k, v, (8, 8, 8), chunk_thw=(4, 4, 4), topk=3, return_indices=True)
    b, ib = bsa_attention(q.contiguous(), k.contiguous(), v.contiguous(), (8, 8, 8), chunk_thw=(4, 4, 4), topk=3,
                          return_indices=True)
    assert torch.equal(ia, ib) and torch.equal(a, b)


def test_attention_strided_inputs_match_contiguous(cuda):
    from longcat_video.models.block_sparse_attention_cuda import bsa_attention_cuda

    B, N, H, D = 1, 512, 4, 128
    qkv = _rand((B, N, 3, H, D), torch.bfloat16, 70, cuda).permute(2, 0, 3, 1, 4)
    q, k, v = qkv[0], qkv[1], qkv[2]
    idx = torch.from_numpy(_random_indices(B, H, N // 64, 3, 71)).to(cuda)
    a = bsa_attention_cuda(q, k, v, idx, chunk_thw=(4, 4, 4), shape=(8, 8, 8))
    b = bsa_attention_cuda(q.contiguous(), k.contiguous(), v.contiguous(), idx, chunk_thw=(4, 4, 4), shape=(8, 8, 8))
    assert torch.equal(a, b)


def test_bad_block_index_sets_device_error(cuda):
    from longcat_video import _native
    from longcat_video.models.block_sparse_attention_cuda import bsa_attention_cuda

    _native.device_error(clear=True)
    q = _rand((1, 1, 128, 128), torch.bfloat16, 72, cuda)
    idx = torch.tensor([[[[0, 1]], [[1, 1 << 20]]]], dtype=torch.int32, device=cuda).view(1, 1, 2, 2)
    bsa_attention_cuda(q, q, q, idx, chunk_thw=(1, 1, 64), shape=(1, 1, 128))
    assert _native.device_error(clear=True) == _native.BSA_ERR_INDEX


def test_rejections(cuda):
    from longcat_video.models.block_sparse_attention import bsa_attention
    from longcat_video.models.block_sparse_attention_cuda import bsa_attention_cuda

    q = _rand((1, 1, 96, 128), torch.bfloat16, 73, cuda)
    with pytest.raises(ValueError, match="multiple of"):
        bsa_attention(q, q, q, shape=(4, 4, 6), sparsity=0.9)
    with pytest.raises(ValueError, match="required"):
        bsa_attention_cuda(q, q, q, torch.zeros((1, 1, 1, 1), dtype=torch.int32, device=cuda))
    with pytest.raises(ValueError, match="multiple of block_size"):
        bsa_attention_cuda(q, q, q, torch.zeros((1, 1, 1, 1), dtype=torch.int32, device=cuda), shape=(1, 1, 96),
                           chunk_thw=(1, 1, 64))
    x = _rand((1, 1, 64, 128), torch.float32, 74, cuda).double()
    with pytest.raises(ValueError, match="dtype"):
        bsa_attention_cuda(x, x, x, torch.zeros((1, 1, 1, 1), dtype=torch.int32, device=cuda), shape=(4, 4, 4))
    y = _rand((1, 1, 64, 12), torch.bfloat16, 75, cuda)
    with pytest.raises(ValueError, match="multiple of 8"):
        bsa_attention_cuda(y, y, y, torch.zeros((1, 1, 1, 1), dtype=torch.int32, device=cuda), shape=(4, 4, 4))


def _full_forward_check(q, k, v, shape, chunk, topk, heads=None, qblocks=None, rope=None):
    """Engine forward vs oracle: indices exact on the checked heads, outputs within tolerance."""
    from longcat_video.models.block_sparse_attention import bsa_attention

    out, idx = bsa_attention(q, k, v, shape, chunk_thw=chunk, topk=topk, return_indices=True, rope=rope)
    torch.cuda.synchronize()
    hs = list(range(q.shape[1])) if heads is None else heads
    qn, kn, vn = (_np(t[:, hs]) for t in (q, k, v))
    if rope is not None:
        cos, sin = orc.rope_full_tables(rope.grid, q.shape[-1])
        dt = "bf16" if q.dtype == torch.bfloat16 else "fp16"
        qn = orc.apply_rope(qn, cos, sin, dt)
        kn = orc.apply_rope(kn, cos, sin, dt)
    qb = orc.mean_pool_blocks_3d(qn, shape, chunk)
    kb = orc.mean_pool_blocks_3d(kn, shape, chunk)
    ref_idx, _ = orc.topk_block_indices(orc.block_routing_scores(qb, kb), topk=topk)
    got_idx = idx[:, hs].cpu().numpy()
    assert np.array_equal(got_idx, ref_idx)
    ref = orc.bsa_sparse_attention(qn, kn, vn, ref_idx, shape, chunk, qblocks=qblocks)
    got = _np(out[:, hs])
    if qblocks is not None:
        got = orc.to_block_major(got, shape, chunk)[:, :, qblocks].reshape(ref.shape)
    return _close(got, ref)


def test_forward_config1_bf16(cuda):
    """Config 1 (H=4, S=4096, top-4) with the fp32 inputs rounded to bf16 on the device."""
    from longcat_video.workloads import make_config1_numpy

    q, k, v = (torch.from_numpy(a).to(cuda).to(torch.bfloat16) for a in make_config1_numpy(0))
    _full_forward_check(q, k, v, (1, 1, 4096), (1, 1, 64), 4)


def test_forward_config1_fp32(cuda):
    """Config 1 exactly as specified (fp32 inputs): fp32 routing equal to the oracle's, outputs within the
    contract (the attention runs on device-side fp16 copies and returns fp32)."""
    from longcat_video.workloads import make_config1_numpy

    q, k, v = (torch.from_numpy(a).to(cuda) for a in make_config1_numpy(0))
    _full_forward_check(q, k, v, (1, 1, 4096), (1, 1, 64), 4)


def test_attention_indices_fp32_io(cuda):
    from longcat_video.models.block_sparse_attention_cuda import bsa_attention_cuda

    shape, chunk = (1, 1, 1024), (1, 1, 64)
    q, k, v = (_rand((1, 2, 1024, 128), torch.float32, s, cuda) for s in (76, 77, 78))
    idx = torch.from_numpy(np.random.default_rng(3).integers(0, 16, size=(1, 2, 16, 5)).astype(np.int32)).to(cuda)
    out = bsa_attention_cuda(q, k, v, idx, chunk_thw=chunk, shape=shape)
    assert out.dtype == torch.float32
    ref = orc.bsa_sparse_attention(_np(q), _np(k), _np(v), idx.cpu().numpy(), shape, chunk)
    _close(_np(out), ref)


def test_forward_config1_golden_indices(cuda):
    """Config 1 fp32 routing on the engine equals the committed golden routing (oracle output)."""
    import os

    from longcat_video.models.block_sparse_attention import (block_routing_scores, mean_pool_blocks_3d,
                                                             topk_block_indices)
    from longcat_video.workloads import make_config1_numpy

    gold = np.load(os.path.join(os.path.dirname(__file__), "golden", "config1.npz"))
    q, k, _ = (torch.from_numpy(a).to(cuda) for a in make_config1_numpy(0))
    qb = mean_pool_blocks_3d(q, (1, 1, 4096), (1, 1, 64))
    kb = mean_pool_blocks_3d(k, (1, 1, 4096), (1, 1, 64))
    idx, n = topk_block_indices(block_routing_scores(qb, kb), sparsity=0.9375)
    assert n == 4
    assert np.array_equal(idx.cpu().numpy(), gold["block_indices"])


def test_forward_voxel_blocks_fp16(cuda):
    q, k, v = (_rand((1, 4, 8 * 16 * 16, 128), torch.float16, s, cuda) for s in (80, 81, 82))
    _full_forward_check(q, k, v, (8, 16, 16), (4, 4, 4), 5)


def test_forward_fused_rope(cuda):
    from longcat_video.models.rope_3d import RopeTables

    grid = (4, 8, 16)
    S = 512
    q, k, v = (_rand((1, 2, S, 128), torch.bfloat16, s, cuda) for s in (83, 84, 85))
    _full_forward_check(q, k, v, (1, 1, S), (1, 1, 64), 3, rope=RopeTables(grid, 128, cuda))


def test_forward_config2_fullsize(cuda):
    """Config 2 at full size: routing exact on two heads, outputs checked on sampled q blocks."""
    from longcat_video.workloads import CONFIGS, make_qkv

    cfg = CONFIGS["config2"]
    q, k, v = make_qkv(cfg, cuda, seed=0)
    _full_forward_check(q, k, v, cfg.shape, cfg.chunk, cfg.topk, heads=[0, 31], qblocks=[0, 1, 677, 1348, 1349])


def test_forward_config3_fp16_near_ties(cuda):
    """Config 3 (fp16, i.i.d. inputs, near-tied pooled scores): exact routing on 3 heads."""
    from longcat_video.workloads import CONFIGS, make_qkv

    cfg = CONFIGS["config3_s0.9375"]
    q, k, v = make_qkv(cfg, cuda, seed=1, heads=3)
    _full_forward_check(q, k, v, cfg.shape, cfg.chunk, cfg.topk, qblocks=[0, 5, 900])


def test_attention_hook_routes_to_engine(cuda):
    from longcat_video.models.attention import Attention

    torch.manual_seed(0)
    attn = Attention(256, 2).to(cuda).to(torch.bfloat16)
    x = torch.randn((1, 512, 256), device=cuda, dtype=torch.bfloat16)
    dense = attn(x, (8, 8, 8))
    attn.enable_bsa = True
    attn.bsa_sparsity = 0.0  # keep every block: must equal dense attention
    sparse = attn(x, (8, 8, 8))
    _close(_np(sparse), _np(dense))
    attn.bsa_sparsity = 0.75
    part = attn(x, (8, 8, 8))
    assert torch.isfinite(part).all()


@pytest.mark.parametrize("B,H,group", [(1, 5, 2), (2, 3, None), (1, 32, None)])
def test_host_tensors_stream_through_gpu(cuda, B, H, group):
    """Host q/k/v: the head-group pipeline returns a host tensor equal bit for bit to the device call
    (heads are independent; the same kernels run on the same values), ragged last group included."""
    from longcat_video.models import block_sparse_attention as bsa

    S = 1024 if H < 32 else 4096
    q, k, v = (_rand((B, H, S, 128), torch.bfloat16, s, "cpu") for s in (90, 91, 92))
    shape, chunk, topk = (1, 1, S), (1, 1, 64), 3
    dev_out, dev_idx = bsa.bsa_attention(q.to(cuda), k.to(cuda), v.to(cuda), shape, chunk_thw=chunk, topk=topk,
                                         return_indices=True)
    if group is None:
        host_out, host_idx = bsa.bsa_attention(q.pin_memory(), k.pin_memory(), v.pin_memory(), shape,
                                               chunk_thw=chunk, topk=topk, return_indices=True)
    else:
        host_out, host_idx = bsa._forward_host_streamed(q, k, v, shape, chunk, topk, 1.0 / math.sqrt(128), None,
                                                        True, heads_per_group=group)
    assert host_out.device.type == "cpu" and host_idx.device.type == "cpu"
    assert torch.equal(host_idx, dev_idx.cpu())
    assert torch.equal(host_out, dev_out.cpu())


# ------------------------------------------------------------------ the benchmark shapes at full size
@pytest.mark.parametrize("name", ["config3_s0.875", "config3_s0.75"])
def test_forward_config3_fp16_sparsity_sweep(cuda, name):
    """Config 3 at k = 169 and k = 338 (fp16, i.i.d. inputs, near-tied pooled scores): routing exact on
    every q block of two heads, outputs on sampled q blocks."""
    from longcat_video.workloads import CONFIGS, make_qkv

    cfg = CONFIGS[name]
    q, k, v = make_qkv(cfg, cuda, seed=2, heads=2)
    _full_forward_check(q, k, v, cfg.shape, cfg.chunk, cfg.topk, qblocks=[0, 1, 500, 1348, 1349])


def test_forward_config4_fused_rope_fullsize(cuda):
    """Config 4: pre-RoPE Q/K with the 3-D RoPE of the real 24x45x80 latent grid fused into routing.
    The rotated bytes equal the oracle's, routing is exact on two heads, outputs on sampled q blocks."""
    from longcat_video import _native
    from longcat_video.models.rope_3d import RopeTables
    from longcat_video.workloads import CONFIGS, make_qkv

    cfg = CONFIGS["config4"]
    q, k, v = make_qkv(cfg, cuda, seed=3, heads=2)
    rope = RopeTables(cfg.grid, cfg.D, cuda)
    _, q_rot = _native.mean_pool(q, cfg.shape, cfg.chunk, rope=rope.native_args())
    cos, sin = orc.rope_full_tables(cfg.grid, cfg.D)
    rows = np.r_[0:256, 40000:40256, cfg.S - 256:cfg.S]  # first, middle and last tokens of every head
    ref_rot = orc.apply_rope(_np(q[:, :, rows]), cos[rows], sin[rows], "bf16")
    assert _np(q_rot[:, :, rows]).tobytes() == ref_rot.tobytes()
    _full_forward_check(q, k, v, cfg.shape, cfg.chunk, cfg.topk, qblocks=[0, 700, 1349], rope=rope)


def test_forward_config5_fullsize(cuda):
    """Config 5 (S = 172,800, 2,700 blocks, top-169): rows of 2,700 keys take the 96-keys-per-lane
    selection, and every unit runs 85 two-block steps.  Routing exact on two heads."""
    from longcat_video.workloads import CONFIGS, make_qkv

    cfg = CONFIGS["config5"]
    q, k, v = make_qkv(cfg, cuda, seed=4, heads=2)
    _full_forward_check(q, k, v, cfg.shape, cfg.chunk, cfg.topk, qblocks=[0, 1351, 2699])


@pytest.mark.parametrize("k", [1, 2, 3])
def test_attention_many_units_per_cta(cuda, k):
    """608 (head, q-block) units on 148 persistent CTAs: every CTA runs four or five units back to back.
    With k = 1 or 2 there is one two-block step per unit, so lane half 1 of the kernel stays idle while
    the unit loop, the Q buffers and the epilogue hand-offs cycle."""
    from longcat_video.models.block_sparse_attention_cuda import bsa_attention_cuda

    B, H, S, D = 1, 8, 4864, 128
    nb = S // 64
    q, kk, v = (_rand((B, H, S, D), torch.bfloat16, s, cuda) for s in (100 + k, 110 + k, 120 + k))
    idx = _random_indices(B, H, nb, k, 130 + k)
    out = bsa_attention_cuda(q, kk, v, torch.from_numpy(idx).to(cuda), chunk_thw=(1, 1, 64), shape=(1, 1, S))
    torch.cuda.synchronize()
    ref = orc.bsa_sparse_attention(_np(q), _np(kk), _np(v), idx, (1, 1, S), (1, 1, 64))
    _close(_np(out), ref)


def test_misaligned_view_runs_the_engine(cuda):
    """A view the TMA maps cannot read in place (base 2 bytes past a 16-byte boundary) is copied once by
    the host layer and computed by the engine: bit-identical to the contiguous call, no dense fallback."""
    from longcat_video.models.block_sparse_attention import bsa_attention

    B, H, S, D = 1, 2, 512, 128
    flat = _rand((3 * B * H * S * D + 1,), torch.bfloat16, 140, cuda)
    q, k, v = (flat[1 + i * B * H * S * D:1 + (i + 1) * B * H * S * D].view(B, H, S, D) for i in range(3))
    a, ia = bsa_attention(q, k, v, (8, 8, 8), chunk_thw=(4, 4, 4), topk=3, return_indices=True)
    b, ib = bsa_attention(q.clone(), k.clone(), v.clone(), (8, 8, 8), chunk_thw=(4, 4, 4), topk=3,
                          return_indices=True)
    assert torch.equal(ia, ib) and torch.equal(a, b)


def _route_vs_oracle(cuda, qp, kp, k):
    from longcat_video import _native

    got, _ = _native.score_topk(qp.to(cuda), kp.to(cuda), k)
    assert _native.device_error(clear=True) == 0
    ref, _ = orc.topk_block_indices(orc.block_routing_scores(_np(qp), _np(kp)), topk=k)
    assert np.array_equal(got.cpu().numpy(), ref)


@pytest.mark.parametrize("nb,D,k", [(1, 128, 1), (7, 8, 3), (129, 40, 128), (1350, 128, 85), (1350, 128, 338),
                                    (1536, 64, 1), (1537, 128, 700), (2700, 128, 169), (3072, 16, 3072)])
def test_route_bitexact_sizes(cuda, nb, D, k):
    """Routing without the score matrix equals the exact scores + top-k at every row-tile remainder, both
    key-row widths (48 and 96 keys per lane), k = 1 and k = nb, and small head dims."""
    g = torch.Generator().manual_seed(nb * 7 + D)
    qp, kp = (torch.randn((1, 2, nb, D), generator=g) for _ in range(2))
    _route_vs_oracle(cuda, qp, kp, k)


def test_route_near_ties(cuda):
    """Pooled i.i.d. fp16 blocks (the config-3 regime: scores crowd around the threshold): the band of
    blocks scored exactly is dense, and the result is still exact."""
    g = torch.Generator().manual_seed(11)
    x = torch.randn((2, 3, 1350, 64, 128), generator=g).half().float().mean(dim=3)
    _route_vs_oracle(cuda, x[0].unsqueeze(0), x[1].unsqueeze(0), 169)


def test_route_degenerate_rows_fall_back_to_exact(cuda):
    """Rows the fast path cannot bound -- all scores tied, a non-finite or enormous key block, a zero query
    block -- are scored exactly in full and still match the oracle."""
    g = torch.Generator().manual_seed(12)
    nb, D = 300, 64
    qp = torch.randn((1, 4, nb, D), generator=g)
    kp = torch.randn((1, 4, nb, D), generator=g)
    kp[0, 0] = 1.0                      # head 0: every key block equal -> every score of a row tied
    kp[0, 1, 17, 3] = 3.0e20            # head 1: one enormous key value (outside the norm bound's range)
    qp[0, 2, 5] = 0.0                   # head 2: a zero query block (a row of zero scores)
    qp[0, 3] = torch.round(qp[0, 3] * 4) / 4   # head 3: coarse values, many exact score ties
    kp[0, 3] = torch.round(kp[0, 3] * 4) / 4
    for k in (1, 30, 150):
        _route_vs_oracle(cuda, qp, kp, k)


def test_route_wide_rows_take_the_radix_select(cuda):
    """Rows whose k-th largest score lies far (more than a factor of 4) below the row's largest: the window
    next to the largest key cannot hold the k-th key and the select falls back to the two-byte radix.  A
    few key blocks scaled by 1000 in head 0, and k near the median score (mixed signs) in both heads."""
    g = torch.Generator().manual_seed(13)
    nb, D = 1350, 128
    qp = torch.randn((1, 2, nb, D), generator=g)
    kp = torch.randn((1, 2, nb, D), generator=g)
    kp[0, 0, ::100] *= 1000.0
    for k in (10, 85, 675):
        _route_vs_oracle(cuda, qp, kp, k)


def test_phase_event_splits_one_forward_call(cuda):
    """bsa_set_phase_event: the event lands between the routing and the attention launches of a forward call
    (both phases take time), the call's results are those of a call without it, and clearing it stops it."""
    from longcat_video import _native

    B, H, S, D = 1, 2, 4096, 128
    q, k, v = (_rand((B, H, S, D), torch.bfloat16, 150 + i, cuda) for i in range(3))
    ref, ref_idx = _native.forward(q, k, v, (1, 1, S), (1, 1, 64), 8, D ** -0.5)
    e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    e0.record()
    _native.set_phase_event(e1)
    try:
        out, idx = _native.forward(q, k, v, (1, 1, S), (1, 1, 64), 8, D ** -0.5)
    finally:
        _native.set_phase_event(None)
    e2.record()
    torch.cuda.synchronize()
    assert _native.device_error(clear=True) == 0
    assert e0.elapsed_time(e1) > 0 and e1.elapsed_time(e2) > 0
    assert torch.equal(idx, ref_idx) and torch.equal(out, ref)


def test_cond_branch_through_the_engine(cuda):
    """attention.py:203-223 on the GPU: with conditioning latents the cond frames run BSA on the engine over
    (num_cond_latents, H, W) and the noise queries attend densely to cond + noise keys.  Each branch is
    checked against its reference on the same bf16 q/k/v: the cond rows against the oracle's bsa_attention
    on the RoPE'd q/k, the noise rows against fp32 dense SDPA; the module output is proj(cond | noise)."""
    from longcat_video.models.attention import Attention

    torch.manual_seed(0)
    attn = Attention(256, 2).to(cuda).to(torch.bfloat16)
    attn.enable_bsa = True
    attn.bsa_sparsity = 0.5  # 4 cond blocks of 4x4x4 -> top-2
    shape, ncl = (8, 8, 8), 4
    x = torch.randn((1, 512, 256), device=cuda, dtype=torch.bfloat16)
    calls = []
    orig = Attention._process_attn

    def record(self, q, k, v, shape=None, rope_grid=None):
        out = orig(self, q, k, v, shape=shape, rope_grid=rope_grid)
        calls.append((q.clone(), k.clone(), v.clone(), shape, out.clone()))
        return out

    Attention._process_attn = record
    try:
        with torch.no_grad():
            y = attn(x, shape, num_cond_latents=ncl)
    finally:
        Attention._process_attn = orig
    torch.cuda.synchronize()
    assert len(calls) == 2
    (qc, kc, vc, cond_shape, oc), (qn, kn, vn, noise_shape, on) = calls
    assert cond_shape == (ncl, 8, 8) and noise_shape is None and qc.shape[2] == ncl * 64
    ref_c, _ = orc.bsa_attention(_np(qc), _np(kc), _np(vc), cond_shape, sparsity=0.5, chunk_thw=(4, 4, 4),
                                 sm_scale=attn.scale)
    _close(_np(oc), ref_c)
    ref_n = torch.nn.functional.scaled_dot_product_attention(qn.float(), kn.float(), vn.float(), scale=attn.scale)
    _close(_np(on), _np(ref_n))
    want = attn.proj(torch.cat([oc, on], dim=2).transpose(1, 2).reshape(1, 512, 256))
    assert torch.equal(y, want)


def test_kv_cache_continuation_on_gpu(cuda):
    """attention.py:235-275 on the GPU: the continuation from the cached (k, v) of the conditioning frames
    gives the noise rows of the one-shot cond + noise forward (bf16, within the output tolerance)."""
    from longcat_video.models.attention import Attention

    torch.manual_seed(1)
    attn = Attention(128, 2).to(cuda).to(torch.bfloat16)
    attn.enable_bsa = True
    T, Hl, Wl, ncl = 8, 4, 4, 4
    nc = ncl * Hl * Wl
    x = torch.randn((1, T * Hl * Wl, 128), device=cuda, dtype=torch.bfloat16)
    with torch.no_grad():
        full = attn(x, (T, Hl, Wl), num_cond_latents=ncl)
        _, kv = attn(x[:, :nc], (ncl, Hl, Wl), return_kv=True)
        cont = attn.forward_with_kv_cache(x[:, nc:], (T - ncl, Hl, Wl), ncl, kv)
    _close(_np(cont), _np(full[:, nc:]))


def test_hook_writes_the_proj_layout_in_place(cuda):
    """The BSA path of the hook hands the engine a [B, N, H, D] buffer (viewed as [B, H, N, D]), so proj reads
    it without the transpose copy of attention.py:228-229; the result is the same as the transpose path."""
    from longcat_video.models.attention import Attention

    torch.manual_seed(3)
    attn = Attention(256, 2).to(cuda).to(torch.bfloat16)
    attn.enable_bsa = True
    attn.bsa_sparsity = 0.5
    x = torch.randn((1, 512, 256), device=cuda, dtype=torch.bfloat16)
    with torch.no_grad():
        y = attn(x, (8, 8, 8))
        qkv = attn.qkv(x).reshape(1, 512, 3, 2, 128).permute(2, 0, 3, 1, 4)
        q, k, v = attn.q_norm(qkv[0]), attn.k_norm(qkv[1]), qkv[2]
        o = attn._process_attn(q, k, v, shape=(8, 8, 8), rope_grid=(8, 8, 8))
        want = attn.proj(o.transpose(1, 2).reshape(1, 512, 256))
    assert torch.equal(y, want)


def test_enable_bsa_prewarms_the_engine(cuda):
    """enable_bsa on a CUDA model runs the engine once (longcat_video_dit.py:220-257 + the Metal tier's
    prewarm, block_sparse_attention_metal.py:298-333): the library is loaded and no device error is left."""
    from longcat_video import _native
    from longcat_video.models.longcat_video_dit import LongCatVideoTransformer3DModel

    dit = LongCatVideoTransformer3DModel(hidden_size=256, depth=2, num_heads=2).to(cuda).to(torch.bfloat16)
    dit.enable_bsa(backend="cuda")
    assert _native.library_loaded()
    assert _native.device_error(clear=True) == 0
    assert all(b.attn.enable_bsa for b in dit.blocks)


def _ulp_distance(a: np.ndarray, b: np.ndarray, dtype: str) -> np.ndarray:
    """Distance in units in the last place of bf16 / fp16 values (fp32 arrays holding exact 16-bit values)."""
    if dtype == "bf16":
        ia = (a.astype(np.float32).view(np.uint32) >> 16).astype(np.int64)
        ib = (b.astype(np.float32).view(np.uint32) >> 16).astype(np.int64)
        sign = 0x8000
    else:
        ia = a.astype(np.float16).view(np.uint16).astype(np.int64)
        ib = b.astype(np.float16).view(np.uint16).astype(np.int64)
        sign = 0x8000
    oa = np.where(ia & sign, -(ia & (sign - 1)), ia)
    ob = np.where(ib & sign, -(ib & (sign - 1)), ib)
    return np.abs(oa - ob)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fused_qk_norm_rope_pool(cuda, dtype):
    """RMSNorm_FP32 + 3-D RoPE + pooling in one pass (blocks.py:55-73, rope_3d.py:107-128,
    block_sparse_attention.py:67-104).  The normalised rows are within one input-dtype ulp of the
    fp64-normed oracle (the engine's fp32 rsqrt is within a few fp32 ulps); after the rotation, which
    mixes two such values, within two.  The pooled blocks are bit-exact to the oracle's pooling of the
    engine's own rows."""
    from longcat_video import _native
    from longcat_video.models.rope_3d import RopeTables

    grid = (4, 6, 8)
    S = 192
    g = torch.Generator().manual_seed(21)
    x = (torch.randn((1, 2, S, 128), generator=g) * 3.0).to(dtype).to(cuda)
    w = (1.0 + 0.1 * torch.randn((128,), generator=g)).to(dtype).to(cuda)
    dt = "bf16" if dtype == torch.bfloat16 else "fp16"
    normed = orc.rms_norm_fp32(_np(x), _np(w), 1e-6, dt)
    pooled_n, x_n = _native.mean_pool(x, (1, 1, S), (1, 1, 64), norm=(w, 1e-6))
    rt = RopeTables(grid, 128, cuda)
    pooled, x_rot = _native.mean_pool(x, (1, 1, S), (1, 1, 64), rope=rt.native_args(), norm=(w, 1e-6))
    torch.cuda.synchronize()
    d_norm = _ulp_distance(_np(x_n), normed, dt)
    assert d_norm.max() <= 1 and (d_norm > 0).mean() < 0.01
    cos, sin = orc.rope_full_tables(grid, 128)
    assert _ulp_distance(_np(x_rot), orc.apply_rope(normed, cos, sin, dt), dt).max() <= 2
    # the rotation of the engine's own normalised rows is exact
    assert _np(x_rot).tobytes() == orc.apply_rope(_np(x_n), cos, sin, dt).tobytes()
    for pool, rows in ((pooled_n, x_n), (pooled, x_rot)):
        assert _np(pool).tobytes() == orc.mean_pool_blocks_3d(_np(rows), (1, 1, S), (1, 1, 64)).tobytes()


def test_fused_qk_norm_forward_config4(cuda):
    """Config-4 shape with the raw q/k of the projection: RMSNorm, RoPE and pooling fused.  The routing is
    exact on the engine's own normalised, rotated q/k; outputs within the contract; and the result agrees
    with normalising in torch first and fusing only the RoPE."""
    from longcat_video.models.block_sparse_attention import bsa_attention
    from longcat_video.models.rope_3d import RopeTables
    from longcat_video.workloads import CONFIGS, make_qkv

    cfg = CONFIGS["config4"]
    q, k, v = make_qkv(cfg, cuda, seed=5, heads=2)
    g = torch.Generator().manual_seed(22)
    wq, wk = ((1.0 + 0.1 * torch.randn((128,), generator=g)).to(torch.bfloat16).to(cuda) for _ in range(2))
    rope = RopeTables(cfg.grid, cfg.D, cuda)
    out, idx = bsa_attention(q, k, v, cfg.shape, chunk_thw=cfg.chunk, topk=cfg.topk, rope=rope,
                             qk_norm=(wq, wk, 1e-6), return_indices=True)
    from longcat_video import _native

    _, q_rot = _native.mean_pool(q, cfg.shape, cfg.chunk, rope=rope.native_args(), norm=(wq, 1e-6))
    _, k_rot = _native.mean_pool(k, cfg.shape, cfg.chunk, rope=rope.native_args(), norm=(wk, 1e-6))
    torch.cuda.synchronize()
    qn, kn, vn = _np(q_rot), _np(k_rot), _np(v)
    qb = orc.mean_pool_blocks_3d(qn, cfg.shape, cfg.chunk)
    kb = orc.mean_pool_blocks_3d(kn, cfg.shape, cfg.chunk)
    ref_idx, _ = orc.topk_block_indices(orc.block_routing_scores(qb, kb), topk=cfg.topk)
    assert np.array_equal(idx.cpu().numpy(), ref_idx)
    ref = orc.bsa_sparse_attention(qn, kn, vn, ref_idx, cfg.shape, cfg.chunk, qblocks=[0, 700, 1349])
    _close(orc.to_block_major(_np(out), cfg.shape, cfg.chunk)[:, :, [0, 700, 1349]].reshape(ref.shape), ref)


def test_hook_fuses_the_qk_norm(cuda):
    """The DiT hook on the BSA path passes the raw q/k with the norm weights (no torch RMSNorm); its output
    is within the contract of the unfused hook (norm in torch, RoPE fused)."""
    from longcat_video.models.attention import Attention

    torch.manual_seed(4)
    attn = Attention(256, 2).to(cuda).to(torch.bfloat16)
    with torch.no_grad():
        attn.q_norm.weight.mul_(1.1)
        attn.k_norm.weight.mul_(0.9)
    attn.enable_bsa = True
    attn.bsa_sparsity = 0.5
    x = torch.randn((1, 512, 256), device=cuda, dtype=torch.bfloat16)
    calls = []
    orig_norm = type(attn.q_norm).forward

    def counting(self, t):
        calls.append(1)
        return orig_norm(self, t)

    type(attn.q_norm).forward = counting
    try:
        with torch.no_grad():
            fused = attn(x, (8, 8, 8))
            assert not calls  # the norms ran in the engine
            _, kv = attn(x, (8, 8, 8), return_kv=True)  # the unfused hook (a cache needs the normed k)
            assert calls
            qkv = attn.qkv(x).reshape(1, 512, 3, 2, 128).permute(2, 0, 3, 1, 4)
            o = attn._process_attn(attn.q_norm(qkv[0]), attn.k_norm(qkv[1]), qkv[2], shape=(8, 8, 8),
                                   rope_grid=(8, 8, 8))
            unfused = attn.proj(o.transpose(1, 2).reshape(1, 512, 256))
    finally:
        type(attn.q_norm).forward = orig_norm
    _close(_np(fused), _np(unfused))
