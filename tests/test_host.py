"""Host-side logic on CPU: DiT BSA wiring (reference tests/smoke/test_bsa_dit_wiring_smoke.py),
argument validation of the Python layer, workload definitions, and the Ulysses re-sharding on
gloo ranks (world size 2)."""

import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp


def _cfg(enable_bsa=False):
    return {"hidden_size": 64, "depth": 2, "num_heads": 4,
            "bsa_params": {"sparsity": 0.9375, "chunk_3d_shape_q": [4, 4, 4], "chunk_3d_shape_k": [4, 4, 4]},
            "enable_bsa": enable_bsa}


def test_default_bsa_off():
    from longcat_video.models.longcat_video_dit import LongCatVideoTransformer3DModel

    dit = LongCatVideoTransformer3DModel.from_config(_cfg(False))
    assert all(b.attn.enable_bsa is False for b in dit.blocks)


def test_config_enable_bsa_flips_attention():
    from longcat_video.models.longcat_video_dit import LongCatVideoTransformer3DModel

    dit = LongCatVideoTransformer3DModel.from_config(_cfg(True))
    for b in dit.blocks:
        assert b.attn.enable_bsa is True
        assert b.attn.bsa_sparsity == 0.9375
        assert b.attn.bsa_chunk_thw == (4, 4, 4)


def test_enable_disable_roundtrip_and_backends():
    from longcat_video.models.longcat_video_dit import LongCatVideoTransformer3DModel

    dit = LongCatVideoTransformer3DModel.from_config(_cfg(False))
    for backend in ("tier_a", "metal", "metal_v2", "metal_v3", "metal_v4", "cuda"):
        dit.enable_bsa(backend=backend)
        assert all(b.attn.enable_bsa and b.attn.bsa_backend == backend for b in dit.blocks)
    dit.disable_bsa()
    assert all(b.attn.enable_bsa is False for b in dit.blocks)
    with pytest.raises(AssertionError):
        dit.enable_bsa(backend="triton")


def test_bsa_params_preserved_through_enable():
    from longcat_video.models.longcat_video_dit import LongCatVideoTransformer3DModel

    cfg = _cfg(False)
    cfg["bsa_params"]["sparsity"] = 0.5
    cfg["bsa_params"]["chunk_3d_shape_q"] = [2, 2, 2]
    dit = LongCatVideoTransformer3DModel.from_config(cfg)
    dit.enable_bsa()
    assert all(b.attn.bsa_sparsity == 0.5 and b.attn.bsa_chunk_thw == (2, 2, 2) for b in dit.blocks)


def test_cpu_tensors_are_rejected_not_computed():
    from longcat_video.models.block_sparse_attention import bsa_attention

    q = torch.zeros((1, 1, 64, 128), dtype=torch.bfloat16)
    with pytest.raises((ValueError, RuntimeError)):
        bsa_attention(q, q, q, shape=(4, 4, 4))


def test_python_geometry_errors_match_reference_wording():
    from longcat_video import _native

    with pytest.raises(ValueError, match="multiple of"):
        _native._geometry(96, (4, 4, 6), (4, 4, 4))
    with pytest.raises(ValueError, match="doesn't match"):
        _native._geometry(100, (4, 4, 4), (4, 4, 4))


def test_workload_configs():
    from longcat_video.workloads import CONFIGS, ceil_topk

    c2 = CONFIGS["config2"]
    assert (c2.S, c2.nb, c2.topk) == (86400, 1350, 85)
    assert c2.sparse_flops() == pytest.approx(7.70e12, rel=1e-3)
    assert CONFIGS["config5"].nb == 2700 and CONFIGS["config5"].topk == 169
    assert [ceil_topk(1350, s) for s in (0.75, 0.875, 0.9375)] == [338, 169, 85]
    assert [CONFIGS[f"config3_s{s}"].topk for s in ("0.75", "0.875", "0.9375")] == [338, 169, 85]


def test_build_token_block_indices_and_mask():
    from longcat_video.models.block_sparse_attention import build_token_block_indices, build_token_pair_mask

    t = build_token_block_indices((8, 4, 4), (4, 4, 4))
    assert (t[:64] == 0).all() and (t[64:] == 1).all()
    m = build_token_pair_mask(torch.tensor([[[[3, 5], [0, 7]]]]), torch.arange(8), 8)
    assert m[0, 0, 0, 3] and m[0, 0, 0, 5] and not m[0, 0, 0, 0]


# ------------------------------------------------------------------ Ulysses on gloo ranks
def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _ulysses_worker(rank, world, port, q):
    import torch.distributed as dist

    from longcat_video.context_parallel import heads_to_seq, seq_to_heads

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        B, H, S, D = 1, 4, 16, 3
        full = torch.arange(B * H * S * D, dtype=torch.float32).reshape(B, H, S, D)
        Sl = S // world
        shard = full[:, :, rank * Sl:(rank + 1) * Sl].clone()
        # q, k, v stacked travel in one collective
        stacked = torch.stack((shard, shard + 1, shard + 2))
        heads = seq_to_heads(stacked)
        Hl = H // world
        ok1 = torch.equal(heads[0], full[:, rank * Hl:(rank + 1) * Hl])
        ok2 = torch.equal(heads[2], full[:, rank * Hl:(rank + 1) * Hl] + 2)
        back = heads_to_seq(heads[1] * 10)
        ok3 = torch.equal(back, (shard + 1) * 10)
        q.put((rank, bool(ok1 and ok2 and ok3)))
    finally:
        dist.destroy_process_group()


def test_ulysses_resharding_gloo_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ulysses_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: True, 1: True}


def _fake_bsa(q, k, v, shape, sparsity=0.9375, chunk_thw=(4, 4, 4), sm_scale=None, *, topk=None, rope=None,
              sm_reserve=0):
    """CPU stand-in for the engine call with the dependencies BSA has: every output token of a head
    needs the whole sequence of that head (reversed k, per-head mean of v)."""
    return q + 10 * k.flip(-2) + 100 * v.mean(dim=-2, keepdim=True)


def _ulysses_pipeline_worker(rank, world, port, q, groups):
    import torch.distributed as dist

    import longcat_video.context_parallel as cp

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cp.bsa_attention = _fake_bsa
        B, H, S, D = 2, 8, 12, 3
        g = torch.Generator().manual_seed(5)
        fq, fk, fv = (torch.randn((B, H, S, D), generator=g) for _ in range(3))
        want = _fake_bsa(fq, fk, fv, (1, 1, S))
        Sl = S // world
        sh = slice(rank * Sl, (rank + 1) * Sl)
        got = cp.ulysses_bsa_attention(fq[:, :, sh].contiguous(), fk[:, :, sh].contiguous(),
                                       fv[:, :, sh].contiguous(), (1, 1, S), head_groups=groups)
        q.put((rank, bool(torch.allclose(got, want[:, :, sh], atol=1e-5))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("groups", [1, 2, 4, 3])
def test_ulysses_head_group_pipeline_gloo_world2(groups):
    """The head-group pipelined exchange (async all-to-alls around each group's call) returns the
    same sequence shards as the unsharded call, for any group count (3 falls back to 2)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ulysses_pipeline_worker, args=(r, 2, port, q, groups)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: True, 1: True}


def test_head_group_choice():
    from longcat_video.context_parallel import _head_groups

    assert _head_groups(32, 2, None) == 2 and _head_groups(32, 4, None) == 2 and _head_groups(32, 8, None) == 4
    assert _head_groups(8, 8, None) == 1
    assert _head_groups(32, 8, 3) == 2  # 32/3 does not split; 2 groups of 16 heads do
    assert _head_groups(24, 8, 2) == 1  # 12 heads per group do not split over 8 ranks


def test_kv_cache_continuation_matches_full_forward():
    """attention.py:235-275: continuing from the cached (k, v) of the conditioning frames gives the noise rows
    of the one-shot cond + noise forward (same RoPE positions, same dense attention), also when a batch-1
    cache is broadcast to batch 2."""
    from longcat_video.models.attention import Attention

    torch.manual_seed(0)
    attn = Attention(64, 2).float()
    T, Hl, Wl, ncl = 4, 2, 3, 2
    nc = ncl * Hl * Wl
    x = torch.randn(2, T * Hl * Wl, 64)
    x[1, :nc] = x[0, :nc]  # one conditioning clip for both batch rows
    with torch.no_grad():
        full = attn(x, (T, Hl, Wl), num_cond_latents=ncl)
        for cache_batch in (2, 1):
            out_c, kv = attn(x[:cache_batch, :nc], (ncl, Hl, Wl), return_kv=True)
            assert out_c.shape == (cache_batch, nc, 64) and kv[0].shape == (cache_batch, 2, nc, 32)
            cont = attn.forward_with_kv_cache(x[:, nc:], (T - ncl, Hl, Wl), ncl, kv)
            torch.testing.assert_close(cont, full[:, nc:], rtol=1e-5, atol=1e-6)


def test_kv_cache_continuation_without_cond_skips_rope():
    """Without conditioning latents the continuation attends the fresh queries to cache + fresh keys with no
    RoPE, as the reference does (attention.py:266-268)."""
    import torch.nn.functional as F
    from longcat_video.models.attention import Attention

    torch.manual_seed(1)
    attn = Attention(32, 2).float()
    x_prev, x = torch.randn(1, 6, 32), torch.randn(1, 4, 32)
    with torch.no_grad():
        _, kv = attn(x_prev, (1, 2, 3), return_kv=True)
        got = attn.forward_with_kv_cache(x, (1, 2, 2), 0, kv)
        qkv = attn.qkv(x).reshape(1, 4, 3, 2, 16).permute(2, 0, 3, 1, 4)
        q, k, v = attn.q_norm(qkv[0]), attn.k_norm(qkv[1]), qkv[2]
        o = F.scaled_dot_product_attention(q, torch.cat([kv[0], k], 2), torch.cat([kv[1], v], 2), scale=attn.scale)
        want = attn.proj(o.transpose(1, 2).reshape(1, 4, 32))
    torch.testing.assert_close(got, want)


def test_batched_dit_views_are_merged_before_the_kernel():
    """The attention kernel's TMA map merges batch and heads (stride(0) == H * stride(1)).  The DiT's
    qkv.reshape(B, N, 3, H, D).permute(2, 0, 3, 1, 4) views break that at B > 1 and are copied once;
    B = 1 views and mergeable tensors are used in place (no copy)."""
    from longcat_video import _native

    B, N, H, D = 2, 128, 4, 32
    qkv = torch.randn(B, N, 3, H, D).permute(2, 0, 3, 1, 4)
    q = qkv[0]
    m = _native._merge_batch(q)
    assert m.stride(0) == H * m.stride(1) and torch.equal(m, q) and m.data_ptr() != q.data_ptr()
    q1 = torch.randn(1, N, 3, H, D).permute(2, 0, 3, 1, 4)[0]
    assert _native._merge_batch(q1) is q1
    c = torch.randn(B, H, N, D)
    assert _native._merge_batch(c) is c
    heads_view = torch.randn(B, 2 * H, N, D)[:, :H]  # a head slice keeps stride(0) = 2H * stride(1)
    assert _native._merge_batch(heads_view).stride(0) == H * heads_view.stride(1)


# ------------------------------------------------------------------ the hook's dense fallback
def _hook_attn(monkeypatch, exc):
    from longcat_video.models import attention as attn_mod

    def fake_bsa(*_a, **_k):
        raise exc

    monkeypatch.setattr(attn_mod, "bsa_attention", fake_bsa)
    torch.manual_seed(0)
    a = attn_mod.Attention(64, 2)
    a.enable_bsa = True
    return a


def test_hook_falls_back_to_dense_only_on_shape_errors(monkeypatch):
    from longcat_video._native import BSAShapeError

    a = _hook_attn(monkeypatch, BSAShapeError("Latent shape (4, 4, 6) must be a multiple of chunk_thw (4, 4, 4)"))
    q, k, v = (torch.randn(1, 2, 96, 32) for _ in range(3))
    out = a._process_attn(q, k, v, shape=(4, 4, 6))
    assert torch.allclose(out, torch.nn.functional.scaled_dot_product_attention(q, k, v, scale=a.scale))


@pytest.mark.parametrize("exc", [ValueError("head_dim D=136 must be a multiple of 8 in [8, 128]"),
                                 RuntimeError("bsa_forward failed (code 5)")])
def test_hook_does_not_swallow_engine_errors(monkeypatch, exc):
    a = _hook_attn(monkeypatch, exc)
    q, k, v = (torch.randn(1, 2, 64, 32) for _ in range(3))
    with pytest.raises(type(exc)):
        a._process_attn(q, k, v, shape=(4, 4, 4))


def test_real_shape_error_reaches_dense_path():
    """Through the real engine module: the divisibility check runs on the host before any device work,
    so on a machine without a GPU the hook still lands on dense attention (attention.py:174-179)."""
    from longcat_video.models.attention import Attention

    torch.manual_seed(0)
    a = Attention(64, 2)
    a.enable_bsa = True
    q, k, v = (torch.randn(1, 2, 96, 32) for _ in range(3))
    out = a._process_attn(q, k, v, shape=(4, 4, 6))
    assert torch.allclose(out, torch.nn.functional.scaled_dot_product_attention(q, k, v, scale=a.scale))


def test_unreadable_views_are_copied_not_refused():
    from longcat_video import _native

    base = torch.zeros(2 * 3 * 64 * 128 + 1, dtype=torch.bfloat16)
    off = base[1:].view(2, 3, 64, 128)  # base address 2 bytes past a 16-byte boundary
    assert _native._misaligned(off)
    fixed = _native._merge_batch(off)
    assert fixed.is_contiguous() and not _native._misaligned(fixed) and torch.equal(fixed, off)
    assert _native._aligned(off).is_contiguous()
    ok = torch.zeros(2, 3, 64, 128, dtype=torch.bfloat16)
    assert _native._merge_batch(ok) is ok and _native._aligned(ok) is ok
    # DiT view at B > 1: aligned, but batch and head strides do not merge -> copied for attention only
    qkv = torch.zeros(2, 64, 3, 3, 128, dtype=torch.bfloat16).permute(2, 0, 3, 1, 4)
    q = qkv[0]
    assert _native._aligned(q) is q
    assert _native._merge_batch(q) is not q


# ------------------------------------------------------------------ the copy-engine exchange's copy plan
def _apply_copy_3d(arena, row):
    dst, dpitch, dslice, src, spitch, sslice, width, height, depth = row
    # the extents bsa_copy_3d accepts (bsa_xfer.cu): pitches hold a row, slice pitches whole rows of a slice
    assert 0 < width <= min(dpitch, spitch) and height > 0 and depth > 0
    if depth > 1:
        assert dslice % dpitch == 0 and sslice % spitch == 0
        assert dslice >= dpitch * height and sslice >= spitch * height
    for z in range(depth):
        for y in range(height):
            d0, s0 = dst + z * dslice + y * dpitch, src + z * sslice + y * spitch
            arena[d0:d0 + width] = arena[s0:s0 + width].copy()


@pytest.mark.parametrize("P,B,H,G,nin", [(2, 1, 8, 4, 1), (2, 2, 8, 2, 2), (4, 1, 8, 2, 1), (4, 2, 16, 4, 3),
                                         (8, 1, 32, 4, 1), (2, 1, 4, 1, 1)])
def test_exchange_copy_plan_moves_every_piece(P, B, H, G, nin):
    """``exchange_copy_plan`` (the copies of PeerExchange) restated on one byte arena per rank set: after the
    pulls of every head group each rank's input slot holds the whole sequence of its heads of the group, and
    after the pushes every rank's out_recv holds its token range of every head, as seq_to_heads /
    heads_to_seq define them."""
    from longcat_video.context_parallel import exchange_copy_plan

    Sl, D, elt = 3, 4, 2
    S, Hg = Sl * P, H // G
    Hl = Hg // P
    # one arena: per rank a stage [3,B,H,Sl,D], an out_recv [B,H,Sl,D], two input slots, two output slots
    sizes = [3 * B * H * Sl * D, B * H * Sl * D] + [3 * B * Hl * S * D] * 2 + [B * Hl * S * D] * 2
    base, offs = 0, []
    for r in range(P):
        o = []
        for n in sizes:
            o.append(base)
            base += n * elt
        offs.append(o)
    arena = np.zeros(base, dtype=np.uint8)
    view = lambda off, shape: arena[off:off + int(np.prod(shape)) * elt].view(np.uint16).reshape(shape)
    rng = np.random.default_rng(P * 100 + H)
    full = rng.integers(1, 60000, size=(3, B, H, S, D), dtype=np.uint16)  # q/k/v of the whole sequence
    for r in range(P):
        view(offs[r][0], (3, B, H, Sl, D))[...] = full[:, :, :, r * Sl:(r + 1) * Sl]
    plans = [exchange_copy_plan(P, r, B, H, Sl, D, elt, G, [offs[p][0] for p in range(P)],
                                [offs[p][1] for p in range(P)], offs[r][2:4], offs[r][4:6], nin, nin)
             for r in range(P)]
    out_full = rng.integers(1, 60000, size=(B, H, S, D), dtype=np.uint16)  # what attention would return
    for g in range(G):
        sl = g % 2
        for r in range(P):
            for stream in plans[r][0][g]:
                for row in stream:
                    _apply_copy_3d(arena, row)
            heads = [g * Hg + r * Hl + j for j in range(Hl)]
            got = view(offs[r][2 + sl], (3, B, Hl, S, D))
            assert np.array_equal(got, full[:, :, heads]), (g, r)
            view(offs[r][4 + sl], (B, Hl, S, D))[...] = out_full[:, heads]
        for r in range(P):
            for stream in plans[r][1][g]:
                for row in stream:
                    _apply_copy_3d(arena, row)
    for r in range(P):
        assert np.array_equal(view(offs[r][1], (B, H, Sl, D)), out_full[:, :, r * Sl:(r + 1) * Sl]), r
