"""torchrun worker for tests/test_multi_gpu.py: the sequence-parallel BSA call on every rank equals
the single-GPU call on the whole problem (bit for bit: heads are independent and run the same kernels)."""
import os
import sys
from datetime import timedelta

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "longcat-video-mlx_b200"))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main():
    rank, world, local = (int(os.environ[k]) for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=60))
    from longcat_video.context_parallel import close_exchanges, ulysses_bsa_attention
    from longcat_video.models.block_sparse_attention import bsa_attention
    from longcat_video.models.rope_3d import RopeTables

    ok = True
    cases = [(1, 8, (1, 1, 4096), (1, 1, 64), 5, None), (2, 4, (4, 8, 16), (4, 4, 4), 3, None),
             (1, 8, (1, 1, 2048), (1, 1, 64), 4, (4, 8, 64))]
    for B, H, shape, chunk, topk, rope_grid in cases:
        S = shape[0] * shape[1] * shape[2]
        g = torch.Generator(device="cpu").manual_seed(7)
        q, k, v = (torch.randn((B, H, S, 128), generator=g).to(torch.bfloat16).to(dev) for _ in range(3))
        rope = RopeTables(rope_grid, 128, dev) if rope_grid else None
        want = bsa_attention(q, k, v, shape, chunk_thw=chunk, topk=topk, rope=rope)
        Sl = S // world
        sh = slice(rank * Sl, (rank + 1) * Sl)
        qs, ks, vs = (x[:, :, sh].contiguous() for x in (q, k, v))
        # the copy-engine exchange with its default head groups and with one and four groups (other copy plans)
        for exchange, groups in (("copy_engine", None), ("copy_engine", 1), ("copy_engine", 4), ("messages", None)):
            for _ in range(2):  # second call reuses the exchange's buffers
                got = ulysses_bsa_attention(qs, ks, vs, shape, chunk_thw=chunk, topk=topk, rope=rope,
                                            exchange=exchange, head_groups=groups)
                same = torch.equal(got, want[:, :, sh])
                if not same:
                    print(f"rank {rank}: mismatch B={B} H={H} shape={shape} exchange={exchange} groups={groups}",
                          flush=True)
                ok &= same
    close_exchanges()
    flag = torch.tensor([0 if ok else 1], device=dev)
    dist.all_reduce(flag)
    dist.destroy_process_group()
    if rank == 0:
        print("ULYSSES_PARITY_OK" if flag.item() == 0 else "ULYSSES_PARITY_FAIL", flush=True)
    return 0 if flag.item() == 0 else 1


if __name__ == "__main__":
    sys.exit(main())
