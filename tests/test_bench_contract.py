"""bench.py contract on the CPU: the reference arm (the oracle timed on the host cores) prints one JSON
line with the keys the driver reads; the GPU arm is exercised by the GPU runs."""
import json
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)


def test_reference_arm_prints_contract_line():
    cmd = [sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "3",
           "--ref-qblocks", "4"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, cwd=REPO)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e", "gpu_launches"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["config"]["workload"] == "config2"


def test_gather_roofline_bytes():
    """The attention gather roofline counts one 64-token K and V tile pair per (q-block, selected kv-block);
    fp32 configs run their attention in fp16."""
    sys.path.insert(0, REPO)
    sys.path.insert(0, os.path.join(REPO, "longcat-video-mlx_b200"))
    import bench
    from longcat_video.workloads import CONFIGS

    c2 = CONFIGS["config2"]
    assert bench.attn_gather_bytes(c2) == 32 * 1350 * 85 * 2 * 64 * 128 * 2
    assert bench.attn_gather_bytes(c2, 4) == bench.attn_gather_bytes(c2) / 4
    c1 = CONFIGS["config1"]
    assert bench.attn_gather_bytes(c1) == c1.B * c1.H * (c1.S // 64) * c1.topk * 2 * 64 * c1.D * 2
