"""bench.py's reference arm runs on the CPU; its JSON line must carry the
keys the benchmark contract names (checked here on a one-step run)."""
import json
import os
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_json_line():
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "0"], capture_output=True, text=True, timeout=600, cwd=REPO)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["value"] > 0 and d["unit"] == "TFLOP/s"
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert "workload" in d["config"]


def test_bench_help():
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--help"], capture_output=True, text=True,
                       timeout=120, cwd=REPO)
    assert r.returncode == 0 and "--gpus" in r.stdout and "--impl" in r.stdout


def test_peak_choice_follows_the_observed_power_state():
    import bench

    P = {"bf16_tflops": 1600.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6500.0}
    capped = {"sm_mhz": 1200.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"]}
    free = {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": []}
    low_no_reason = {"sm_mhz": 1300.0, "sm_max_mhz": 1965.0, "reasons": []}
    assert bench.pick_peak(P, capped)[0] == 1400.0
    assert bench.pick_peak(P, free)[0] == 1600.0
    assert bench.pick_peak(P, low_no_reason)[0] == 1400.0   # clocks well below max: not the burst state
    assert bench.pick_peak(P, free, div=2.0)[0] == 800.0     # tf32 rate
    assert bench.pick_peak(P, None)[0] == 1400.0


def test_rotating_input_sets_exceed_three_l2():
    import torch

    import bench
    from cmp_ext_b200.workloads import Config

    small = Config(99, "tiny", torch.float16, 64, 64, 64, "normal", 1.0, "tensor")
    sets, desc = bench.input_sets(small, "cpu", 64, 0)
    assert len(sets) == 16 and "rotated" in desc  # capped at 16 sets
    assert not torch.equal(sets[0][0], sets[1][0])  # different A per set
    one, _ = bench.input_sets(Config(98, "big", torch.float16, 4096, 4096, 4096, "normal", 1.0, "tensor"), "cpu",
                              4096, 0)
    assert len(one) == 4  # 100.7 MB per set: 4 sets exceed 3 x 126 MB
