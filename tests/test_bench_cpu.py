"""bench.py's output contract, on the CPU: the reference arm prints one JSON line with the
keys the driver reads (the GPU arm is exercised on a B200)."""
import json
import os
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_the_contract_line():
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--steps", "2",
                        "--warmup", "1", "--cpu-budget-s", "1"], capture_output=True, text=True, timeout=600,
                       cwd=REPO)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    j = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in j, key
    assert j["impl"] == "reference" and j["value"] > 0 and j["higher_is_better"] is True
    assert j["cpu_baseline"]["kind"] == "port" and j["cpu_baseline"]["cores"] >= 1
    assert j["e2e"]["h2d_bytes_per_step"] == 0 and j["e2e"]["d2h_bytes_per_step"] == 0
    assert "workload" in j["config"]
    # the same --steps / --warmup and the same config object as the GPU arm prints
    assert j["steps"] == 2 and j["warmup"] == 1
    sys.path.insert(0, REPO)
    import bench
    ns = type("A", (), {"config": "decode", "l2": "none", "ep_layout": "auto", "ep_transport": "auto"})()
    assert j["config"] == bench.workload_config(ns, 1)
    for key in ("T", "E", "hidden", "intermediate", "top_k"):
        assert key in j["config"], key


def test_configs_cover_the_baseline_configs():
    sys.path.insert(0, REPO)
    import bench
    assert set(bench.CONFIGS) == {"decode", "prefill", "stack", "zipf"}
    T, E, H, I, k, _, _ = bench.CONFIGS["decode"]
    assert (T, E, H, I, k) == (32, 32, 2880, 2880, 4)


def test_algorithmic_bytes_follow_the_per_unit_figures():
    # one touched expert costs 13,253,760 B per layer step (unpadded K: gate_up 8,294,400 +
    # scales 518,400 + fp32 bias 23,040; down 4,147,200 + 259,200 + 11,520); the router weight
    # and bias scale with E; the decode config moves 425,813,824 B per step, 32 experts touched
    sys.path.insert(0, REPO)
    import bench
    _, _, full, touched = bench.alg_bytes([1] * 32, 32, 4, 2880, 2880, 32)
    assert touched == 32 and full == 425_813_824
    assert full - bench.alg_bytes([1] * 31 + [0], 32, 4, 2880, 2880, 32)[2] == 13_253_760
    assert bench.alg_bytes([1] * 32 + [0] * 96, 32, 4, 2880, 2880, 128)[2] - full == 96 * (2880 * 2 + 2)
