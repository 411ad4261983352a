"""CPU: bench.py's reference arm (the oracle port timed on the host cores)
prints one JSON line with the keys the benchmark contract requires."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_json_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["steps"] == 1 and d["warmup"] == 3
    assert d["higher_is_better"] is True and d["config"]["workload"]
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_matches_repo_arm_metric_and_times_its_own_steps():
    """Both arms print the same metric string (so their values divide), and
    the reference arm's ms_per_step is the measured time of one step, so
    steps x ms_per_step is the time the run actually spent stepping."""
    import time
    sys.path.insert(0, ROOT)
    import bench
    t0 = time.perf_counter()
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "4",
                        "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    wall = time.perf_counter() - t0
    assert r.returncode == 0, r.stderr[-2000:]
    d = json.loads([l for l in r.stdout.splitlines() if l.startswith("{")][0])
    assert d["metric"] == bench.METRIC
    assert d["steps"] * d["ms_per_step"] / 1e3 < wall
    src = open(os.path.join(ROOT, "bench.py")).read()
    assert '"metric": METRIC' in src and src.count('"metric": METRIC') == 2


def test_compact_secondary_is_short():
    """The secondary summary stays a few hundred characters with every
    config present (it ends the bench line)."""
    sys.path.insert(0, ROOT)
    import bench
    dec = {"us_per_step": 2514.2345, "GBs": 6833.33, "frac_of_hbm": 1.04231}
    sec = {"decode_128k": dec, "decode_cfg3": dec, "vllm_fog_decode": dec, "decode_f32": dict(dec, cfg1_us=31.23),
           "page_ops": {"gather_b2b_frac": 0.86341, "remap_b2b_frac": 0.7601, "insert_remap_b2b_frac": 0.7891,
                        "cpu_baseline": {"gather_GBs": 3.981, "remap_GBs": 0.9312}},
           "prefill": {"ms": 40.931, "tflops": 846.21, "frac_of_bf16_peak": 0.51101, "cpu_baseline": {"value": 0.2461}},
           "index_query": {"n1000000_topk_frac": 0.98731, "n78125_topk_us": 27.812, "cpu_baseline": {"value": 1292.1}},
           "tiered_cache": {"step_ms": 0.26251, "frac_of_hbm": 0.4691, "speedup_vs_reference_ops": 9.71}}
    c = bench.compact_secondary(sec)
    assert len(json.dumps(c)) < 900
    assert c["decode_128k"] == {"us": 2514, "GBs": 6833, "frac": 1.04}
    assert c["prefill"]["frac"] == 0.511 and c["page_ops_b2b_frac"]["gather"] == 0.863
