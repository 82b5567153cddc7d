"""bench.py pieces that need no GPU: the reference arm's JSON line (the reference's own
CPU forward pass, Model::forward, on a reduced-layer copy of the workload) and the
helpers that feed the roofline fields."""
import json
import os
import subprocess
import sys

import pytest

from conftest import ROOT, load_package

sys.path.insert(0, ROOT)
import bench  # noqa: E402

load_package()  # registers inference_cpp_b200 for the imports below


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                        "--steps", "1", "--warmup", "3"],
                       capture_output=True, text=True, timeout=600, cwd=ROOT,
                       env={k: v for k, v in os.environ.items()
                            if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")})
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["metric"] == bench.METRIC
    assert d["unit"] == "tok/s" and d["higher_is_better"] is True and d["value"] > 0
    assert d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] >= 3
    assert d["config"]["workload"] == "llama-3-8b-decode"
    # the sampled steps fit in the run: ms_per_step is one sampled token
    assert d["ms_per_step"] * d["steps"] / 1e3 <= d["wall_s"]
    assert d["extrapolated_ms_per_token"] >= d["ms_per_step"]
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] == 1 and cb["value"] == d["value"]
    assert "2-layer copy" in cb["sample"] and "extrapolated to 32 layers" in cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_roofline_helpers():
    peak, kind = bench.measured_peaks()
    tpeak, tkind = bench.measured_tensor_peak()
    if kind == "fallback":
        assert peak == 6650.0
    if tkind == "fallback":
        assert tpeak == 1590.0
    assert peak > 1000 and tpeak > 100
    # the committed capture of the roofline shape gives its DRAM bytes; others give None
    t = bench.traffic_from_profile(14336, 4096)
    assert t is not None and 30e6 < t < 40e6
    assert bench.traffic_from_profile(123, 456) is None


def test_cpu_forward_sample_extrapolates_from_measured_layers(ib):
    from inference_cpp_b200 import gguf_writer as gw
    r = bench.cpu_forward_sample(ib, gw.CONFIGS["tinyllama-1.1b"], 1)
    assert r["sample_layers"] == 2 and len(r["sample_s"]) == 1
    assert r["t_head_s"] > 0 and r["t_layer_s"] > 0
    assert abs(r["per_token_s"] - (r["t_head_s"] + 22 * r["t_layer_s"])) < 1e-9
    # the whole model when it has no more layers than the sample
    s = bench.cpu_forward_sample(ib, gw.CONFIGS["stories15M"], 1, layers=6)
    assert s["sample_layers"] == 6 and s["per_token_s"] == s["sample_s"][0]
    with pytest.raises(bench.CpuBaselineUnavailable, match="stack arrays"):
        bench.cpu_forward_sample(ib, gw.CONFIGS["llama-3-70b"], 1)


def test_metric_follows_the_workload():
    from inference_cpp_b200 import gguf_writer as gw
    assert bench.metric_for(gw.CONFIGS["llama-3-8b"]) == bench.METRIC
    assert "Llama-3-70B-shape" in bench.metric_for(gw.CONFIGS["llama-3-70b"])
    assert "stories15M-shape Q4_0" in bench.metric_for(gw.CONFIGS["stories15M"])


def test_clock_records_that_force_a_remeasurement():
    ok = {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": []}
    assert not bench.clocks_rejected(ok)
    # the power cap alone is normal under load
    assert not bench.clocks_rejected({"sm_mhz": 1300.0, "sm_max_mhz": 1965.0,
                                      "reasons": ["sw_power_cap"]})
    for r in ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown"):
        assert bench.clocks_rejected(dict(ok, reasons=[r]))
    # clocks well below their maximum with no reason: a lock left by someone else
    assert bench.clocks_rejected({"sm_mhz": 1200.0, "sm_max_mhz": 1965.0, "reasons": []})
    # no samples: nothing to reject on
    assert not bench.clocks_rejected({"sm_mhz": None, "sm_max_mhz": None,
                                      "reasons": ["nvidia-smi unavailable"]})
