"""bench.py's performance gate: figures compared with recorded floors (host logic only)."""
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

import bench  # noqa: E402


def test_gate_passes_and_fails_at_the_ratio(tmp_path):
    floor = tmp_path / "floor.json"
    floor.write_text(json.dumps({"ratio": 0.9, "floors": {"value_tops": 2800.0, "tops_8192x3072x3072": 2500.0,
                                                          "gbs_rms_mod_quant_fp8_e4m3": 5200.0,
                                                          "not_measured_here": 1.0}}))
    extras = {"per_shape_tops": {"8192x3072x3072": 2300.0},
              "row_kernels": {"rms_mod_quant_fp8_e4m3": {"gbs": 4700.0}}}
    g = bench.perf_gate(2600.0, extras, str(floor))
    assert g["ok"] and set(g["checks"]) == {"value_tops", "tops_8192x3072x3072", "gbs_rms_mod_quant_fp8_e4m3"}
    g = bench.perf_gate(2500.0, extras, str(floor))            # 2500 < 0.9 * 2800
    assert not g["ok"] and not g["checks"]["value_tops"]["ok"] and g["checks"]["tops_8192x3072x3072"]["ok"]


def test_gate_without_floor_file(tmp_path):
    assert bench.perf_gate(1.0, {}, str(tmp_path / "missing.json")) is None


def test_committed_floor_file_is_well_formed():
    with open(bench.PERF_FLOOR) as f:
        spec = json.load(f)
    assert 0.5 < spec["ratio"] <= 1.0 and spec["floors"] and all(v > 0 for v in spec["floors"].values())
