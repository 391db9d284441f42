"""bench.py's reporting helpers on the CPU: DRAM traffic looked up from the committed ncu
captures and scaled to a launch, the nominal-peak fractions added to every HBM roofline,
and the host record that goes with the CPU baselines."""
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(REPO))

import bench  # noqa: E402


def test_traffic_lines_scale_to_the_jobs_of_a_launch():
    full = bench.profiled_traffic("restore_rows", "C2_restore_T32768_H8_D128_byte", 32)
    half = bench.profiled_traffic("restore_rows", "C2_restore_T32768_H8_D128_byte", 16)
    assert full is not None and full > 8 * 10**9  # 4 GiB read + ~4 GiB written for 32 layers
    assert abs(half - full / 2) <= 1
    # the quantized kernels: steady-state traffic of a one-layer launch, close to its
    # algorithmic bytes (KIVI: 155,631,616; CacheGen: 172,097,536)
    kivi = bench.profiled_traffic("kivi2_to_cache", "KIVI_layer_T32768_H8_D128_b2_g64", 1)
    cg = bench.profiled_traffic("cachegen_staged", "CG_layer_T32768_H8_D128_k5_v4", 1)
    assert 0.95 < kivi / 155_631_616 < 1.05
    assert 0.95 < cg / 172_097_536 < 1.05
    assert bench.profiled_traffic("no_such_kernel", "C2_restore_T32768_H8_D128_byte", 1) is None


def test_every_hbm_roofline_gets_its_nominal_fraction():
    line = {"roofline": {"unit": "GB/s", "achieved": 4000.0},
            "pack": {"roofline": {"unit": "GB/s", "achieved": 6000.0}},
            "attn": {"roofline": {"unit": "TFLOP/s", "achieved": 100.0}}}
    out = bench.with_nominal(line)
    assert out["roofline"]["nominal_peak"] == bench.NOMINAL_HBM_GBS
    assert out["roofline"]["nominal_frac"] == round(4000.0 / bench.NOMINAL_HBM_GBS, 4)
    assert out["pack"]["roofline"]["nominal_frac"] == round(6000.0 / bench.NOMINAL_HBM_GBS, 4)
    assert "nominal_frac" not in out["attn"]["roofline"]


def test_host_record_and_measured_peak():
    host = bench.host_cpu()
    assert isinstance(host["nproc"], int) and host["nproc"] >= 1
    assert host["numa_nodes"] is None or host["numa_nodes"] >= 1
    peak, kind = bench.measured_hbm_peak()
    assert kind in ("measured", "fallback") and peak > 1000
