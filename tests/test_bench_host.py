"""CPU: the arithmetic behind bench.py's JSON line.

Algorithmic bytes per format (the roofline numerators), unit conversions and
the roofline fraction, the arithmetic label of each path, the measured peaks
read from MEASURED_PEAKS.json, the ncu traffic figures' profile summaries, and
the clock/throttle summary computed from NVML samples (a fake sampler here:
the logic that decides which throttle reasons a run reports).
"""
import json
import os
import re

import pytest

import bench

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_weight_bytes_per_format():
    wl = bench.WORKLOADS
    assert bench.weight_bytes(wl["decode"]) == 4096 * 4096
    # codes + one f32 scale per 128-code group
    assert bench.weight_bytes(wl["grouped_decode"]) == 4096 * 4096 + 4 * 4096 * 32
    # packed nibbles + f32 scale and zero point per group
    assert bench.weight_bytes(wl["int4_decode"]) == 4096 * 4096 // 2 + 8 * 4096 * 32 == 9437184
    # gate and up matrices of the MLP front
    assert bench.weight_bytes(wl["mlp_decode"]) == 2 * 11008 * 4096


def test_throughput_and_roofline_units():
    peaks = {"hbm": 6500.0, "tc": 1600.0, "source": "measured"}
    dec = bench.WORKLOADS["decode"]
    ms = 0.005  # 5 us
    gbs = bench.throughput(dec, ms)
    assert gbs == pytest.approx(4096 * 4096 / 5e-6 / 1e9)
    r = bench.roofline(dec, ms, peaks, "decode")
    assert r["unit"] == "GB/s" and r["bound"] == "hbm"
    assert r["frac"] == pytest.approx(gbs / 6500.0, abs=1e-4)
    assert r["traffic"] == bench.NCU_TRAFFIC["decode"]
    pf = bench.WORKLOADS["prefill"]
    tf = bench.throughput(pf, 0.065)
    assert tf == pytest.approx(2 * 2048 * 4096 * 4096 / 65e-6 / 1e12)
    r = bench.roofline(pf, 0.065, peaks, "prefill")
    assert r["unit"] == "TFLOP/s" and r["frac"] == pytest.approx(tf / 1600.0, abs=1e-4)


def test_traffic_is_close_to_the_algorithmic_bytes():
    # DRAM traffic per launch well above the algorithmic bytes would mean
    # re-reads; each recorded figure stays within 5 % above them (the fused
    # MLP capture counts 3.5 MB of DRAM writes against the kernel's 44 KB of
    # stores; its reads are the weights to within 0.2 %).
    for name, traffic in bench.NCU_TRAFFIC.items():
        wl = bench.WORKLOADS[name]
        if wl["unit"] != "GB/s":
            continue
        algo = bench.weight_bytes(wl)
        assert algo <= traffic <= 1.05 * algo, name


def test_traffic_figures_name_existing_profiles():
    src = open(os.path.join(ROOT, "bench.py")).read()
    block = src[src.index("NCU_TRAFFIC = {"):]
    block = block[:block.index("}")]
    named = re.findall(r"profiles/([\w.]+\.md)", block)
    assert len(named) == len(bench.NCU_TRAFFIC)
    for f in named:
        assert os.path.isfile(os.path.join(ROOT, "profiles", f)), f


def test_compute_dtype_routes():
    # M = 1 per channel: fixed-point activations times int8 codes on dp2a.
    assert bench.compute_dtype("simt_f32", 1, 4096, False) == "s30 fixed-point x s8 (dp2a) -> s32/f32"
    assert bench.compute_dtype("simt_f32 (staged rows, mma.sync s8)", 1, 4096, False).endswith("(mma.sync) -> s32/f64")
    assert bench.staged_mma(4096, 4096, 148) and bench.staged_mma(1024, 8192, 148)
    assert not bench.staged_mma(4096, 4500, 148)  # 31 rows x 4112 B > 115,648 B
    assert not bench.staged_mma(11008, 4096, 148) and not bench.staged_mma(4096, 12288, 148)
    assert not bench.staged_mma(3072, 8192, 148)  # 4 row groups x 6 k-steps > 20 MMAs per warp
    assert bench.staged_mma_grouped(4096, 4096, 128, 148) and bench.staged_mma_grouped(1024, 8192, 32, 148)
    assert not bench.staged_mma_grouped(4096, 4096, 64, 148)  # four scale flushes per warp: slower
    assert not bench.staged_mma_grouped(2048, 6000, 32, 148)  # 32 scales per lane
    assert bench.compute_dtype("grouped_f32 (group 128, staged rows, mma.sync s8)", 1, 4096, True).endswith("f64")
    assert bench.staged_mma_i4(4096, 4096, 128, 148) and bench.staged_mma_i4(1024, 8192, 64, 148)
    assert not bench.staged_mma_i4(4096, 4096, 64, 148) and not bench.staged_mma_i4(4096, 4096, 4096, 148)
    assert "u4" in bench.compute_dtype("int4 (group 128, staged rows, mma.sync u8)", 1, 4096, True)
    assert bench.compute_dtype("simt_f32", 2, 4096, False) == "f32"
    assert bench.compute_dtype("simt_f32", 1, 4096, True) == "f32"
    assert bench.compute_dtype("tensor_f16", 32, 4096, False).startswith("s8")
    assert bench.compute_dtype("tensor_f16", 128, 65536, False).startswith("s8")
    assert bench.compute_dtype("tensor_f16", 129, 4096, False) == "f16xf16->f32"
    assert bench.compute_dtype("tensor_f16", 32, 4096, True) == "f16xf16->f32"


def test_quantize_and_dequantize_bytes():
    # 5*N*K + 4*N for the quantizer; N*K + 4*N + 4*N*K (f32 out) for the dequantizer.
    assert bench.weight_bytes(bench.WORKLOADS["quantize"]) == 5 * 4096 * 4096 + 4 * 4096
    assert bench.weight_bytes(bench.WORKLOADS["dequantize"]) == 4096 * 4096 + 4 * 4096 + 4 * 4096 * 4096
    assert bench.weight_bytes(dict(bench.WORKLOADS["dequantize"], out_bytes=2)) == 4096 * 4096 * 3 + 4 * 4096


def test_measured_peaks_read_from_file():
    peaks = bench.measured_peaks()
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if not os.path.exists(path):
        assert peaks["source"] == "fallback"
        return
    d = json.load(open(path))
    assert peaks["source"] == "measured"
    assert peaks["hbm"] == pytest.approx(float(d["hbm_gbs"]))
    assert peaks["tc"] == pytest.approx(float(d["bf16_tflops"]))


def _fake_sampler(samples, max_mhz=1965):
    s = bench.ClockSampler.__new__(bench.ClockSampler)
    s.samples = samples
    s.ok = True
    s.max_mhz = max_mhz
    return s


def test_clock_summary_reports_reasons_under_load():
    R = bench.ClockSampler.REASONS
    samples = [
        (0.0, 345, R["gpu_idle"]),                     # idle before the run: ignored
        (1.0, 1965, 0),
        (2.0, 1950, R["sw_power_cap"]),               # kept and noted
        (3.0, 1965, 0),
        (4.0, 1200, R["hw_slowdown"]),                # a slowdown the driver rejects
        (9.0, 1965, 0),                                # outside the window
    ]
    out = _fake_sampler(samples).summary(0.0, 5.0, 1.5, 4.5)
    assert out["sm_mhz"] == 1957.5  # median of the four loaded samples in the window
    assert set(out["reasons"]) == {"sw_power_cap", "hw_slowdown"}
    assert out["samples"] == 4 and out["samples_in_timed_region"] == 3
    assert out["sm_max_mhz"] == 1965


def test_clock_summary_without_nvml():
    s = bench.ClockSampler.__new__(bench.ClockSampler)
    s.ok = False
    out = s.summary(0, 1, 0, 1)
    assert out["sm_mhz"] is None and out["reasons"] == ["nvml unavailable"]


def test_cpu_baseline_runs_on_host_tensors():
    # The CPU baseline leg on a small case: popcorn's own loop (or the oracle
    # port) on all threads and on one core, reported in the workload's unit.
    import types

    import numpy as np
    import torch

    import oracle

    M, N, K = 1, 256, 512
    x = torch.from_numpy(oracle.fill_normal(M * K, 0, 1.0).reshape(M, K))
    q, s = oracle.quantize(oracle.fill_normal(N * K, 1, 0.02).reshape(N, K))
    setup = types.SimpleNamespace(x=[x], q=[torch.from_numpy(q)], s=[torch.from_numpy(s)])
    wl = dict(M=M, K=K, N=N, unit="GB/s", bound="hbm")
    out = bench.cpu_baseline(torch, setup, wl)
    assert out["unit"] == "GB/s" and out["value"] > 0 and out["cores"] >= 1
    assert out["kind"] == ("reference" if oracle.have_ref_loops() else "port")
    assert out["single_core"]["cores"] == 1 and out["single_core"]["value"] > 0
    assert np.isfinite(out["value"]) and np.isfinite(out["single_core"]["value"])
