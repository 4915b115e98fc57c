"""The B200 roofline model (work_llm_accelerator_b200/performance_model): its byte and FLOP counts against the
figures the reference and the benchmark configurations state, and the roofline arithmetic bench.py uses."""
from __future__ import annotations

import json

import pytest

from work_llm_accelerator_b200 import performance_model as pm


def test_parameter_counts_match_reference_layout():
    p = pm.param_breakdown()
    # the reference estimator's keys and totals (performance_model/estimate_qwen_prefill_decode.py:27-52)
    assert p["attention_per_layer"] == 2 * 1536 * 1536 + 2 * 1536 * 256
    assert p["mlp_per_layer"] == 3 * 1536 * 8960
    assert p["embed_or_lm_head"] == 151936 * 1536
    assert pm.projection_macs_per_token() == 46_792_704
    # the DDR layer image sizes of hls/common/llm_memory_layout.h (W4) and its one-byte twin (W8)
    assert pm.layer_param_bytes(4) == 23_508_992
    assert pm.layer_param_bytes(8) == 46_905_344


def test_config_work_figures():
    # config 1: 2 * 46.79 M * 128 + 4 * 12 * 128 * (128 * 129 / 2) = 12.03 GFLOP
    assert pm.prefill_flops(128, layers=1)["total"] == pytest.approx(12.0297e9, rel=1e-4)
    # config 4, per sequence: 10.73 TFLOP dense + 1.44 TFLOP causal attention
    f = pm.prefill_flops(4096)
    assert f["dense"] == pytest.approx(10.733e12, rel=1e-3)
    assert f["attention"] == pytest.approx(1.4433e12, rel=1e-3)
    # config 2: 1.81 GB per W8 batch-1 step at history 512 (layers + LM head)
    assert pm.decode_step_bytes(8, 512) == pytest.approx(1.8104e9, rel=1e-3)
    # config 3: weights once, 64 sequences' K/V over 2049 rows
    b = pm.decode_step_bytes(8, 2048, 64)
    assert b == pytest.approx(28 * 46_905_344 + 151936 * 1536 * 2 + 1536 * 4 + 64 * 28 * 2050 * 2048, rel=1e-9)
    # config 0: one layer's parameters + 129 rows read + 1 written + in/out activations
    assert pm.decode_layer_bytes(8, 128) == 46_905_344 + 130 * 2048 + 2 * 1536 * 4


def test_roofline_arithmetic(tmp_path):
    peaks_file = tmp_path / "peaks.json"
    peaks_file.write_text(json.dumps({"hbm_gbs": 6000.0, "bf16_tflops": 1500.0, "bf16_tflops_sustained": 1400.0}))
    pk = pm.load_peaks(peaks_file)
    assert pk.source == "measured" and pk.hbm_gbs == 6000.0
    r = pm.roofline(3.0e9, 1e-3, "hbm", pk)
    assert r["achieved"] == pytest.approx(3000.0) and r["frac"] == pytest.approx(0.5) and r["unit"] == "GB/s"
    r = pm.roofline(7.0e12, 10e-3, "tensor", pk, sustained=True)
    assert r["achieved"] == pytest.approx(700.0) and r["frac"] == pytest.approx(0.5)
    fb = pm.load_peaks(tmp_path / "absent.json")
    assert fb.source == "fallback" and fb.hbm_gbs == pm.FALLBACK_HBM_GBS
    # the lower bound is the slower of the byte stream and the FLOPs
    assert pm.lower_bound_seconds(6.0e9, 0.0, pk) == pytest.approx(1e-3)
    assert pm.lower_bound_seconds(0.0, 1.5e12, pk) == pytest.approx(1e-3)


def test_reports_classify_bounds():
    rep = pm.baseline_configs_report(8)
    assert rep["config2_decode_bs1_hist512"]["bound"] == "hbm"
    assert rep["config3_decode_bs64_hist2048"]["bound"] == "hbm"
    assert rep["config4_prefill_4096"]["bound"] == "tensor"
    assert rep["config2_decode_bs1_hist512"]["max_tok_s"] > 1000


def test_bench_uses_the_model():
    import bench

    for h in (512.0, 1000.5):
        assert bench.step_bytes(8, h) == pm.decode_step_bytes(8, h)
        assert bench.layers_bytes(8, h) == pm.decode_layers_bytes(8, h)
