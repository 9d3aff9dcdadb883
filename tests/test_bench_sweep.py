"""Host logic of bench.py: the isolated sweep's lower bounds and the traffic field."""
from __future__ import annotations

import importlib.util
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PEAKS = {"hbm_gbs": 6452.2, "bf16_tflops": 1661.6}


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_mod", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def int4_bytes(k: int, n: int) -> float:
    return k * n / 2 + (k // 128) * n * 4


def test_decode_is_hbm_bound(bench):
    b = bench.sweep_bounds("int4-g128", 1, 14336, 4096, 1, int4_bytes(14336, 4096), PEAKS)
    assert b["bound"] == "hbm" and b["nvlink_bytes"] == 0
    assert b["t_min_us"] == pytest.approx(b["hbm_bytes"] / (PEAKS["hbm_gbs"] * 1e3))


def test_large_m_single_gpu_is_tensor_bound(bench):
    b = bench.sweep_bounds("int8", 16384, 28672, 8192, 1, 28672 * 8192 + 4 * 28672, PEAKS)
    assert b["bound"] == "tensor"
    assert b["flops"] == 2.0 * 16384 * 28672 * 8192


def test_large_m_at_tp8_is_nvlink_bound(bench):
    k = 14336 // 8
    b = bench.sweep_bounds("int4-g128", 4096, k, 4096, 8, int4_bytes(k, 4096), PEAKS)
    assert b["bound"] == "nvlink"
    assert b["nvlink_bytes"] == 7 * 4096 * 4096 * 2


def test_traffic_field_comes_from_the_committed_capture(bench):
    """The bench line's roofline.traffic is the gate/up DRAM bytes of the
    committed ncu summary, scaled to a rank's launch by algorithmic bytes."""
    from types import SimpleNamespace

    shape = SimpleNamespace(hidden=4096, intermediate=14336)
    args = SimpleNamespace(scheme="int4-g128", batch=16, model="llama3-8b")
    h, i = shape.hidden, shape.intermediate
    tp1 = (h * 2 * i / 2 + (h // 128) * 2 * i * 4) + 16 * h * 2 + 16 * i * 2
    traffic, src = bench.measured_traffic(args, tp1, shape)
    assert src.endswith("qgemm_tc_int4g128_b16_ncu_full.md")
    # within 1 % of the algorithmic bytes: nothing is fetched twice
    assert abs(traffic - tp1) / tp1 < 0.01
    half, _ = bench.measured_traffic(args, tp1 / 2, shape)
    assert half == pytest.approx(traffic / 2)
    other, why = bench.measured_traffic(SimpleNamespace(scheme="int8", batch=16, model="llama3-8b"),
                                        tp1, shape)
    assert other is None and "no capture" in why


def test_traffic_field_for_the_native_fp8_capture(bench):
    """Llama-3-70B fp8-native at batch 32 reads its gate/up traffic from the
    native kernel's committed capture: within 2 % of the algorithmic bytes
    (the extra is the stream-K partials of shared tiles)."""
    from types import SimpleNamespace

    shape = SimpleNamespace(hidden=8192, intermediate=28672)
    args = SimpleNamespace(scheme="fp8-native", batch=32, model="llama3-70b")
    tp1 = bench.gate_up_tp1_bytes("fp8-native", 32, shape)
    assert tp1 == 472350720
    traffic, src = bench.measured_traffic(args, tp1, shape)
    assert src.endswith("qgemm_tc_fp8native_llama70b_b32_ncu_full.md")
    assert 0 <= (traffic - tp1) / tp1 < 0.02
