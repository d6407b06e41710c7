"""CPU tests of bench.py's bookkeeping: the FLOP convention (fwd 4BHS^2D,
bwd 2.5x fwd, causal halves both), the traffic scaling of the dominant
kernel's ncu capture, the defaults the driver relies on (N=1, K/W that end in
minutes, 20 pipelined end-to-end steps), and the config line."""
import sys

import pytest

import bench


def _args(*argv):
    old = sys.argv
    sys.argv = ["bench.py", *argv]
    try:
        return bench.parse()
    finally:
        sys.argv = old


def test_flop_convention():
    B, H, S, D = 4, 32, 8192, 128
    assert bench.attn_flops(B, H, S, D, causal=False) == 14.0 * B * H * S * S * D
    assert bench.attn_flops(B, H, S, D, causal=True) == pytest.approx(7.697e12, rel=1e-3)


def test_traffic_scales_with_heads_only_for_the_captured_shape():
    full = bench.traffic_per_launch("bwd", 4, 32, 8192, 128)
    assert full == pytest.approx(bench.DOMINANT_KERNEL_TRAFFIC_BYTES)
    assert bench.traffic_per_launch("bwd", 4, 4, 8192, 128) == pytest.approx(full / 8)  # 8 GPUs: 4 heads each
    assert bench.traffic_per_launch("bwd", 4, 32, 4096, 128) is None  # another S: not captured
    assert bench.traffic_per_launch("fwd", 4, 32, 8192, 128) is None


def test_defaults_match_the_driver_contract():
    a = _args()
    assert (a.gpus, a.impl, a.workload) == (1, "haelixe", "attention")
    assert a.warmup >= 3 and a.steps >= 1
    assert (a.batch, a.heads, a.seq, a.head_dim, a.rope_theta) == (4, 32, 8192, 128, 500000.0)
    assert not a.no_causal and a.e2e_steps == 20


def test_config_names_the_workload_and_the_l2_rule():
    a = _args()
    cfg = bench.config_of(a, 1)
    assert cfg["workload"].startswith("attention layer core B4 H32 S8192 D128 causal")
    assert "larger than L2" in cfg["l2"]  # each operand 268 MB > 126 MB
    assert bench.config_of(a, 8)["parallelism"].startswith("heads/8 per GPU")
    small = bench.config_of(_args("--seq", "1024", "--heads", "2"), 1)
    assert "smaller than L2" in small["l2"]


def test_peak_rule_burst_for_short_regions_sustained_for_long():
    peaks = {"bf16_tflops": 1643.5, "bf16_tflops_sustained": 1348.1}
    p, src = bench.choose_peak(peaks, 0.083)  # ten 8.3 ms steps
    assert p == 1643.5 and "burst" in src
    p, src = bench.choose_peak(peaks, 5.0)
    assert p == 1348.1 and "sustained" in src
    p, src = bench.choose_peak(None, 0.1)
    assert p == bench.FALLBACK_PEAK_TFLOPS and "fallback" in src
