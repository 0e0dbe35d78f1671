"""Host-side arithmetic of bench.py (no GPU): the e2e schedule bound and the
configuration records the bench line carries."""
import importlib.util
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def load_bench():
    spec = importlib.util.spec_from_file_location("bench_module", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


bench = load_bench()


def simulate(h2d, d2h, r_in, r_out, steps=4000):
    """Time-stepped pipeline: input arrives at r_in; after a fraction f of it
    arrived, f^2 of the output may leave, at most at r_out."""
    t_in = h2d / r_in
    dt = t_in * 4 / steps
    sent, t = 0.0, 0.0
    while sent < d2h - 1e-9 * d2h:
        t += dt
        f = min(1.0, t / t_in)
        sent = min(d2h * f * f, sent + r_out * dt)
    return t


@pytest.mark.parametrize("h2d,d2h,r_in,r_out", [
    (268e6, 268e6, 50e9, 50e9),      # fp16 8192^3 on one GPU
    (302e6, 268e6, 55e9, 45e9),      # bf16 + bias configuration, unequal rates
    (33.5e6, 33.5e6, 25e9, 25e9),    # one of 8 ranks' share
    (268e6, 30e6, 50e9, 50e9),       # little output: the input bounds the time
])
def test_growing_blocks_bound_matches_a_simulated_pipeline(h2d, d2h, r_in, r_out):
    got_ms = bench.growing_blocks_bound_ms(h2d, d2h, r_in / 1e9, r_out / 1e9)
    want_ms = simulate(h2d, d2h, r_in, r_out) * 1e3
    assert got_ms == pytest.approx(want_ms, rel=2e-3)
    # never below the plain bound of either direction
    assert got_ms >= max(h2d / r_in, d2h / r_out) * 1e3 * (1 - 1e-9)


def test_growing_blocks_bound_of_the_fp16_configuration():
    # 268 MB each way at 50 GB/s: the copy-out is starved until half the
    # input is in (t* = T_in / 2), then runs at its rate: 6.71 ms, not 5.37
    ms = bench.growing_blocks_bound_ms(268435456, 268435456, 50.0, 50.0)
    assert ms == pytest.approx(2.68435456 + 4.02653184, rel=1e-9)


def test_config_records_name_the_workloads():
    for name, wl in bench.WORKLOADS.items():
        cfg = bench.config_of(name, wl, 1)
        assert cfg["workload"] == name
        assert "timed_region" in cfg and "l2" in cfg
    fp32 = bench.config_of("matmul_fp32", bench.WORKLOADS["matmul_fp32"], 1, "graph")
    assert fp32["timed_region"] == "one CUDA-graph replay of the K steps"
    assert "buffer sets" in fp32["l2"]  # 12 MB per set: steps rotate through sets > 2x L2
    f16 = bench.config_of("matmul_f16", bench.WORKLOADS["matmul_f16"], 8)
    assert f16["parallelism"] == "M-row shards x8" and f16["timed_region"] == "K host launches"


def test_flops_and_buffer_sets():
    wl = bench.WORKLOADS["matmul_bf16"]
    assert bench.flops_of(wl, wl["m"]) == 2 * 32768 * 4096 * 4096 + 32768 * 4096
    assert bench.matmul_buffer_sets(bench.WORKLOADS["matmul_f16"], 8192) == 1
    sets = bench.matmul_buffer_sets(bench.WORKLOADS["matmul_fp32"], 1024)
    assert sets * 3 * 1024 * 1024 * 4 > 2 * bench.L2_BYTES
