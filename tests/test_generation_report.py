"""``generate_report`` (generation.py) on CPU: percentiles and throughput."""
from llama1b_megakernel_b200.generation import generate_report


def test_report_percentiles_and_throughput():
    r = generate_report([10.0, 20.0, 30.0, 40.0, 50.0], max_length=100, max_batch_size=2, n_runs=5)
    assert r["latency_ms_p50"] == 30.0 and r["latency_ms_p100"] == 50.0
    assert r["latency_ms_avg"] == 30.0 and r["n_runs"] == 5
    assert abs(r["throughput"] - 2 * 100 / 0.030) < 1e-6
    assert set(r) >= {"latency_ms_p50", "latency_ms_p90", "latency_ms_p95", "latency_ms_p99",
                      "latency_ms_p100", "latency_ms_avg", "throughput"}
