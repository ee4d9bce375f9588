"""bench.py's roofline arithmetic (no GPU): a launch is tensor-bound or HBM-bound by its
arithmetic intensity against the ridge (dense FP8 peak / HBM bandwidth), and `achieved` is
the algorithmic rate in that bound's unit."""
import math

import bench

PEAK = (3236.8, "measured")  # TFLOP/s, dense FP8 (2 x the driver's bf16 figure)
HBM = (6549.4, "measured")   # GB/s


def test_headline_is_tensor_bound():
    M = N = K = 8192
    flops, alg = 2.0 * M * N * K, float(M * K + N * K + 2 * M * N)
    r = bench.roofline(flops, alg, 0.38, PEAK, 2759.6, HBM, 463e6)
    assert r["bound"] == "tensor" and r["unit"] == "TFLOP/s"
    assert math.isclose(r["achieved"], flops / 0.38e-3 / 1e12)
    assert math.isclose(r["frac"], r["achieved"] / PEAK[0])
    assert math.isclose(r["frac_sustained"], r["achieved"] / 2759.6)
    assert r["traffic"] == 463e6


def test_skinny_is_hbm_bound():
    M, N, K = 128, 8192, 8192
    flops, alg = 2.0 * M * N * K, float(M * K + N * K + 2 * M * N)
    r = bench.roofline(flops, alg, 0.0186, PEAK, 2759.6, HBM, None)
    assert r["bound"] == "hbm" and r["unit"] == "GB/s"
    assert math.isclose(r["achieved"], alg / 0.0186e-3 / 1e9)  # ~3780 GB/s
    assert math.isclose(r["frac"], r["achieved"] / HBM[0])
    assert r["arithmetic_intensity"] < r["ridge"]


def test_traffic_table_names_real_workloads():
    for (workload, world), traffic in bench.TRAFFIC_BYTES_PER_LAUNCH.items():
        assert workload in bench.WORKLOADS and world >= 1 and traffic > 0


def test_parity_rows_cover_every_rank_edge_and_row_block():
    from hipgemm_b200.shard import row_range
    for M, world in [(8192, 1), (8192, 8), (16384, 4), (1000, 3), (128, 2)]:
        rows = bench.parity_rows(M, world)
        assert rows == sorted(set(rows)) and 0 <= rows[0] and rows[-1] < M
        for r in range(world):
            r0, r1 = row_range(M, r, world)
            assert r0 in rows and r1 - 1 in rows
        blocks = {x // 128 for x in rows}
        assert blocks == set(range((M + 127) // 128))


def test_both_arms_report_the_same_config():
    """The reference arm and ours describe the workload with the same dict."""
    import inspect
    src = inspect.getsource(bench.run_reference) + inspect.getsource(bench.run_ours)
    assert src.count('"config": workload_config(args.workload)') == 2
    for name in bench.WORKLOADS:
        c = bench.workload_config(name)
        M, N, K, _ = bench.WORKLOADS[name]
        assert (c["M"], c["N"], c["K"]) == (M, N, K) and "l2" in c


def test_cpu_baseline_times_the_reference_function():
    """The CPU baseline times the reference's own gemm_cpu where oracle/_ref holds it (kind
    "reference"), else the oracle's restatement of the same loop (kind "port"), with every
    host core, on a bounded sample."""
    import os
    from oracle import reference
    r = bench.cpu_reference_rate(512, 512, 512, 1.0, 0, budget_s=0.5, steps=2, warmup=1)
    expect = "reference" if os.path.isfile(reference.LIB_PATH) else "port"
    assert r["kind"] == expect and r["unit"] == "TFLOP/s" and r["value"] > 0
    assert r["cores"] == len(os.sched_getaffinity(0))
    assert "512x512x512" in r["sample"]
