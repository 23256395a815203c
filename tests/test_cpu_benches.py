"""The CPU benchmarks run end to end on a small load: the directory control
plane (registrations, updates, lookups and event notifications all counted)
and the resume proxy's added latency (every chunk seen on both paths)."""
from connex_b200.bench.control_plane_bench import bench as cp_bench
from connex_b200.bench.proxy_overhead import bench as proxy_bench


def test_control_plane_bench_small():
    r = cp_bench(endpoints=50, updaters=1, duration_s=1.0)
    assert r["updates_per_s"] > 0 and r["lookups"] > 0 and r["events"] > 0
    assert r["lookup_p50_ms"] is not None and r["notify_p99_ms"] is not None


def test_proxy_overhead_bench_small():
    r = proxy_bench(requests=8, concurrency=4, tokens=8, tpot_ms=1.0, passes=1)
    assert r["direct"]["chunks"] == r["proxy"]["chunks"] == 64
