"""bench.py's host-side arithmetic (CPU only): the PCIe bound, the per-kernel table and the
in-run CPU baseline's median-of-3 legs."""
import importlib.util
import os

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(REPO, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


PEAKS = {"h2d_gbs": 55.0, "d2h_gbs": 57.0, "duplex_gbs": 100.0}


def test_pcie_bound_overlaps_the_smaller_direction(bench):
    # 3 GB in, 2 GB out: 2 GB each way at half the duplex rate, then 1 GB H2D alone
    f = bench.pcie_fields(3_000_000_000, 2_000_000_000, 0.1, PEAKS)
    bound = 2e9 / 50e9 + 1e9 / 55e9
    assert f["pcie_bound_ms"] == pytest.approx(bound * 1e3, abs=1e-3)
    assert f["pcie_frac"] == pytest.approx(bound / 0.1, abs=1e-4)
    assert f["pcie_gbs"] == pytest.approx(50.0)


def test_pcie_bound_never_below_a_direction_alone(bench):
    # a duplex rate above twice the solo rates cannot make one direction faster than solo
    f = bench.pcie_fields(1_000_000_000, 1_000_000_000, 1.0, dict(PEAKS, duplex_gbs=500.0))
    assert f["pcie_bound_ms"] == pytest.approx(1e9 / 55e9 * 1e3, abs=1e-3)
    assert bench.pcie_fields(1, 1, 1.0, None) == {}


def test_summarize_kernels_groups_by_name_and_picks_the_dominant(bench):
    names = ["a", "b", "a"]
    per = [[1.0, 1.0], [3.0, 3.0], [1.0, 1.0]]  # ms per launch, two steps
    table, dom = bench.summarize_kernels(names, per, [1e9, 2e9, 1e9], [10, 10, 10], 1000.0)
    assert dom == "b"  # 6 ms in all against 4 ms for a's two launches per step
    assert table["a"]["launches"] == 4 and table["b"]["launches"] == 2
    assert table["a"]["gbs"] == pytest.approx(1000.0) and table["a"]["frac_of_peak"] == 1.0
    assert table["b"]["gbs"] == pytest.approx(2e9 / 3e-3 / 1e9, rel=1e-3)
    r = bench.roofline_of(table, dom, 1000.0, "measured", "no-such-key")
    assert r["kernel"] == "b" and r["traffic"] is None and r["bound"] == "hbm"


def test_cpu_baseline_reports_all_cores_and_one_thread(bench):
    import runner
    cfg = runner.CONFIGS["c1"]
    r = bench.cpu_chain_baseline(cfg, 64, 32, 0.3)
    assert r["value"] > 0 and r["value_1t"] > 0 and r["threads"] >= 1
    assert r["rows_all"] == 64 and r["rows_1t"] == 32
