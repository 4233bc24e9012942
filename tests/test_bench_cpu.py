"""Host-side pieces of bench.py that need no GPU: the clock sampler's summary
(with a stand-in for NVML) and the algorithmic byte counts."""
import importlib.util
import time
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_clock_sampler_summarises_samples(bench):
    seq = [(1965.0, 1965.0, 700.0, frozenset()),
           (1340.0, 1965.0, 1004.0, frozenset({"sw_power_cap", "gpu_idle"}))]
    i = iter(seq * 1000)
    with bench.ClockSampler(0, reader=lambda: next(i)) as c:
        time.sleep(0.08)
    s = c.summary()
    assert s["samples"] >= 2
    assert s["sm_max_mhz"] == 1965.0
    assert s["sm_min_mhz"] == 1340.0
    assert 1340.0 <= s["sm_mhz"] <= 1965.0
    assert s["power_w_max"] == 1004.0
    # only the reasons that decide whether a run is kept are reported
    assert s["reasons"] == ["sw_power_cap"]


def test_clock_sampler_reports_reader_failure(bench):
    def broken():
        raise RuntimeError("no device")

    with bench.ClockSampler(0, reader=broken) as c:
        time.sleep(0.02)
    s = c.summary()
    assert s["samples"] == 0 and s["sm_mhz"] is None
    assert "no device" in s["error"]


def test_algorithmic_bytes_split_modes(bench):
    m = n = k = 8192
    # packed operands: 8 bytes per element of A and of B^T, C written once
    assert bench.algorithmic_bytes(3, m, n, k) == 8 * m * k + 8 * n * k + 4 * m * n
    assert bench.algorithmic_bytes(1, m, n, k) == 8 * m * k + 8 * n * k + 4 * m * n
