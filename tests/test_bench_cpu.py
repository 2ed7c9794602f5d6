"""The reference arm of bench.py (the reference's own CPU build, timed on the
host) prints one JSON line with the keys the benchmark contract asks for; it
needs no GPU. Skipped where the reference build (oracle/_ref) is absent."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_line():
    if not os.path.exists(os.path.join(ROOT, "oracle", "_ref", "libttref.so")):
        pytest.skip("oracle/_ref not built (it needs the reference sources)")
    env = dict(os.environ, OMP_NUM_THREADS="4")
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--config", "llama-13m",
                        "--steps", "1", "--warmup", "3"], cwd=ROOT, capture_output=True,
                       text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    for k in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
              "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
              "cpu_baseline", "e2e"):
        assert k in line, k
    assert line["impl"] == "reference" and line["metric"] == "train tokens/sec"
    assert line["value"] > 0 and line["higher_is_better"] is True
    assert line["e2e"]["value"] == line["value"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    cb = line["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] == 4 and cb["value"] == line["value"]
    assert "depth 1" in cb["sample"] and "depth 2" in cb["sample"]
    parts = line["reference_parts"]
    # full depth = rest + layers * per_layer, with the parts from the two samples
    assert parts["micro_s"] == pytest.approx(parts["rest_s"] + 6 * parts["per_layer_s"])
    # per layer = t(2) - t(1), or t(2) / 2 when timing noise makes the difference <= 0
    assert parts["per_layer_s"] > 0 and parts["rest_s"] >= 0
    assert parts["per_layer_s"] in (pytest.approx(parts["timed"]["2"] - parts["timed"]["1"]),
                                    pytest.approx(parts["timed"]["2"] / 2))
    assert line["steps"] == 2 and line["steps_requested"] == 1
    assert line["config"]["workload"].startswith("llama-13m")


def test_clock_samples_windowed_by_timestamp():
    """The clock summary keeps only the samples stamped inside the timed
    region, so nvidia-smi's start-up and the idle seconds before the region do
    not count; the throttle reasons come from the samples inside it."""
    import datetime
    sys.path.insert(0, ROOT)
    import bench

    def row(ts, mhz, cap):
        return (f"2026/12/02 10:00:{ts:06.3f}, 0, {mhz}, 1965, 900.0, 0x4, Not Active, "
                f"Not Active, Not Active, {'Active' if cap else 'Not Active'}")
    lines = [row(1.0, 300, False), row(2.0, 300, False),  # before the region: idle
             row(3.0, 1450, True), row(3.2, 1460, True), row(3.4, 1440, False),
             row(5.0, 1965, False), "garbage line", ""]
    t0 = datetime.datetime(2026, 12, 2, 10, 0, 2, 500000)
    t1 = datetime.datetime(2026, 12, 2, 10, 0, 4, 0)
    s = bench.ClockSampler.parse(lines, t0, t1)
    assert s["samples"] == 3 and s["sm_mhz"] == 1450.0 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"]
    empty = bench.ClockSampler.parse(lines, t1, t1)
    assert empty["sm_mhz"] is None and empty["reasons"] == ["no samples"]


def test_clock_summary_of_a_short_region_uses_neighbouring_samples(tmp_path):
    """A region shorter than the 200 ms sampling period holds no sample; its
    summary then takes the samples within half a second of it."""
    import datetime
    sys.path.insert(0, ROOT)
    import bench
    path = tmp_path / "clocks.csv"
    path.write_text("".join(
        f"2026/12/02 10:00:{s:06.3f}, 0, {mhz}, 1965, 900.0, 0x4, Not Active, Not Active, "
        f"Not Active, Active\n" for s, mhz in ((1.0, 1400), (1.2, 1500), (3.0, 1600))))
    c = bench.ClockSampler([0], active=False)
    c.path = str(path)
    t0 = datetime.datetime(2026, 12, 2, 10, 0, 1, 50000)
    t1 = datetime.datetime(2026, 12, 2, 10, 0, 1, 100000)
    s = c.summary(t0, t1)
    assert s["samples"] == 2 and s["sm_mhz"] == 1450.0 and "window" in s
    assert s["reasons"] == ["sw_power_cap"]
