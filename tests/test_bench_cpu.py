"""bench.py pieces that run without a GPU: the clock sampler's window (samples inside the
timed region; for a region shorter than the sampling period, those within 0.5 s of it) and
its throttle-reason flags, on synthetic nvidia-smi lines."""
import datetime
import importlib.util
import os
import time

from conftest import ROOT


def load_bench():
    spec = importlib.util.spec_from_file_location("bench", os.path.join(ROOT, "bench.py"))
    b = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(b)
    return b


def line(t, mhz, power_cap="Not Active", thermal="Not Active"):
    ts = datetime.datetime.fromtimestamp(t).strftime("%Y/%m/%d %H:%M:%S.%f")[:-3]
    return f"{ts}, 0, {mhz}, 1965, 900.0, 0x0, Not Active, Not Active, {thermal}, {power_cap}"


def test_clock_window_and_reasons():
    b = load_bench()
    now = time.time()
    c = b.ClockSampler(0)
    c.lines = [line(now - 1.0, 1000), line(now + 0.1, 1900, power_cap="Active"),
               line(now + 0.3, 1965), line(now + 2.0, 500, thermal="Active")]
    c.t_begin, c.t_end = now, now + 0.5
    s = c.summary()
    assert s["samples"] == 2 and s["sm_mhz"] == 1932.5 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"] and s["window"] == "timed region"
    # a region shorter than the 200 ms period: the samples within 0.5 s of it
    c.t_begin, c.t_end = now + 0.7, now + 0.8
    s = c.summary()
    assert s["samples"] == 1 and s["sm_mhz"] == 1965.0 and "within 0.5 s" in s["window"]
    # no window marked: every sample, all reasons seen
    c.t_begin = c.t_end = None
    s = c.summary()
    assert s["samples"] == 4 and s["reasons"] == ["sw_power_cap", "sw_thermal_slowdown"]
    c.lines = []
    assert c.summary()["reasons"] == ["unsampled"]


def test_reference_arm_line():
    """`bench.py --impl reference` (the reference's own CPU code, on the host cores) prints
    one JSON line with the metric of our arm and its CPU-baseline description."""
    import json
    import subprocess
    import sys
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "0", "--ref-seqs", "1"],
                         capture_output=True, text=True, timeout=600, cwd=ROOT, check=True).stdout
    d = json.loads([ln for ln in out.splitlines() if ln.startswith("{")][-1])
    assert d["impl"] == "reference" and d["metric"].startswith("DeltaNet+GQA decode tokens/s")
    assert d["value"] > 0 and d["unit"] == "tokens/s" and d["higher_is_better"] is True
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] in ("reference", "port") and cb["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["value"] == d["value"]
