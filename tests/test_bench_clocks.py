"""The bench's clock sampler keeps only the nvidia-smi rows stamped inside
the timed window (plus the first one after it), exercised against a fake
nvidia-smi on PATH so it runs without a GPU."""
import importlib.util
import os
import stat
import time

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

FAKE = """#!/bin/bash
# prints one timestamped row every 20 ms; the first 0.3 s report a throttle
# reason that must fall outside the timed window
start=$(date +%s%N)
while true; do
  now=$(date +%s%N)
  ts=$(date +"%Y/%m/%d %H:%M:%S.%3N")
  if [ $(( (now - start) / 1000000 )) -lt 300 ]; then slow=Active; else slow="Not Active"; fi
  echo "$ts, 0, 1900, 1965, 700.0, 0x0, $slow, Not Active, Not Active, Active"
  sleep 0.02
done
"""


def _load_bench():
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(REPO, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_clock_sampler_window(tmp_path, monkeypatch):
    exe = tmp_path / "nvidia-smi"
    exe.write_text(FAKE)
    exe.chmod(exe.stat().st_mode | stat.S_IEXEC)
    monkeypatch.setenv("PATH", str(tmp_path) + os.pathsep + os.environ["PATH"])
    bench = _load_bench()
    s = bench.ClockSampler(0)
    s.start()
    time.sleep(0.5)               # past the fake's throttled prefix
    s.mark_begin()
    time.sleep(0.05)              # a short "timed region"
    s.mark_end()
    clocks = s.stop()
    assert clocks is not None and clocks["samples"] >= 1
    assert clocks["sm_mhz"] == 1900 and clocks["sm_max_mhz"] == 1965
    assert clocks["reasons"] == ["sw_power_cap"]
