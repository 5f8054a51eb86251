"""Host logic of bench.py that needs no GPU: a run whose tensor-core kernels raised the device
error flag ends the measurement (it is neither measured nor repeated), a stalled phase ends the
run with the launch monitor's report, and the clock samples taken during the timed region are
summarised with the throttle reasons seen under load."""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


class FakeFlag:
    """Stands in for the device error flag: raised after the listed runs (0-based)."""

    def __init__(self, raised_on):
        self.raised_on = set(raised_on)
        self.labels = []

    def __call__(self, label):
        n = len(self.labels)
        self.labels.append(label)
        return "a tensor-core kernel gave up a bounded wait (site 3)" if n in self.raised_on \
            else None


def test_clean_run_is_returned():
    calls = []
    flag = FakeFlag(raised_on=[])
    out = bench.run_checked(lambda: calls.append(1) or len(calls), flag, "timed steps")
    assert out == 1 and len(calls) == 1
    assert flag.labels == ["timed steps"]


def test_run_that_raised_the_flag_ends_the_measurement_without_a_repeat():
    runs = []
    flag = FakeFlag(raised_on=[0])
    with pytest.raises(bench.RunFailed, match="end-to-end steps: .*site 3"):
        bench.run_checked(lambda: runs.append(1), flag, "end-to-end steps")
    assert len(runs) == 1                    # never run a second time


def test_clock_summary_uses_loaded_samples_and_reports_throttle_reasons():
    cs = bench.ClockSampler(0)
    cs.proc = object()                       # as if nvidia-smi had been started
    cs.out = "\n".join([
        "0, 345, 1965, 120.5, 0, Not Active, Not Active, Not Active, Not Active",   # idle
        "0, 1402, 1965, 990.1, 100, Not Active, Not Active, Not Active, Active",
        "0, 1380, 1965, 995.0, 100, Not Active, Not Active, Not Active, Active",
        "0, 1410, 1965, 980.7, 99, Not Active, Not Active, Not Active, Active",
        "garbage line",
    ])
    s = cs.summary()
    assert s["sm_mhz"] == 1402               # median of the three samples under load
    assert s["sm_max_mhz"] == 1965
    assert s["samples"] == 3
    assert s["reasons"] == ["sw_power_cap"]
    assert s["power_w_max"] == 995.0


def test_kernel_table_fractions():
    pk = {"hbm_gbs": 6000.0, "bf16_tflops": 1700.0, "bf16_tflops_sustained": 1400.0}
    summary = {"qb_rmsnorm_fwd": {"launches": 2, "ms_total": 1.0, "bytes": 3_000_000_000,
                                  "flops": 0},
               "qb_gemm2_bf16": {"launches": 4, "ms_total": 10.0, "bytes": 0,
                                 "flops": 14_000_000_000_000}}
    t = bench.kernel_table(summary, pk)
    assert t["qb_rmsnorm_fwd"]["achieved_gbs"] == 3000.0 and t["qb_rmsnorm_fwd"]["frac"] == 0.5
    assert t["qb_gemm2_bf16"]["achieved_tflops"] == 1400.0
    assert t["qb_gemm2_bf16"]["frac"] == 1.0     # against the sustained peak


def test_watchdog_reports_the_launch_monitor_when_a_phase_overruns(monkeypatch, capsys):
    """A phase that overruns its deadline ends the run with the launch monitor's report (read
    from host memory: which launch has CTAs that never finished, the site of a wait that gave
    up) in an error JSON line, instead of hanging until killed."""
    import json
    import threading
    import time
    from types import SimpleNamespace

    exited = threading.Event()
    codes = []

    def fake_exit(code):
        codes.append(code)
        exited.set()

    monkeypatch.setattr(bench.os, "_exit", fake_exit)

    class FakeLib:
        def qb_monitor_report(self, device, buf, n):
            buf.value = (b"launches issued: 12 (last gemm2_bf16); finished through #11; "
                         b"no wait has given up; 148 CTA(s) started but not finished: #12")
            return 0

        def qb_last_error(self):
            return b""

    dog = bench.Watchdog(FakeLib(), 0, 0, 1, SimpleNamespace(steps=5, warmup=3))
    slow = dog.watched("warm-up step 0", 0.05, lambda: time.sleep(0.01))
    slow()                                    # finishes in time: nothing fires
    time.sleep(0.2)
    assert not exited.is_set()
    dog.arm("warm-up step 1", 0.05)           # never disarmed: the phase overruns
    assert exited.wait(5.0)
    assert codes == [3]
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert line["value"] is None
    assert "warm-up step 1" in line["error"]
    assert "started but not finished: #12" in line["launch_monitor"]


def _reference_arm(extra_env, steps=2, warmup=1):
    import subprocess
    env = dict(os.environ, **extra_env)
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                           "--config", "0.5b", "--steps", str(steps), "--warmup", str(warmup),
                           "--cpu-tokens", "32"], env=env, cwd=ROOT, capture_output=True,
                          text=True, timeout=600)


def test_reference_arm_prints_the_driver_contract_line():
    """--impl reference: the eager CPU path on the host cores, one JSON line with the same metric
    and unit as the measured arm, `impl`, the CPU baseline it is, and an e2e without copies.
    `steps` counts the samples actually timed and `ms_per_step` is their measured mean wall
    time; the whole-model figure scaled from them is `value`, with the sample's parts beside it,
    so steps x ms_per_step is time the run really spent."""
    import json
    import time
    t0 = time.monotonic()
    r = _reference_arm({"WORLD_SIZE": "1", "RANK": "0"}, steps=2, warmup=1)
    wall = time.monotonic() - t0
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["metric"] == bench.METRIC
    assert line["unit"] == "tokens/s" and line["higher_is_better"] is True
    assert line["steps"] == 2 and line["warmup"] == 1
    assert line["value"] > 0 and line["cpu_baseline"]["value"] == line["value"]
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    smp = line["sample"]
    assert smp["tokens"] == 32 and smp["layers_scaled"] == 24
    assert line["ms_per_step"] == pytest.approx(1e3 * (smp["layer_s"] + smp["head_s"]), rel=0.02)
    assert line["value"] == pytest.approx(32 / (24 * smp["layer_s"] + smp["head_s"]), rel=0.02)
    assert line["steps"] * line["ms_per_step"] / 1e3 < wall
    assert line["e2e"] == {"value": line["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_without_work():
    r = _reference_arm({"WORLD_SIZE": "2", "RANK": "1"})
    assert r.returncode == 0 and r.stdout.strip() == ""
