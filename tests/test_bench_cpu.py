"""Host logic of bench.py that needs no GPU: a run whose tensor-core kernels raised the device
error flag is repeated and never measured, and the clock samples taken during the timed region
are summarised with the throttle reasons seen under load."""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


class FakeFlag:
    """Stands in for the device error flag: raised after the listed attempts (0-based)."""

    def __init__(self, raised_on):
        self.raised_on = set(raised_on)
        self.labels = []

    def __call__(self, label):
        n = len(self.labels)
        self.labels.append(label)
        return "a tensor-core kernel gave up a bounded wait (site 3)" if n in self.raised_on \
            else None


def test_clean_run_is_kept_at_once():
    calls = []
    flag = FakeFlag(raised_on=[])
    out = bench.run_clean(lambda: calls.append(1) or len(calls), flag, "timed steps")
    assert out == 1 and len(calls) == 1
    assert flag.labels == ["timed steps (attempt 0)"]


def test_run_that_raised_the_flag_is_repeated_and_the_clean_one_returned():
    results = iter([10.0, 20.0, 30.0])
    flag = FakeFlag(raised_on=[0, 1])
    out = bench.run_clean(lambda: next(results), flag, "warm-up step 0")
    assert out == 30.0                       # the measurement of the first clean attempt
    assert flag.labels == [f"warm-up step 0 (attempt {k})" for k in range(3)]


def test_every_attempt_raising_the_flag_is_a_failure():
    runs = []
    flag = FakeFlag(raised_on=range(100))
    with pytest.raises(bench.RunFailed, match="end-to-end steps"):
        bench.run_clean(lambda: runs.append(1), flag, "end-to-end steps", repeats=2)
    assert len(runs) == 3                    # bounded: repeats + 1 attempts, no more


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


def test_watchdog_reports_the_device_flag_when_a_phase_overruns(monkeypatch, capsys):
    """A phase that overruns its deadline ends the run with the kernels' error flag (the site
    of the wait that gave up) in an error JSON line, instead of hanging until killed."""
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
        def qb_device_error(self, stream):
            return 4

        def qb_last_error(self):
            return b"a tensor-core kernel gave up a bounded wait (site 65)"

    dog = bench.Watchdog(FakeLib(), None, 0, 1, SimpleNamespace(steps=5, warmup=3),
                         stream=SimpleNamespace(cuda_stream=0))
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
    assert "site 65" in line["device_error_flag"]


def _completed(code, out):
    import subprocess
    return subprocess.CompletedProcess(args=[], returncode=code, stdout=out)


def test_supervisor_measures_again_after_a_stalled_attempt(capsys):
    """A child whose watchdog fired (status 3) is followed by one fresh child; the line printed
    is the fresh child's measurement, with the stalled attempt's own error line attached."""
    import json
    stalled = json.dumps({"value": None, "error": "watchdog: warm-up step 0 did not finish in 90 s",
                          "device_error_flag": "clear: no bounded wait gave up"})
    good = json.dumps({"metric": "m", "value": 22000.0})
    results = iter([_completed(3, stalled + "\n"), _completed(0, good + "\n")])
    calls = []

    def fake_run(cmd, **kw):
        calls.append(cmd)
        return next(results)

    assert bench.supervise(["python", "bench.py", "--worker"], run=fake_run) == 0
    assert len(calls) == 2
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert line["value"] == 22000.0
    assert line["restarts"][0]["device_error_flag"].startswith("clear")


def test_supervisor_passes_a_clean_run_through_and_stops_after_the_last_attempt(capsys):
    import json
    good = json.dumps({"metric": "m", "value": 1.0})
    assert bench.supervise(["x"], run=lambda cmd, **kw: _completed(0, good)) == 0
    assert json.loads(capsys.readouterr().out.strip()) == {"metric": "m", "value": 1.0}
    stalled = json.dumps({"value": None, "error": "watchdog"})
    n = []

    def always_stalls(cmd, **kw):
        n.append(1)
        return _completed(3, stalled)

    assert bench.supervise(["x"], run=always_stalls) == 3
    assert len(n) == 2                                   # bounded: one fresh attempt only
    assert json.loads(capsys.readouterr().out.strip().splitlines()[-1])["value"] is None


def _reference_arm(extra_env):
    import subprocess
    env = dict(os.environ, **extra_env)
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                           "--config", "0.5b", "--steps", "1", "--warmup", "0",
                           "--cpu-tokens", "32"], env=env, cwd=ROOT, capture_output=True,
                          text=True, timeout=600)


def test_reference_arm_prints_the_driver_contract_line():
    """--impl reference: the eager CPU path on the host cores, one JSON line with the same metric
    and unit as the measured arm, `impl`, the CPU baseline it is, and an e2e without copies."""
    import json
    r = _reference_arm({"WORLD_SIZE": "1", "RANK": "0"})
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["metric"] == bench.METRIC
    assert line["unit"] == "tokens/s" and line["higher_is_better"] is True
    assert line["value"] > 0 and line["cpu_baseline"]["value"] == line["value"]
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"] == {"value": line["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_without_work():
    r = _reference_arm({"WORLD_SIZE": "2", "RANK": "1"})
    assert r.returncode == 0 and r.stdout.strip() == ""
