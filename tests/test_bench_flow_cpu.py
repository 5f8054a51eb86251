"""bench.py's measurement run end to end on the CPU, with only what needs a GPU replaced: CUDA
events / streams / synchronisation, the model's training step, the per-call kernel timer, the
tensor-core error flag and the launch monitor. It checks the Python of every phase (warm-up
under the watchdog, timed steps, instrumented step, end-to-end steps, the JSON line), and that a
run whose kernels raised the error flag ends the measurement with the evidence - never measured,
never repeated."""

import json
import os
import sys
import types

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


class FakeEvent:
    clock = [0.0]

    def __init__(self, enable_timing=False):
        self.t = None

    def record(self, stream=None):
        FakeEvent.clock[0] += 10.0          # 10 "ms" between consecutive records
        self.t = FakeEvent.clock[0]

    def elapsed_time(self, other):
        return other.t - self.t


class FakeCuda:
    Event = FakeEvent
    nvtx = types.SimpleNamespace(range_push=lambda name: 0, range_pop=lambda: 0)

    @staticmethod
    def Stream(device=None):
        return types.SimpleNamespace(cuda_stream=0)

    @staticmethod
    def set_device(d):
        pass

    @staticmethod
    def synchronize(d=None):
        pass


class TorchOnCpu:
    """The torch module as bench.py sees it: real, except CUDA and devices."""
    cuda = FakeCuda

    def __getattr__(self, name):
        return getattr(torch, name)

    @staticmethod
    def device(*a, **k):
        return torch.device("cpu")


class FakeLib:
    def __init__(self, raised_on=()):
        self.calls = 0
        self.raised_on = set(raised_on)

    def qb_device_error(self, stream):
        self.calls += 1
        return 4 if self.calls in self.raised_on else 0

    def qb_last_error(self):
        return b"a tensor-core kernel gave up a bounded wait (site 3)"

    def qb_monitor_report(self, device, buf, n):
        buf.value = b"launches issued: 40 (last gemm2_bf16); last wait that gave up: site 3"
        return 0


class FakeTimer:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False

    def summary(self):
        return {"qb_gemm2_bf16": {"launches": 4, "ms_total": 10.0, "bytes": 0,
                                  "flops": 14_000_000_000_000},
                "qb_rmsnorm_fwd": {"launches": 2, "ms_total": 1.0, "bytes": 3_000_000_000,
                                   "flops": 0}}


def _run(monkeypatch, capsys, lib, steps=2):
    from hackathon_b200 import _lib, dp, qlora
    monkeypatch.setattr(bench, "torch", TorchOnCpu())
    monkeypatch.setattr(torch.Tensor, "pin_memory", lambda self: self)
    monkeypatch.setattr(_lib, "load", lambda: lib)
    monkeypatch.setattr(_lib, "stream", lambda d=None: 0)
    monkeypatch.setattr(_lib, "KernelTimer", FakeTimer)
    steps_run = []

    def fake_step(model, opt, ids, labels, grad_sync=None, num_items_in_batch=None):
        steps_run.append(ids.shape)
        return torch.tensor(11.5)

    monkeypatch.setattr(qlora, "QwenQLoRA", lambda shape, dev, seed=0: types.SimpleNamespace(
        adapter_parameters=lambda: []))
    monkeypatch.setattr(qlora, "make_optimizer", lambda model: None)
    monkeypatch.setattr(qlora, "synthetic_batch", lambda shape, b, s, dev, seed: (
        torch.zeros(b, s, dtype=torch.int64), torch.zeros(b, s, dtype=torch.int64)))
    monkeypatch.setattr(qlora, "train_step", fake_step)
    monkeypatch.setattr(dp, "global_label_count", lambda lb, group=None: torch.tensor(8.0))
    monkeypatch.setenv("WORLD_SIZE", "1")
    monkeypatch.setenv("RANK", "0")
    monkeypatch.setattr(sys, "argv", ["bench.py", "--config", "0.5b", "--steps",
                                      str(steps), "--warmup", "3", "--no-cpu-baseline"])
    bench.main()
    out = capsys.readouterr().out.strip().splitlines()
    return json.loads(out[-1]), steps_run


def test_run_prints_one_complete_line(monkeypatch, capsys):
    line, steps_run = _run(monkeypatch, capsys, FakeLib())
    # 3 warm-up + 2 timed + 1 instrumented + 2 end-to-end steps
    assert len(steps_run) == 8
    assert line["n_gpus"] == 1 and line["steps"] == 2 and line["warmup"] == 3
    assert line["ms_per_step"] == pytest.approx(5.0)          # 10 "ms" over 2 steps
    assert line["value"] == pytest.approx(2 * 256 / 5e-3)
    assert line["e2e"]["h2d_bytes_per_step"] == 2 * 2 * 256 * 8
    assert line["e2e"]["last_loss"] == 11.5
    assert line["roofline"]["kernel"] == "qb_gemm2_bf16"
    assert line["roofline"]["bound"] == "tensor"
    assert line["gpu_launches"] == 6 * 2
    assert "reasons" in line["clocks"]


def test_run_that_raised_the_flag_ends_the_measurement(monkeypatch, capsys):
    # flag reads: 3 warm-up steps (1-3), the timed block (4: raised)
    line, steps_run = _run(monkeypatch, capsys, FakeLib(raised_on={4}))
    assert len(steps_run) == 3 + 2                          # nothing after the timed block
    assert line["value"] is None
    assert "timed steps" in line["error"] and "site 3" in line["error"]
    assert "site 3" in line["launch_monitor"]


def test_flag_raised_in_warm_up_ends_it_there(monkeypatch, capsys):
    line, steps_run = _run(monkeypatch, capsys, FakeLib(raised_on={1}))
    assert len(steps_run) == 1
    assert line["value"] is None and "warm-up step 0" in line["error"]
