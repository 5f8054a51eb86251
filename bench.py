"""Benchmark of the Qwen2.5 QLoRA training step on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 7b|1.5b|0.5b] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N

Workload (default): the headline configuration, the Qwen2.5-7B-shaped QLoRA step — 28 layers, hidden
3584, intermediate 18944, 28/4 heads x 128, vocab 152064, NF4 (bs 64, double quant) base, LoRA
r=64 alpha=128 (dropout 0.05) on all seven linears, batch 4 x 4096 per GPU, activation
checkpointing, AdamW on the adapters; data-parallel with an fp32 NCCL all-reduce of the adapter
gradients. Synthetic data and random weights (no network). Per-GPU work is fixed as N grows
(weak scaling).

Prints ONE JSON line (rank 0): tokens/s of the whole job timed with CUDA events (max over
ranks), the end-to-end number through the public API with host<->device copies, per-kernel
device times of this package's kernels with their roofline fractions, the roofline of the
dominant one, the CPU baseline (the reference's eager path on the host cores, a bounded sample),
and the SM clocks sampled during the timed region.

Nothing is measured twice: a phase that overruns its deadline ends the run at once with the
launch monitor's report (which tensor-core launch has CTAs that never finished, the site of a
wait that gave up), and a phase whose kernels raised the device error flag ends it with the
flag's message. Either way the line has `value` null and the evidence.
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "QLoRA step tokens/s (Qwen2.5 shapes) + per-kernel % of HBM/tensor roofline"
WORKLOADS = {
    "7b": ("configs[4]: Qwen2.5-7B-shaped QLoRA step, data-parallel, 4 x 4096 tokens per GPU",
           4, 4096),
    "1.5b": ("configs[3]: Qwen2.5-1.5B-shaped QLoRA step, 4 x 2048 tokens per GPU", 4, 2048),
    "0.5b": ("configs[0] shapes: Qwen2.5-0.5B-shaped QLoRA step, 2 x 256 tokens per GPU", 2, 256),
}
# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) of the dominant kernel,
# from ncu captures of each of its launch shapes in the step, averaged over the step's launch mix.
# Keyed by --config.
TRAFFIC_PER_LAUNCH = {"7b": {"qb_gemm2_bf16": 1793e6, "qb_gemm_gateup_swiglu": 4207e6}}
TRAFFIC_SOURCE = ("ncu dram__bytes_read.sum + dram__bytes_write.sum of the one-CTA tcgen05 GEMM "
                  "(the kernel the step runs) at the step's launch shapes")

# per-kernel roofline class: "hbm" (bytes) or "tensor" (flops)
BOUND = {"qb_nf4_dequant": "hbm", "qb_rmsnorm_fwd": "hbm", "qb_rmsnorm_bwd": "hbm",
         "qb_rope_qk": "hbm", "qb_swiglu_fwd": "hbm", "qb_swiglu_bwd": "hbm",
         "qb_dropout_scale": "hbm", "qb_scaled_add": "hbm", "qb_ce_rows": "hbm",
         "qb_ce_reduce": "hbm", "qb_gemm_bf16": "tensor", "qb_gemm2_bf16": "tensor",
         "qb_nf4_linear_fwd": "tensor",
         "qb_nf4_linear_dgrad": "tensor", "qb_linear_ce_stats": "tensor",
         "qb_linear_ce_grad": "tensor", "qb_linear_ce_stats_logits": "tensor",
         "qb_ce_grad_from_logits": "hbm", "qb_gemm_bf16_mask_acc": "hbm",
         "qb_gemm_gateup_swiglu": "tensor", "qb_gemm2_rope_bf16": "tensor",
         # the forward's gate/up GEMM with the next masks drawn in its side warps: its flops are
         # the GEMM's (the Philox rounds it also runs are counted under no roofline)
         "qb_gemm_gateup_swiglu_masks": "tensor",
         "qb_dropout_mask": "hbm", "qb_dropout_apply": "hbm",
         # integer-pipe work (Philox rounds), counted in mask elements drawn: no HBM or tensor
         # roofline applies; on a side stream its events span the GEMMs it shares the SMs with
         "qb_dropout_bits": "philox"}


_T0 = time.monotonic()


def _phase(msg):
    """Progress of the run on stderr (seconds since start), so a run that is stopped early
    still shows which phase it was in; stdout keeps the one JSON line."""
    if int(os.environ.get("RANK", "0")) == 0:
        print(f"bench.py [{time.monotonic() - _T0:7.1f} s] {msg}", file=sys.stderr, flush=True)


# Deadline of one warm-up or instrumented step (and the unit of a K-step block's deadline) after
# which the watchdog ends the run with what it can read of the stall. A 7B step takes under 1 s
# (the first, with library set-up, about 4 s).
STEP_DEADLINE_S = 90.0


def monitor_report(lib, index):
    """The launch monitor's report for device `index`: read from pinned host memory the kernels
    write, with no CUDA call, so it answers while the device is stuck."""
    import ctypes
    buf = ctypes.create_string_buffer(2048)
    if lib.qb_monitor_report(int(index), buf, len(buf)) != 0:
        return "unread: " + lib.qb_last_error().decode(errors="replace")
    return buf.value.decode(errors="replace")


class Watchdog:
    """Ends a run whose phase overruns its deadline with evidence instead of a silent timeout:
    the launch monitor's report (which tensor-core launch, if any, has CTAs that started and
    never finished; the site of a bounded wait that gave up - read from host memory, no CUDA
    call), every thread's stack on stderr, and an error JSON line on rank 0; then the process
    exits with status 3."""

    def __init__(self, lib, index, rank, world, args):
        self.lib, self.index, self.rank, self.world, self.args = lib, index, rank, world, args
        self.cv = threading.Condition()
        self.deadline = None
        self.label, self.seconds = None, None
        threading.Thread(target=self._watch, daemon=True, name="bench-watchdog").start()

    def arm(self, label, seconds):
        with self.cv:
            self.label, self.seconds = label, seconds
            self.deadline = time.monotonic() + seconds
            self.cv.notify()

    def disarm(self):
        with self.cv:
            self.deadline = None
            self.cv.notify()

    def watched(self, label, seconds, fn):
        """fn wrapped so that each call runs under a deadline of `seconds`."""
        def run():
            self.arm(label, seconds)
            try:
                return fn()
            finally:
                self.disarm()
        return run

    def _watch(self):
        while True:
            with self.cv:
                if self.deadline is None:
                    self.cv.wait()
                    continue
                left = self.deadline - time.monotonic()
                if left > 0:
                    self.cv.wait(timeout=left)
                    continue
                label, seconds = self.label, self.seconds
            self._fire(label, seconds)
            return

    def _fire(self, label, seconds):
        import traceback
        try:
            report = monitor_report(self.lib, self.index)
        except Exception as e:  # noqa: BLE001 - evidence only
            report = f"unread: {e!r}"
        print(f"bench.py rank {self.rank}: watchdog: {label} overran {seconds:.0f} s; launch "
              f"monitor: {report}", file=sys.stderr, flush=True)
        names = {t.ident: t.name for t in threading.enumerate()}
        for ident, frame in sys._current_frames().items():
            print(f"-- thread {names.get(ident, ident)}", file=sys.stderr)
            traceback.print_stack(frame, file=sys.stderr)
        if self.rank == 0:
            print(json.dumps({"metric": METRIC, "value": None, "unit": "tokens/s",
                              "n_gpus": self.world, "steps": self.args.steps,
                              "warmup": self.args.warmup,
                              "error": f"watchdog: {label} did not finish in {seconds:.0f} s",
                              "launch_monitor": report}), flush=True)
        sys.stderr.flush()
        os._exit(3)


class RunFailed(Exception):
    """A tensor-core kernel gave up a bounded wait during a phase: its work is undone."""


def run_checked(run, device_error, where):
    """run(), then device_error(where) reads (and clears) the tensor-core kernels' error flag
    once the run's work is done. A raised flag ends the measurement (RunFailed): the run is
    neither measured nor repeated."""
    out = run()
    msg = device_error(where)
    if msg is not None:
        raise RunFailed(f"{where}: {msg}")
    return out


def fail(args, world, error, monitor):
    """A phase's kernels raised the device error flag: no measurement, say why."""
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps({"metric": METRIC, "value": None, "unit": "tokens/s", "n_gpus": world,
                          "steps": args.steps, "warmup": args.warmup,
                          "error": f"a tensor-core kernel gave up a bounded wait: {error}",
                          "launch_monitor": monitor}), flush=True)
    if world > 1:
        dist.destroy_process_group()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"],
                "bf16_tflops_sustained": p.get("bf16_tflops_sustained", p["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons every 200 ms while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out = ""

    def summary(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in getattr(self, "out", "").splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                rows.append((float(f[1]), float(f[2]), float(f[3]), float(f[4]), f[5:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        loaded = [r for r in rows if r[3] >= 50] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in loaded for i, v in enumerate(r[4]) if v == "Active"})
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": rows[0][1],
                "power_w_max": max(r[2] for r in rows), "samples": len(loaded),
                "reasons": reasons}


def kernel_table(summary, pk):
    """Per kernel: launches, ms, achieved GB/s (algorithmic bytes / device time), fraction."""
    table = {}
    for name, d in summary.items():
        ms = d["ms_total"]
        entry = {"launches": d["launches"], "kernels": d.get("kernels", d["launches"]),
                 "ms_total": round(ms, 3), "bound": BOUND.get(name, "hbm")}
        if ms > 0 and entry["bound"] == "hbm":
            gbs = d["bytes"] / (ms * 1e-3) / 1e9
            entry.update(achieved_gbs=round(gbs, 1), frac=round(gbs / pk["hbm_gbs"], 3),
                         bytes_per_launch=d["bytes"] // max(1, d["launches"]))
        elif ms > 0 and entry["bound"] == "philox":
            entry.update(achieved_gdraws_per_s=round(d["flops"] / (ms * 1e-3) / 1e9, 1),
                         draws_per_launch=d["flops"] // max(1, d["launches"]))
        elif ms > 0:
            tf = d["flops"] / (ms * 1e-3) / 1e12
            # kernels timed inside a seconds-long step: the sustained (power-capped) GEMM peak
            entry.update(achieved_tflops=round(tf, 1),
                         frac=round(tf / pk["bf16_tflops_sustained"], 3),
                         flops_per_launch=d["flops"] // max(1, d["launches"]))
        table[name] = entry
    return table


def cpu_baseline(shape, tokens):
    from oracle import cpu_step  # the checker's eager path, timed on the host cores
    v, threads, desc = cpu_step.time_sample(shape, tokens=tokens)
    return {"value": round(v, 3), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": desc["sample"], "tokens": desc["tokens"], "layer_s": desc["layer_s"],
            "head_s": desc["head_s"]}


def run_reference(args, rank, world):
    """--impl reference: the reference's eager CPU path (the oracle port) on the host cores.
    A step is one bounded sample of the configured step (one decoder layer fwd + checkpoint
    recompute + bwd, and the head + CE, on --cpu-tokens tokens): `steps` counts the samples
    timed and `ms_per_step` is their mean measured wall time; `value` is the whole-model
    tokens/s scaled from them (layers x layer time + head time), reported beside the parts."""
    if rank != 0:
        return
    from hackathon_b200.qlora import preset
    workload, _, _ = WORKLOADS[args.config]
    shape = preset(args.config)
    from oracle import cpu_step
    smp = cpu_step.CpuSample(shape, tokens=args.cpu_tokens)
    for _ in range(args.warmup):
        smp.run()
    steps = max(1, args.steps)
    tl = th = 0.0
    for _ in range(steps):
        a, b = smp.run()
        tl += a
        th += b
    t_layer, t_head = tl / steps, th / steps
    value = smp.scaled_tokens_per_s(t_layer, t_head)
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": steps, "warmup": args.warmup,
            "ms_per_step": round(1e3 * (t_layer + t_head), 1), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": workload, "parallelism": "none (host CPU)",
                       "sample_tokens": args.cpu_tokens},
            "sample": {"what": smp.describe(), "tokens": args.cpu_tokens,
                       "layer_s": round(t_layer, 4), "head_s": round(t_head, 4),
                       "layers_scaled": shape.layers,
                       "scaled_step_s": round(shape.layers * t_layer + t_head, 3),
                       "ms_per_step_is": "the measured wall time of one sample"},
            "cpu_baseline": {"value": round(value, 3), "unit": "tokens/s",
                             "cores": smp.threads, "kind": "port", "sample": smp.describe()},
            "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


KERNELS = ("gemm2", "gemm_dgrad", "nf4_fwd_fused", "nf4_fwd_dequant", "nf4_dgrad_fused",
           "nf4_dequant",
           "dropout_mask", "dropout_apply", "swiglu_fwd", "rmsnorm_fwd", "rmsnorm_bwd",
           "rope_bwd", "linear_ce", "mask_acc", "gateup_swiglu", "gemm2_dgrad_pair",
           "gemm2_rope", "dropout_bits", "lora_xa", "lora_xa_xd", "lora_grads",
           "gateup_swiglu_masks")
GRAPHABLE = ("nf4_dequant", "dropout_mask", "dropout_apply", "swiglu_fwd", "rmsnorm_fwd",
             "rmsnorm_bwd", "rope_bwd", "dropout_bits")


def kernel_case(args):
    """One op of the step on its own at a projection shape (--tokens x --in-features ->
    --out-features), timed with CUDA events over --steps launches after --warmup: the command the
    ncu summaries cite. Inputs are larger than L2 at the default 16384 tokens. `linear_ce` is the
    fused linear cross-entropy (forward + dH) with hidden size --in-features and vocabulary
    --out-features. --graph replays the --steps launches from one CUDA graph (bandwidth kernels
    too short to time behind Python launch gaps)."""
    from hackathon_b200 import _lib
    from hackathon_b200 import nf4 as nf4m
    from hackathon_b200.gemm import device_error, gemm, gemm2
    from hackathon_b200.lora import dropout_apply, dropout_mask
    from hackathon_b200.rmsnorm import rmsnorm
    from hackathon_b200.swiglu import swiglu

    dev = torch.device("cuda", 0)
    T, fo, fi, r = args.tokens, args.out_features, args.in_features, 64
    g = torch.Generator(device=dev).manual_seed(0)

    def rnd(*shape, s=1.0):
        return (torch.randn(*shape, device=dev, generator=g) * s).to(torch.bfloat16)

    name = args.kernel
    flops, nbytes, draws = 0, 0, 0
    if name in ("gemm2", "gemm_dgrad", "nf4_fwd_fused", "nf4_fwd_dequant", "nf4_dgrad_fused",
                "nf4_dequant"):
        packed, st = nf4m.quantize_nf4(rnd(fo, fi, s=0.02))
        w = nf4m.dequantize_nf4(packed, st, torch.bfloat16)
        if name == "gemm2":
            x, u, sb = rnd(T, fi), rnd(T, r), rnd(fo, r, s=0.05)
            fn = lambda: gemm2(x, w, u, sb)  # noqa: E731
            flops = 2 * T * fo * (fi + r)
        elif name == "gemm_dgrad":
            dy = rnd(T, fo)
            fn = lambda: gemm(dy, w.t())  # noqa: E731
            flops = 2 * T * fo * fi
        elif name == "nf4_fwd_fused":
            x, u, sb = rnd(T, fi), rnd(T, r), rnd(fo, r, s=0.05)
            fn = lambda: nf4m.nf4_linear_fwd(x, packed, st, None, u, sb, path="fused")  # noqa
            flops = 2 * T * fo * (fi + r)
        elif name == "nf4_fwd_dequant":
            # the same projection on the long-token path: transient bf16 W, then the TMA GEMM
            x, u, sb = rnd(T, fi), rnd(T, r), rnd(fo, r, s=0.05)
            fn = lambda: nf4m.nf4_linear_fwd(x, packed, st, None, u, sb, path="dequant")  # noqa
            flops = 2 * T * fo * (fi + r)
        elif name == "nf4_dgrad_fused":
            dy = rnd(T, fo)
            fn = lambda: nf4m.nf4_linear_dgrad(dy, packed, st, path="fused")  # noqa: E731
            flops = 2 * T * fo * fi
        else:
            fn = lambda: nf4m.dequantize_nf4(packed, st, torch.bfloat16, out=w)  # noqa: E731
            nbytes = fo * fi // 2 + fo * fi * 2 + fo * fi // 64
    elif name in ("dropout_mask", "dropout_apply"):
        x = rnd(T, fi)
        xd, bits = dropout_mask(x, 0.05, 1234, 1 / 0.95)
        if name == "dropout_mask":
            fn = lambda: dropout_mask(x, 0.05, 1234, 1 / 0.95)  # noqa: E731
        else:
            fn = lambda: dropout_apply(x, bits, 1 / 0.95, out=xd)  # noqa: E731
        nbytes = 2 * T * fi * 2 + bits.numel() * 4
    elif name == "dropout_bits":
        # the mask alone (no data), full grid: Philox draws per second
        from hackathon_b200.lora import dropout_bits
        bits = dropout_bits(T, fi, 0.05, 1234, dev)
        fn = lambda: dropout_bits(T, fi, 0.05, 1234, dev, out=bits)  # noqa: E731
        draws = T * fi
    elif name in ("lora_xa", "lora_xa_xd"):
        # U = dropout(x) A^T from x and the mask bits (rank r); _xd also stores xd
        from hackathon_b200.lora import dropout_bits, lora_xa
        x, a_l = rnd(T, fi), rnd(r, fi, s=0.05)
        bits = dropout_bits(T, fi, 0.05, 1234, dev)
        xd = torch.empty_like(x) if name == "lora_xa_xd" else None
        fn = lambda: lora_xa(x, a_l, bits, 1 / 0.95, xd_out=xd)  # noqa: E731
        nbytes = T * fi * 2 * (2 if xd is not None else 1) + bits.numel() * 4 + T * r * 2
    elif name == "swiglu_fwd":
        gate, up = rnd(T, fo), rnd(T, fo)
        fn = lambda: swiglu(gate, up)  # noqa: E731
        nbytes = 3 * T * fo * 2
    elif name in ("gateup_swiglu", "gemm2_dgrad_pair", "gateup_swiglu_masks"):
        # the MLP pair at intermediate size --out-features: h = silu(g) * u in one GEMM (LoRA
        # terms as extra K), or its input gradient dx = dg W_g + du W_u; `_masks`: the forward's
        # launch, h only, with the side warps drawing a layer's seven masks (six --in-features
        # wide, one --out-features wide, p = 0.05)
        from hackathon_b200.gemm import gemm_gateup_swiglu
        wg, wu = rnd(fo, fi, s=0.02), rnd(fo, fi, s=0.02)
        if name == "gateup_swiglu":
            x, lu = rnd(T, fi), rnd(T, 2 * r)
            bg, bu = rnd(fo, 2 * r, s=0.05), rnd(fo, 2 * r, s=0.05)
            fn = lambda: gemm_gateup_swiglu(x, wg, wu, lu, bg, bu, save_gu=True)  # noqa
            flops = 2 * T * 2 * fo * (fi + 2 * r)
        elif name == "gateup_swiglu_masks":
            x, lu = rnd(T, fi), rnd(T, 2 * r)
            bg, bu = rnd(fo, 2 * r, s=0.05), rnd(fo, 2 * r, s=0.05)
            jobs = [(torch.empty((T, (c + 31) // 32), dtype=torch.int32, device=dev), T, c,
                     1000 + k, 0.05) for k, c in enumerate([fi] * 6 + [fo])]
            fn = lambda: gemm_gateup_swiglu(x, wg, wu, lu, bg, bu, mask_jobs=jobs)  # noqa
            flops = 2 * T * 2 * fo * (fi + 2 * r)
            draws = T * (6 * fi + fo)
        else:
            dg, du = rnd(T, fo), rnd(T, fo)
            fn = lambda: gemm2(dg, wg.t(), du, wu.t())  # noqa: E731
            flops = 2 * T * fi * 2 * fo
    elif name == "gemm2_rope":
        from hackathon_b200.gemm import gemm2_rope
        w, x, u, sb = rnd(fo, fi, s=0.02), rnd(T, fi), rnd(T, r), rnd(fo, r, s=0.05)
        pos = torch.arange(4096, device=dev, dtype=torch.float32)
        inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2, device=dev, dtype=torch.float32) / 128))
        emb = torch.cat([torch.outer(pos, inv)] * 2, dim=-1)
        cos, sin = emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)
        fn = lambda: gemm2_rope(x, w, u, sb, cos, sin)  # noqa: E731
        flops = 2 * T * fo * (fi + r)
    elif name == "lora_grads":
        # the LoRA branch's backward products of one projection: V = g (s B), dA = V^T xd,
        # dB = s g^T U (tcgen05 GEMMs, dA / dB split over the tokens)
        from hackathon_b200.gemm import lora_products
        gy, u, xd, sb = rnd(T, fo), rnd(T, r), rnd(T, fi), rnd(fo, r, s=0.05)
        fn = lambda: lora_products(gy, u, xd, sb, (r, fi), 2.0)  # noqa: E731
        flops = 2 * T * fo * r + 2 * r * fi * T + 2 * fo * r * T
    elif name == "mask_acc":
        # the backward LoRA input-gradient term: dx[T, in] += s * mask .* (V[T, r] A[r, in])
        from hackathon_b200.gemm import gemm_mask_acc
        v, a_l, dx = rnd(T, r), rnd(r, fi, s=0.05), rnd(T, fi)
        _, bits = dropout_mask(dx, 0.05, 7, 1 / 0.95)
        fn = lambda: gemm_mask_acc(v, a_l.t(), bits, 1 / 0.95, dx)  # noqa: E731
        nbytes = 2 * T * fi * 2 + bits.numel() * 4 + T * r * 2 + r * fi * 2
    elif name == "linear_ce":
        from hackathon_b200.cross_entropy import fused_causal_lm_loss
        h = rnd(T, fi).requires_grad_()
        wv = rnd(fo, fi, s=0.02)
        labels = torch.randint(0, fo, (1, T), device=dev, generator=g)
        labels[torch.rand((1, T), device=dev, generator=g) < 0.1] = -100
        fn = lambda: fused_causal_lm_loss(h.view(1, T, fi), wv, labels)  # noqa: E731
        flops = 4 * T * fi * fo        # algorithmic: logits + dH (executed: 6 N H V)
    elif name == "rmsnorm_bwd":
        # dx from dy, x, w and the saved rstd (the C-ABI call the backward makes)
        from hackathon_b200.rmsnorm import bwd_into
        x, wn, dy = rnd(T, fi), rnd(fi), rnd(T, fi)
        rstd = torch.rsqrt(x.float().pow(2).mean(-1) + 1e-6)
        dx = torch.empty_like(x)
        fn = lambda: bwd_into(dy, x, wn, rstd, dx)  # noqa: E731
        nbytes = 3 * T * fi * 2 + fi * 2 + T * 4
    elif name == "rope_bwd":
        # the transposed rotation of the q/k projection outputs as the step applies it (rows of
        # tokens, 128-dim heads, one [S, 128] table; --out-features = heads x 128)
        from hackathon_b200.rope import rope_rows
        S = 4096
        pos = torch.arange(S, device=dev, dtype=torch.float32)
        inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2, device=dev, dtype=torch.float32) / 128))
        emb = torch.cat([torch.outer(pos, inv)] * 2, dim=-1)
        cos, sin = emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)
        g2 = rnd(T, fo)
        fn = lambda: rope_rows(g2, cos, sin, backward=True)  # noqa: E731
        nbytes = 2 * T * fo * 2 + 2 * S * 128 * 2
    else:
        x, wn = rnd(T, fi), rnd(fi)
        fn = lambda: rmsnorm(x, wn, 1e-6)  # noqa: E731
        nbytes = 2 * T * fi * 2 + fi * 2
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    run = fn
    if args.graph:
        if name not in GRAPHABLE:
            raise SystemExit(f"--graph: {name} builds tensor maps on the host per call")
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(args.steps):
                fn()
        run = graph.replay
        run()
        torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    if args.graph:
        run()
    else:
        for _ in range(args.steps):
            run()
    e1.record()
    torch.cuda.synchronize()
    device_error()
    ms = e0.elapsed_time(e1) / args.steps
    pk = peaks()
    line = {"kernel": name, "tokens": T, "in_features": fi, "out_features": fo, "ms": round(ms, 4),
            "graph": bool(args.graph)}
    if draws and not flops:   # integer-pipe work: Philox draws/s, no HBM / tensor peak applies
        line.update(achieved=round(draws / (ms * 1e-3) / 1e9, 1), unit="Gdraws/s",
                    draws_per_launch=draws)
        print(json.dumps(line), flush=True)
        return
    if draws:      # a GEMM that also draws masks in its side warps
        line.update(draws_per_s_g=round(draws / (ms * 1e-3) / 1e9, 1), draws_per_launch=draws)
    if flops:
        tf = flops / (ms * 1e-3) / 1e12
        line.update(achieved=round(tf, 1), unit="TFLOP/s", peak=pk["bf16_tflops"],
                    frac=round(tf / pk["bf16_tflops"], 3), flops_per_launch=flops)
    else:
        gbs = nbytes / (ms * 1e-3) / 1e9
        line.update(achieved=round(gbs, 1), unit="GB/s", peak=pk["hbm_gbs"],
                    frac=round(gbs / pk["hbm_gbs"], 3), bytes_per_launch=nbytes)
    line["peak_source"] = pk["source"] + " (burst)"
    if not args.graph:
        # one more launch with events around every C-ABI call: where the op's time goes
        with _lib.KernelTimer() as kt:
            fn()
        line["calls"] = {k: {"launches": v["launches"], "ms": round(v["ms_total"], 4)}
                         for k, v in kt.summary().items()}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="7b", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--seq", type=int, default=None)
    ap.add_argument("--cpu-tokens", type=int, default=128)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-step", action="store_true",
                    help="print every kernel of one step with its device time (torch.profiler)")
    ap.add_argument("--capture-step", action="store_true",
                    help="after the warm-up, run one step between cudaProfilerStart/Stop and exit "
                         "(for ncu --profile-from-start off)")
    ap.add_argument("--step-deadline", type=float, default=STEP_DEADLINE_S,
                    help="seconds a step may take before the watchdog ends the run (raise it "
                         "under a profiler, which serialises every launch)")
    ap.add_argument("--kernel", default=None, choices=KERNELS,
                    help="time one op of the step alone at a projection shape")
    ap.add_argument("--graph", action="store_true",
                    help="with --kernel: replay the timed launches from one CUDA graph")
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--in-features", type=int, default=3584)
    ap.add_argument("--out-features", type=int, default=3584)
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.kernel:
        kernel_case(args)
        return
    if args.warmup < 3:
        print("bench.py: at least 3 warm-up steps are required", file=sys.stderr)
        args.warmup = 3

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    from hackathon_b200 import _lib
    from hackathon_b200.dp import AdapterGradSync, global_label_count
    from hackathon_b200.qlora import QwenQLoRA, make_optimizer, preset, synthetic_batch, train_step

    workload, batch, seq = WORKLOADS[args.config]
    batch = args.batch or batch
    seq = args.seq or seq
    shape = preset(args.config)
    _phase(f"building the {shape.name} model (NF4 quantisation on the GPU)")
    model = QwenQLoRA(shape, dev, seed=0)
    opt = make_optimizer(model)
    sync = AdapterGradSync(model.adapter_parameters()) if world > 1 else None
    data = [synthetic_batch(shape, batch, seq, dev, seed=1000 * rank + i) for i in range(2)]
    counts = [global_label_count(lb) for _, lb in data]

    def step(i):
        ids, labels = data[i % 2]
        return train_step(model, opt, ids, labels, grad_sync=sync,
                          num_items_in_batch=counts[i % 2])

    def barrier():
        if world > 1:
            dist.barrier()

    lib = _lib.load()
    dog = Watchdog(lib, local, rank, world, args)

    def device_error(where):
        """Reads (and clears) the tensor-core kernels' error flag after the current stream's work,
        agreed over the ranks so that every rank takes the same next step. A raised flag means a
        kernel gave up a bounded wait and left its work undone: the run that raised it ends the
        measurement."""
        rc = lib.qb_device_error(_lib.stream(dev))
        msg = lib.qb_last_error().decode(errors="replace") if rc else None
        if world > 1:
            f = torch.tensor([1 if rc else 0], device=dev)
            dist.all_reduce(f, op=dist.ReduceOp.MAX)
            if int(f[0]) and msg is None:
                msg = "raised on another rank"
        if msg:
            _phase(f"{where}: {msg}")
        return msg

    def synced_step(i):
        step(i)
        torch.cuda.synchronize()

    _phase(f"{args.warmup} warm-up steps")
    try:
        for i in range(args.warmup):
            run_checked(dog.watched(f"warm-up step {i}", args.step_deadline,
                                  lambda: synced_step(i)), device_error, f"warm-up step {i}")
            _phase(f"warm-up step {i} done")
    except RunFailed as e:
        fail(args, world, str(e), monitor_report(lib, local))
        return

    if args.capture_step:
        # one step between cudaProfilerStart / Stop, every thread's launches included (the
        # autograd engine launches the backward from its own thread): the range that
        # `ncu --profile-from-start off` captures for the launch list
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        run_checked(dog.watched("captured step", args.step_deadline, lambda: synced_step(0)),
                    device_error, "captured step")
        torch.cuda.profiler.stop()
        if rank == 0:
            print(json.dumps({"captured_step": workload}), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return

    if args.profile_step:
        # every kernel of one step (ours, cuDNN, cuBLAS, torch) with its device time, from
        # CUPTI via torch.profiler: launches run unserialised, as in the timed region
        from torch.profiler import ProfilerActivity, profile
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            step(0)
            torch.cuda.synchronize()
        rows = [(e.key, e.count, e.device_time_total / 1e3) for e in prof.key_averages()
                if e.device_time_total > 0 and not e.key.startswith("cuda")]
        total = sum(r[2] for r in rows)
        rows.sort(key=lambda r: -r[2])
        if rank == 0:
            print(json.dumps({"profile_step": workload, "device_ms": round(total, 2),
                              "launches": sum(r[1] for r in rows),
                              "kernels": [{"name": k[:160], "launches": c, "ms": round(ms, 3),
                                           "share": round(ms / total, 4)} for k, c, ms in rows]}))
        if world > 1:
            dist.destroy_process_group()
        return

    _phase(f"timing {args.steps} steps")
    # ---- timed region: K steps, inputs resident in HBM (working set >> 126 MB L2)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed_steps():
        with ClockSampler(local) as clocks:
            barrier()
            torch.cuda.synchronize()
            start.record()
            torch.cuda.nvtx.range_push("timed_steps")   # selects these launches in a profiler
            for i in range(args.steps):
                step(i)
            torch.cuda.nvtx.range_pop()
            end.record()
            torch.cuda.synchronize()
            barrier()
        return clocks

    try:
        clocks = run_checked(dog.watched("timed steps", args.step_deadline * (1 + args.steps / 4),
                                       timed_steps), device_error, "timed steps")
    except RunFailed as e:
        fail(args, world, str(e), monitor_report(lib, local))
        return
    ms = start.elapsed_time(end) / args.steps
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t[0])
    tokens_per_step = batch * seq * world
    value = tokens_per_step / (ms * 1e-3)

    _phase(f"{ms:.1f} ms/step; one instrumented step")
    # ---- per-kernel device times inside one step (events around every C-ABI call)
    def instrumented_step():
        barrier()
        with _lib.KernelTimer() as kt:
            step(0)
        return kt.summary()

    try:
        ksum = run_checked(dog.watched("instrumented step", args.step_deadline, instrumented_step),
                         device_error, "instrumented step")
    except RunFailed as e:
        fail(args, world, str(e), monitor_report(lib, local))
        return

    _phase("end-to-end steps through train_step")
    # ---- end to end through the public API: pinned host inputs copied in, loss read back
    host = [(ids.cpu().pin_memory(), lb.cpu().pin_memory()) for ids, lb in data]
    h2d = sum(x.numel() * x.element_size() for x in host[0])
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def e2e_steps():
        barrier()
        torch.cuda.synchronize()
        e0.record()
        for i in range(args.steps):
            ids_h, lb_h = host[i % 2]
            ids = ids_h.to(dev, non_blocking=True)
            lb = lb_h.to(dev, non_blocking=True)
            loss = train_step(model, opt, ids, lb, grad_sync=sync,
                              num_items_in_batch=global_label_count(lb))
            last = float(loss.cpu())           # device -> host read of the step's result
        e1.record()
        torch.cuda.synchronize()
        barrier()
        return last

    try:
        loss_value = run_checked(dog.watched("end-to-end steps",
                                           args.step_deadline * (1 + args.steps / 4), e2e_steps),
                               device_error, "end-to-end steps")
    except RunFailed as e:
        fail(args, world, str(e), monitor_report(lib, local))
        return
    ems = torch.tensor([e0.elapsed_time(e1) / args.steps], device=dev)
    if world > 1:
        dist.all_reduce(ems, op=dist.ReduceOp.MAX)
    e2e = tokens_per_step / (float(ems[0]) * 1e-3)

    pk = peaks()
    table = kernel_table(ksum, pk)
    ours_ms = sum(v["ms_total"] for v in table.values())
    dom_name = max(table, key=lambda k: table[k]["ms_total"]) if table else None
    roofline = None
    if dom_name is not None:
        d = table[dom_name]
        avg_ms = d["ms_total"] / d["launches"]
        if d["bound"] == "hbm":
            per = ksum[dom_name]["bytes"] / d["launches"]
            achieved = per / (avg_ms * 1e-3) / 1e9
            roofline = {"kernel": dom_name, "bound": "hbm", "achieved": round(achieved, 1),
                        "peak": pk["hbm_gbs"], "unit": "GB/s",
                        "frac": round(achieved / pk["hbm_gbs"], 3),
                        "traffic": TRAFFIC_PER_LAUNCH.get(args.config, {}).get(dom_name),
                        "algorithmic_bytes_per_launch": int(per),
                        "peak_source": pk["source"]}
        else:
            per = ksum[dom_name]["flops"] / d["launches"]
            achieved = per / (avg_ms * 1e-3) / 1e12
            roofline = {"kernel": dom_name, "bound": "tensor", "achieved": round(achieved, 1),
                        "peak": pk["bf16_tflops_sustained"], "unit": "TFLOP/s",
                        "frac": round(achieved / pk["bf16_tflops_sustained"], 3),
                        "traffic": TRAFFIC_PER_LAUNCH.get(args.config, {}).get(dom_name),
                        "traffic_source": TRAFFIC_SOURCE,
                        "algorithmic_flops_per_launch": int(per),
                        "peak_source": pk["source"] + " (sustained)"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        _phase("CPU baseline sample")
        cpu = cpu_baseline(shape, args.cpu_tokens)
        _phase("CPU baseline done")

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random token ids, random-init weights quantised to NF4)",
            "config": {"workload": workload, "model": shape.name, "global_batch": batch * world,
                       "seq_len": seq, "parallelism": f"dp{world}", "lora_r": shape.lora_r,
                       "lora_dropout": shape.lora_dropout, "activation_checkpointing": True,
                       "l2": "working set (NF4 weights, activations) far larger than the 126 MB L2"},
            "e2e": {"value": round(e2e, 1), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": 4, "last_loss": round(loss_value, 4)},
            "gpu_launches": sum(v["kernels"] for v in table.values()) * args.steps,
            "roofline": roofline,
            "kernels": table,
            "kernel_ms_per_step_ours": round(ours_ms, 2),
            "cpu_baseline": cpu,
            "clocks": clocks.summary(),
            "peaks": pk,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
