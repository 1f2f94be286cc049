#!/usr/bin/env python3
"""INT8 samples/s and achieved INT8 TOPS of the B200 Npu(Int8) execution provider.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c3c|c3a|c3b|c2|c1|c4|c5]
                    [--impl ours|reference] [--precision int8|fp16|f32] [--weight-quant per_tensor|per_channel]

The default workload is the largest single-GPU configuration, C3c: one fused
INT8 Linear + GELU of 65536 x 4096 x 14336 (a sample is a row of the GEMM).

N > 1 runs under torchrun (one process per GPU).  Weak scaling: every rank
runs its own shard of a global batch of N x per-GPU batch; each Linear's
activation absmax is max-all-reduced over NCCL inside the session's CUDA
graph, so every rank quantizes exactly as one device running the global batch
would.  At N > 1 the line also carries a gather-inclusive figure (each step
followed by the all-gather of every rank's output over NVLink) and
`sharded_bit_exact`: a small global batch run sharded through the library's
NCCL path, gathered, and compared bit for bit with one device running it whole.

`value` times the program on device-resident inputs: the steps are enqueued
back to back as asynchronous runs (a CUDA graph of the program after the
second identical run), CUDA events on the launching stream bracket each run,
L2 is flushed by a 256 MiB write before every timed step, max over ranks.  `e2e` times the public host-buffer call
(InferenceSession.run -> rg_session_run) from pinned memory, H2D and D2H
included.  `--impl reference` times the CPU restatement of the reference
Npu(Int8) path (oracle/, built from oracle/configs.py only) on the host
cores, the reference itself being Rust that this image cannot compile.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "INT8 samples/sec and achieved TOPS vs B200 dense INT8 peak at 1/2/4/8 GPUs"
# --precision fp16: the Npu(Fp16) arm (fp16-rounded operands, f32 sums in k order)
METRIC_FP16 = "FP16 NPU (Npu(Fp16)) samples/sec and achieved f32 FMA TFLOP/s"
# --precision f32: the f32 ExecutionProvider::Cpu arm (run_standard) on the B200
METRIC_F32 = "f32 Cpu-provider (run_standard) samples/sec and achieved f32 FMA TFLOP/s"
L2_FLUSH_BYTES = 256 << 20
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of the
# dominant kernel, taken from a one-pass ncu capture of the same workload.  Each
# figure is a fixed constant tied to the SHA-256 of the kernel source it was
# captured from: once that source changes the line reports null (with the reason)
# instead of a figure that no longer describes the kernel.
MEASURED_TRAFFIC = {
    ("c2", 32768): dict(bytes=102898432 + 146457856, source="rustgears_b200/csrc/k_convblock.cu",
                        sha256="146f0d5bcb7af96aa633b2c7eb863b1ee83598a9b96375c2c08c654d3eecbd14"),
    ("c3c", 65536): dict(bytes=1356924160 + 3707432704, source="rustgears_b200/csrc/k_gemm_tc.cu",
                         sha256="f6f52b72ab4fca4d15a42a851817bd28b3370703d059a12ad0dd32757fa69b73"),
}
NOMINAL_INT8_TOPS = 4500.0


def measured_traffic(cfg: str, units: int):
    t = MEASURED_TRAFFIC.get((cfg, units))
    if t is None:
        return None, "no capture of this workload"
    try:
        with open(os.path.join(ROOT, t["source"]), "rb") as f:
            digest = hashlib.sha256(f.read()).hexdigest()
    except OSError:
        return None, f"{t['source']} not found"
    if digest != t["sha256"]:
        return None, f"{t['source']} changed since the capture"
    return t["bytes"], f"one-pass ncu capture of {os.path.basename(t['source'])} (source sha256 {digest[:12]})"

WORKLOADS = {
    "c2": dict(name="small CNN INT8 (Conv(1,16,3,p1)+BN+ReLU, MaxPool2, Conv(16,32,3,p1)+BN+ReLU, MaxPool2, "
                    "Flatten, Linear(1568,128)+ReLU, Linear(128,10)), x [B,1,28,28] ~ U(0,1)", batch=32768),
    "c1": dict(name="README MLP INT8 (Linear(4,32)+BN1d+ReLU+Linear(32,3)), x [B,4] ~ N(0,1)", batch=65536),
    "c3a": dict(name="fused INT8 Linear+GELU 4096x4096x4096", shape=(4096, 4096, 4096)),
    "c3b": dict(name="fused INT8 Linear+GELU 16384x8192x8192", shape=(16384, 8192, 8192)),
    "c3c": dict(name="fused INT8 Linear+GELU 65536x4096x14336", shape=(65536, 4096, 14336)),
    "c4": dict(name="ResNet-18-shaped INT8 CNN (residual-block IR extension): x [B,3,224,224] ~ N(0,1), "
                    "conv7x7/2 + maxpool3x3/2 (pad 0) + 8 basic blocks + avgpool + Linear(512,1000)", batch=128),
    "c5": dict(name="transformer encoder INT8 (embedding/RMSNorm/attention/SwiGLU IR extension): 12 pre-norm "
                    "layers d_model 1024, 16 heads, SwiGLU hidden 2816, vocab 32000, seq 512, f32 attention",
               batch=64),
}


def build_workload(cfg: str, rank: int, world: int, batch: int | None):
    """(model, x shard, per-GPU units, units name) built with the reference generator."""
    from rustgears_b200 import configs
    w = WORKLOADS[cfg]
    if cfg in ("c1", "c2", "c4", "c5"):
        b = batch or w["batch"]
        fn = {"c1": configs.c1_mlp, "c2": configs.c2_cnn, "c4": configs.c4_resnet18,
              "c5": configs.c5_transformer}[cfg]
        model, x = fn(b, row_offset=rank * b)
        return model, x, b
    m, k, n = w["shape"]
    mb = batch or m
    model, x = configs.c3_linear(m * world, k, n, rows=mb, row_offset=rank * mb)
    return model, x, mb


def calibration_input(cfg: str, units: int, world: int, rank: int, n: int):
    """A calibration batch for --calibrated: n samples drawn right after every rank's
    benchmark shard (disjoint from the measured batch), this rank's n of them."""
    from rustgears_b200 import configs
    off = world * units + rank * n
    if cfg.startswith("c3"):
        _, k, nn_ = WORKLOADS[cfg]["shape"]
        return configs.c3_linear(0, k, nn_, rows=n, row_offset=off)[1]
    fn = {"c1": configs.c1_mlp, "c2": configs.c2_cnn, "c4": configs.c4_resnet18, "c5": configs.c5_transformer}[cfg]
    return fn(n, row_offset=off)[1]


def program_macs(sess, x_shape) -> int:
    import numpy as _np
    one = (1,) + tuple(x_shape[1:])
    sess.run(_np.zeros(one, _np.float32))
    return int(sess.last_npu_profile().total_macs)


class ClockSampler:
    """SM clock, power and clock-event (throttle) reasons of the benchmark GPU, polled
    through NVML every 2 ms while the timed region runs (a timed region of tens of
    milliseconds is too short for nvidia-smi's 100 ms loop)."""

    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4), ("hw_power_brake_slowdown", 0x80))

    def __init__(self, device: int):
        self.device, self.rows, self.h, self.max_mhz = device, [], None, None
        self.stop = threading.Event()

    def __enter__(self):
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            uuid = "GPU-" + str(torch.cuda.get_device_properties(self.device).uuid)
            self.h = pynvml.nvmlDeviceGetHandleByUUID(uuid)
            self.nv = pynvml
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM))
            self._sample()
            self.rows.clear()
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        except Exception:  # no NVML: the line reports no samples
            self.h = None
        return self

    def _sample(self):
        nv = self.nv
        self.rows.append((float(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)),
                          int(nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)),
                          nv.nvmlDeviceGetPowerUsage(self.h) / 1000.0))

    def _run(self):
        while not self.stop.is_set():
            try:
                self._sample()
            except Exception:
                return
            time.sleep(0.002)

    def __exit__(self, *a):
        if self.h is not None:
            self.stop.set()
            self.t.join(timeout=5)

    def summary(self) -> dict:
        sm = [r[0] for r in self.rows]
        reasons = sorted({name for r in self.rows for name, bit in self.REASONS if r[1] & bit})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.rows),
                "power_w_median": float(np.median([r[2] for r in self.rows])) if self.rows else None,
                "source": "NVML, 2 ms poll over the timed region"}


def measured_peaks() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except OSError:
        return {}


def fp32_fma_peak(sms: int, mhz: float) -> float:
    """FP32 FMA rate in TFLOP/s: SMs x 128 FMA/clk x 2 FLOP at the SM clock."""
    return sms * 128 * 2 * mhz * 1e6 / 1e12


def op_roofline(cfg, sess, per_op_ns, steps, x_shape, peaks, traffic=None, fp32_peak=None, i8_out=False):
    """Roofline of the dominant kernel.  A kernel covers one op, or several when the
    library fused them (the fused-away ops report no time).  Algorithmic work: 2 x
    the INT8 MACs; algorithmic bytes: the kernel's f32 input read + f32 output
    written + its i8 weights and f32 biases.  Bound: tensor when ops/bytes exceeds
    the ridge point of the measured peaks, else HBM."""
    prof = sess.last_npu_profile()
    nops = len(prof.records)
    groups, i = [], 0
    while i < nops:
        j = i + 1
        while j < nops and per_op_ns[j] == 0 and prof.records[j].macs >= 0 and sess.op_info(j)["kind"] != 5:
            j += 1
        groups.append((i, j))
        i = j
    gi = int(np.argmax([per_op_ns[a:b].sum() for a, b in groups]))
    a, b = groups[gi]
    dur_s = per_op_ns[a:b].sum() / steps / 1e9
    shapes = _op_shapes(sess, x_shape)
    in_bytes = 4 * int(np.prod(shapes[a][0]))
    # a calibrated producer writes the next Linear's i8 operand: one byte per element
    out_bytes = (1 if i8_out else 4) * int(np.prod(shapes[b - 1][1]))
    wbytes = sum(sess.op_info(k)["wq_len"] + 4 * sess.op_info(k)["bias_len"] for k in range(a, b))
    algo = in_bytes + out_bytes + wbytes
    ops = 2.0 * sum(prof.records[k].macs for k in range(a, b))
    hbm = peaks.get("hbm_gbs", 6650.0)
    int8_peak = 2.0 * peaks.get("bf16_tflops", 1590.0)
    label = " + ".join(prof.records[k].op for k in range(a, b))
    common = {"kernel": label, "ops_per_launch": ops, "algorithmic_bytes": algo, "mean_launch_us": dur_s * 1e6,
              "traffic": traffic}
    if fp32_peak:  # the FP16 arm: f32 FMA chains on the CUDA cores (f32 weights in HBM)
        algo = in_bytes + out_bytes + sum(4 * (sess.op_info(k)["wq_len"] + sess.op_info(k)["bias_len"])
                                          for k in range(a, b))
        common["algorithmic_bytes"] = algo
        if ops / max(algo, 1) > fp32_peak * 1e12 / (hbm * 1e9):
            achieved = ops / dur_s / 1e12
            return dict(common, bound="fp32", achieved=achieved, peak=fp32_peak, unit="TFLOP/s",
                        frac=achieved / fp32_peak,
                        peak_source="FP32 FMA peak: SMs x 128 FMA/clk x 2 at the sampled SM clock "
                                    "(no FP32 figure in MEASURED_PEAKS.json)")
    if ops / max(algo, 1) > int8_peak * 1e12 / (hbm * 1e9):
        achieved = ops / dur_s / 1e12
        return dict(common, bound="tensor", achieved=achieved, peak=int8_peak, unit="TOPS", frac=achieved / int8_peak,
                    peak_source="2 x measured bf16 dense (MEASURED_PEAKS.json) as the INT8 denominator "
                                "(nominal INT8 dense 4500)")
    achieved = algo / dur_s / 1e9
    return dict(common, bound="hbm", achieved=achieved, peak=hbm, unit="GB/s", frac=achieved / hbm,
                peak_source="measured hbm_gbs (MEASURED_PEAKS.json)")


def attention_roofline(x_shape, dev, clocks_summary, reps: int = 5):
    """C5's dominant kernel is the f32 attention (exact FMA order, CUDA-core FMA pipe),
    timed alone through rg_attention_f32 on one layer's shapes with CUDA events on
    the launching stream.  Work: 2 x 64 FMAs per (query, key) per head; peak: the
    FP32 FMA rate (SMs x 128 FMA/clk x 2 FLOP x the SM clock sampled under load),
    no FP32 figure being in MEASURED_PEAKS.json."""
    import ctypes as C

    import torch

    from rustgears_b200 import _native
    b, t = int(x_shape[0]), int(x_shape[1])
    heads, dh = 16, 64
    d = heads * dh
    qkv = torch.randn((b * t, 3 * d), dtype=torch.float32, device=dev)
    out = torch.empty((b * t, d), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    L = _native.lib()
    call = lambda: _native.check(L.rg_attention_f32(C.c_void_p(qkv.data_ptr()), 3 * d, b, t, heads, dh,
                                                    C.c_void_p(out.data_ptr()), d, C.c_void_p(stream.cuda_stream)))
    for _ in range(2):
        call()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    e0.record(stream)
    for _ in range(reps):
        call()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    dur_s = e0.elapsed_time(e1) / reps / 1e3
    flops = 2.0 * 2.0 * b * heads * t * t * dh
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    mhz = clocks_summary.get("sm_mhz") or 1965.0
    peak = sms * 128 * 2 * mhz * 1e6 / 1e12
    achieved = flops / dur_s / 1e12
    return {"kernel": "k_attention64 (f32 QK^T, softmax, P.V; rg_attention_f32)", "bound": "fp32",
            "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
            "mean_launch_us": dur_s * 1e6, "flops_per_launch": flops, "traffic": None,
            "peak_source": f"FP32 FMA peak: {sms} SMs x 128 FMA/clk x 2 at the sampled {mhz:.0f} MHz "
                           "(no FP32 figure in MEASURED_PEAKS.json)",
            "note": "the INT8 projections of the same layers run on the tensor cores (k_gemm_tc)"}


def _op_shapes(sess, x_shape):
    """(input, output) shape of every op for the input shape x_shape; a shortcut conv
    reads and replaces the saved residual-block input."""
    shapes, saved = [], []
    shape = tuple(x_shape)
    for i in range(sess.num_ops()):
        info = sess.op_info(i)
        if info["kind"] == 8:
            saved.append(shape)
        if info["kind"] == 10:
            out = _out_shape(dict(info, kind=2), saved[-1])
            shapes.append((saved[-1], out))
            saved[-1] = out
            continue
        if info["kind"] == 9:
            saved.pop()
        out = _out_shape(info, shape)
        shapes.append((shape, out))
        shape = out
    return shapes


def _out_shape(info, shape):
    k = info["kind"]
    if k == 1:
        return tuple(shape[:-1]) + (info["out_features"],)
    if k == 11:
        return (shape[0], shape[1], info["kernel"], info["stride"])
    if k == 12:
        return tuple(shape) + (info["out_features"],)
    if k == 2:
        n, c, h, w = shape
        oh = (h + 2 * info["padding"] - info["kernel"]) // info["stride"] + 1
        ow = (w + 2 * info["padding"] - info["kernel"]) // info["stride"] + 1
        return (n, info["out_channels"], oh, ow)
    if k == 4:
        n, c, h, w = shape
        return (n, c, (h - info["kernel"]) // info["stride"] + 1, (w - info["kernel"]) // info["stride"] + 1)
    if k == 5:
        return (shape[0], int(np.prod(shape[1:])))
    return shape


def reference_step(cfg: str, prog, layers, x, sample: int, cores: int, precision: int):
    """One step of the CPU restatement of the reference path on `sample` units of the
    workload.  Returns (seconds measured, seconds of it that do not scale with the
    batch).  For C3 the second figure is the reference's serial absmax pass over the
    whole activation (npu.rs:312), timed on its own: a row sample still pays it in full."""
    from oracle import oracle
    if precision == 2:  # the f32 Cpu provider's run_standard (single-threaded restatement)
        t0 = time.perf_counter()
        oracle.run_standard(layers, x[:sample])
        return time.perf_counter() - t0, 0.0
    if cfg.startswith("c3"):
        t0 = time.perf_counter()
        oracle.linear_rows(prog.ops[0], prog, 0, x, 0, 0, nthreads=cores)        # the absmax pass alone
        t_fixed = time.perf_counter() - t0
        t0 = time.perf_counter()
        oracle.linear_rows(prog.ops[0], prog, 0, x, 0, sample, nthreads=cores)   # absmax + `sample` rows
        return time.perf_counter() - t0, t_fixed
    t0 = time.perf_counter()
    prog.execute(x[:sample], nthreads=cores)
    return time.perf_counter() - t0, 0.0


def extrapolate(units: int, sample: int, t: float, t_fixed: float) -> float:
    """Seconds the whole batch of `units` would take: the fixed part once, the rest
    linearly in the number of units (every unit costs the same: same shapes)."""
    return t_fixed + (t - t_fixed) * units / max(sample, 1)


def cpu_baseline(cfg: str, model, x, units: int, target_s: float = 10.0, precision: int = 0):
    """The oracle (CPU restatement of the reference path) on a bounded sample of the
    benchmark batch, with every host core (the reference's rayon decomposition); the
    throughput is extrapolated linearly to the whole batch."""
    from oracle import oracle
    from rustgears_b200.spec import as_dict
    layers = [as_dict(l) for l in model.export()]
    cores = 1 if precision == 2 else (os.cpu_count() or 1)
    prog = None if precision == 2 else oracle.Program(layers, precision)
    c3 = cfg.startswith("c3")
    sample = min(units, 16 if c3 or precision == 2 else {"c4": 2, "c5": 1}.get(cfg, 64))
    t, tf = reference_step(cfg, prog, layers, x, sample, cores, precision)
    per_unit = (t - tf) / sample
    grow = int(min(units, max(sample, (target_s - tf) / max(per_unit, 1e-9))))
    if c3:
        grow = min(grow, 1024)
    if grow > sample and t < target_s / 2:
        sample = grow
        t, tf = reference_step(cfg, prog, layers, x, sample, cores, precision)
    full = extrapolate(units, sample, t, tf)
    what = "rows" if c3 else "samples"
    how = ("og_run_standard, 1 thread" if precision == 2 else
           f"og_op_linear_rows, {cores} threads; the absmax over all {units} rows timed separately"
           if c3 else f"og_execute, {cores} threads")
    return {"value": units / full, "unit": "samples/s (GEMM rows)" if c3 else "samples/s", "cores": cores,
            "kind": "port",
            "sample": f"{sample} of {units} {what} of the benchmark batch ({how}), extrapolated linearly to the batch",
            "sample_seconds": t}


def _reference_workload(cfg: str, units: int, precision: int):
    """The benchmark workload built by the oracle's own generator (oracle/configs.py,
    the CPU restatement of the reference RNG and initialisers): (layers, x, sample).
    The input is drawn after the weights, so the first `sample` units of the batch
    are the first rows of a batch of `sample`; C3 draws the whole activation, whose
    absmax the reference's serial pass covers."""
    from oracle import configs as oc
    c3 = cfg.startswith("c3")
    if c3:
        _, k, n = WORKLOADS[cfg]["shape"]
        layers, x = oc.c3_linear(units, k, n)
        return layers, x, 8 if precision == 2 else 256
    sample = min(units, 16 if precision == 2 else {"c2": 2048, "c4": 4, "c5": 1}.get(cfg, units))
    build = {"c1": oc.c1_mlp, "c2": oc.c2_cnn, "c4": oc.resnet18,
             "c5": lambda b: oc.transformer_c5(batch=b)}[cfg]
    layers, x = build(sample)
    return layers, x, sample


def workload_units(cfg: str, batch):
    w = WORKLOADS[cfg]
    return batch or (w["shape"][0] if cfg.startswith("c3") else w["batch"])


def workload_config(cfg: str, units: int, world: int, weight_quant: str) -> dict:
    c = {"workload": WORKLOADS[cfg]["name"], "global_batch": units * world, "per_gpu_batch": units,
         "parallelism": f"dp{world}", "l2": "flushed before every timed step (256 MiB write)"}
    if cfg.startswith("c3"):
        c["weights"] = f"{weight_quant} symmetric i8"
    return c


def run_reference(args, rank: int, world: int):
    """The reference arm: the CPU restatement of the reference path (oracle/) on the
    host cores, the model and input built by oracle/configs.py alone (no part of the
    product library is loaded).  Each step times a bounded sample of the workload;
    `value` extrapolates it linearly to the whole per-GPU batch."""
    if rank != 0:
        return
    from oracle import oracle
    cfg = args.config
    fp16 = args.precision == "fp16"
    f32 = args.precision == "f32"
    precision = 1 if fp16 else 2 if f32 else 0
    units = workload_units(cfg, args.batch)
    layers, x, sample = _reference_workload(cfg, units, precision)
    wq = 1 if args.weight_quant == "per_channel" else 0
    prog = None if f32 else oracle.Program(layers, precision, weight_quant=wq)
    cores = 1 if f32 else (os.cpu_count() or 1)   # og_run_standard is single-threaded
    c3 = cfg.startswith("c3")
    measured, full = [], []
    for step in range(args.warmup + args.steps):
        t, tf = reference_step(cfg, prog, layers, x, sample, cores, precision)
        if step >= args.warmup:
            measured.append(t + tf)
            full.append(extrapolate(units, sample, t, tf))
    value = units * args.steps / float(np.sum(full))
    unit = "samples/s (GEMM rows)" if c3 else "samples/s"
    path = "Npu(Fp16)" if fp16 else "Cpu provider" if f32 else "Npu(Int8)"
    line = {"metric": METRIC_FP16 if fp16 else METRIC_F32 if f32 else METRIC, "impl": "reference", "value": value,
            "unit": unit, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": float(np.mean(measured)) * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp16" if fp16 else "f32" if f32 else "int8",
            "data": "synthetic (reference generator, manual_seed(42))",
            "config": workload_config(cfg, units, 1, args.weight_quant),
            "sample_per_step": sample,
            "cpu_baseline": {"value": value, "unit": unit, "cores": cores, "kind": "port",
                             "sample": f"{sample} {'rows' if c3 else 'samples'} of the {units}-unit batch per step, "
                                       f"{cores} threads (CPU restatement of the reference {path} path); "
                                       "value extrapolated linearly to the whole batch"
                                       + ("; the absmax pass over every row timed in full each step" if c3 else "")},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_probe(args):
    """Run the workload a few times on cuda:0 and print the last profile."""
    import torch

    from rustgears_b200 import ExecutionProvider, InferenceSession
    model, x, _ = build_workload(args.config, 0, 1, args.batch)
    prov = {"fp16": ExecutionProvider.npu_fp16(), "f32": ExecutionProvider.cpu()}.get(args.precision,
                                                                                       ExecutionProvider.npu_int8())
    sess = InferenceSession.from_module(model, prov, device=0, weight_quant=args.weight_quant,
                                        flags=session_flags(args))
    xd = torch.from_numpy(x).cuda()
    for _ in range(args.steps):
        sess.run_device(xd)
    torch.cuda.synchronize()
    print(sess.last_npu_profile())


def session_flags(args) -> int:
    from rustgears_b200 import _native
    return _native.RG_SESSION_NO_FUSION if args.no_fusion else 0


def int8_library_tops(dev, size: int = 8192, reps: int = 10) -> float:
    """A measured INT8 tensor-core figure on this box: torch._int_mm (cuBLASLt,
    i8 x i8 -> i32, no epilogue) at size^3, best of `reps` launches after warm-up,
    CUDA events on the current stream."""
    import torch
    g = torch.Generator(device=dev).manual_seed(7)
    a = torch.randint(-127, 128, (size, size), dtype=torch.int8, device=dev, generator=g)
    b = torch.randint(-127, 128, (size, size), dtype=torch.int8, device=dev, generator=g)
    for _ in range(3):
        c = torch._int_mm(a, b)
    best = float("inf")
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        c = torch._int_mm(a, b)
        e1.record()
        torch.cuda.synchronize(dev)
        best = min(best, e0.elapsed_time(e1) / 1e3)
    del a, b, c
    return 2.0 * size ** 3 / best / 1e12


def gemm_kernel_roofline(sess, xd, yd, stream, flush, peaks, reps: int = 10):
    """C3's dominant kernel is the fused tcgen05 GEMM (k_gemm_tc); the op's profile time
    also holds its absmax and quantize passes.  The kernel is timed alone here through
    the kernel-level entry point rg_gemm_i8_fused on the session's own quantized
    weights and the quantized activation, with CUDA events on the launching stream,
    L2 flushed before every launch."""
    import ctypes as C

    import torch

    from rustgears_b200 import _native
    L = _native.lib()
    dev = xd.device
    info = sess.op_info(0)
    k, n = info["in_features"], info["out_features"]
    m = xd.numel() // k
    ld = (k + 15) // 16 * 16
    wq, b = sess.op_weights(0)
    w = torch.zeros((n, ld), dtype=torch.int8, device=dev)
    w[:, :k] = torch.from_numpy(wq.reshape(n, k)).to(dev)
    bias = torch.from_numpy(b).to(dev)
    amax = torch.zeros(1, dtype=torch.float32, device=dev)
    scale = torch.zeros(1, dtype=torch.float32, device=dev)
    q = torch.empty((m, ld), dtype=torch.int8, device=dev)
    p = lambda t: C.c_void_p(t.data_ptr())
    st = C.c_void_p(stream.cuda_stream)
    _native.check(L.rg_absmax_f32(p(xd), m * k, p(amax), st))
    _native.check(L.rg_quantize_f32_i8(p(xd), m, k, ld, p(amax), p(q), p(scale), st))
    w_scale = info["w_scale"] if info["w_scale"] > 0 else 1.0 / 127.0   # per-channel: any scale, same work
    call = lambda: _native.check(L.rg_gemm_i8_fused(p(q), p(w), m, n, ld, p(scale), C.c_float(w_scale), p(bias),
                                                    info["act"], C.c_float(info["act_param"]), p(yd), None, None, st))
    call()
    call()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    torch.cuda.synchronize(dev)
    for e0, e1 in evs:
        flush.fill_(3)
        e0.record(stream)
        call()
        e1.record(stream)
    torch.cuda.synchronize(dev)
    dur_s = float(np.mean([e0.elapsed_time(e1) for e0, e1 in evs])) / 1e3
    ops = 2.0 * m * n * k
    int8_peak = 2.0 * peaks.get("bf16_tflops", 1590.0)
    achieved = ops / dur_s / 1e12
    del q, w
    try:
        lib_tops = int8_library_tops(dev)
    except Exception as exc:  # noqa: BLE001 -- a reported reference figure, not the measurement
        lib_tops, lib_err = None, f"{type(exc).__name__}: {exc}"
    else:
        lib_err = None
    return {"kernel": f"k_gemm_tc (tcgen05 kind::i8 GEMM + fused dequant/bias/{'GELU' if info['act'] == 4 else 'act'} "
                      f"epilogue), {m}x{k}x{n}", "bound": "tensor", "achieved": achieved, "peak": int8_peak,
            "unit": "TOPS", "frac": achieved / int8_peak, "frac_of_nominal_int8": achieved / NOMINAL_INT8_TOPS,
            "ops_per_launch": ops, "mean_launch_us": dur_s * 1e6,
            "algorithmic_bytes": m * ld + n * ld + 4 * m * n + 8 * n,
            "peak_source": "2 x measured bf16 dense burst (MEASURED_PEAKS.json) as the INT8 denominator, "
                           "no INT8 figure being in that file (nominal INT8 dense 4500)",
            "timing": f"kernel alone via rg_gemm_i8_fused, mean of {reps} launches, L2 flushed before each",
            "int8_library": {"tops": lib_tops, "frac": achieved / lib_tops if lib_tops else None,
                             "how": "torch._int_mm (cuBLASLt) i8 x i8 -> i32 without epilogue, 8192^3, best of 10, "
                                    "CUDA events, measured in this run" if lib_tops else lib_err}}


def sharded_parity(sess, model, prov, x, weight_quant, rank, world, dev, tdist, per_rank: int, scales=None):
    """A small global batch (the first `per_rank` units of every rank's shard, gathered)
    run sharded through the library's NCCL path -- the per-Linear max all-reduce -- its
    outputs all-gathered by rg_session_allgather, against one device running the whole
    batch without a communicator.  Every rank takes the same collective steps."""
    import torch

    from rustgears_b200 import InferenceSession, dist
    xs = torch.from_numpy(np.ascontiguousarray(x[:per_rank])).to(dev)
    xg = torch.empty((world * per_rank,) + tuple(xs.shape[1:]), dtype=torch.float32, device=dev)
    tdist.all_gather_into_tensor(xg, xs)
    ys = sess.run_device(xs)
    recv = torch.empty((world * ys.numel(),), dtype=torch.float32, device=dev)
    dist.allgather(sess, ys.reshape(-1), recv)
    torch.cuda.synchronize(dev)
    ok = torch.ones(1, dtype=torch.int32, device=dev)
    if rank == 0:
        single = InferenceSession.from_module(model, prov, device=dev.index, weight_quant=weight_quant)
        if scales is not None:
            single.set_calibration(scales)
        yg = single.run_device(xg)
        torch.cuda.synchronize(dev)
        a, b = recv.view(yg.shape), yg
        same = bool(torch.all((a == b) | (torch.isnan(a) & torch.isnan(b))).item())
        ok.fill_(int(same))
        del single
    tdist.broadcast(ok, src=0)
    return bool(ok.item()), world * per_rank


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5, help=">= 3: the graph is captured on the second warm-up run")
    ap.add_argument("--config", default="c3c", choices=sorted(WORKLOADS))
    ap.add_argument("--batch", type=int, default=None, help="per-GPU batch (rows for c3)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--precision", default="int8", choices=["int8", "fp16", "f32"],
                    help="Npu(Int8) (the headline), the Npu(Fp16) arm, or the f32 Cpu provider's arithmetic")
    ap.add_argument("--weight-quant", default="per_tensor", choices=["per_tensor", "per_channel"],
                    help="i8 weight scales: per tensor (the reference) or per output channel (extension)")
    ap.add_argument("--calibrated", action="store_true",
                    help="static calibration (extension): frozen Linear input scales from a calibration batch "
                         "disjoint from the measured one; producers write the Linears' i8 operands")
    ap.add_argument("--no-fusion", action="store_true",
                    help="every op on its own kernel (no fused CNN block or stem): the op-by-op path")
    ap.add_argument("--probe", action="store_true",
                    help="run the workload --steps times and print the profile (for ncu captures; no timing)")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.probe:
        run_probe(args)
        return

    import datetime

    import torch
    import torch.distributed as tdist

    from rustgears_b200 import ExecutionProvider, InferenceSession, dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    cfg = args.config
    c3 = cfg.startswith("c3")
    model, x, units = build_workload(cfg, rank, world, args.batch)
    fp16 = args.precision == "fp16"
    f32 = args.precision == "f32"
    if (fp16 or f32) and cfg in ("c4", "c5"):
        raise SystemExit("the ResNet and transformer extensions run on the INT8 arm only")
    prov = ExecutionProvider.npu_fp16() if fp16 else ExecutionProvider.cpu() if f32 else ExecutionProvider.npu_int8()
    sess = InferenceSession.from_module(model, prov, device=local, weight_quant=args.weight_quant,
                                        flags=session_flags(args))
    if world > 1:
        uid = dist.exchange_unique_id(rank)
        dist.attach(sess, rank, world, uid)
    calib = None
    if args.calibrated:
        if fp16 or f32:
            raise SystemExit("--calibrated is an Npu(Int8) extension")
        n_cal = min(units, {"c3a": 4096, "c3b": 4096, "c3c": 4096, "c4": 16, "c5": 4}.get(cfg, 2048))
        xcal = calibration_input(cfg, units, world, rank, n_cal)
        scales = sess.calibrate(xcal)        # collective at N > 1: the scales cover every rank's batch
        calib = {"samples": int(n_cal * world), "scales": int(scales.size),
                 "how": "frozen per-tensor Linear input scales from a calibration batch drawn after the measured "
                        "one (static-calibration extension; values beyond them clamp)"}
    xd = torch.from_numpy(x).to(dev)
    oshape = sess.output_shape(tuple(x.shape))
    yd = torch.empty(oshape, dtype=torch.float32, device=dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    # one explicit stream for the runs, the L2 flushes and the timing events (a NULL
    # stream handle would send the runs to the session's own stream)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)

    def barrier():
        if world > 1:
            tdist.barrier()
        torch.cuda.synchronize(dev)

    sess.run_device(xd, yd)                            # a synchronous run: error words, launch count
    if f32:  # no NpuProfile: every op but Flatten launches one kernel
        launches_per_run = sum(1 for i in range(sess.num_ops()) if sess.op_info(i)["kind"] != 5)
    else:
        launches_per_run = sess.last_npu_profile().kernel_launches
    # The warm-up runs are the timed loop's own calls (asynchronous, no per-op events):
    # the session captures its CUDA graph on the second of them, so timed steps replay
    # it (a run with profile events is a different program and would be re-captured).
    for _ in range(args.warmup):
        flush.fill_(1)
        sess.run_device(xd, yd, asynchronous=True)
    nops = sess.num_ops()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier()
    with ClockSampler(local) as clocks:
        # Timed steps are enqueued back to back (asynchronous runs: no host sync and no
        # per-op events inside the timed region); events bracket each run on the stream.
        for s in range(args.steps):
            flush.fill_(s & 0xff)                      # 256 MiB write: evicts L2 before each timed step
            evs[s][0].record(stream)
            sess.run_device(xd, yd, asynchronous=True)
            evs[s][1].record(stream)
        barrier()
    launches = launches_per_run * args.steps
    total_ms = float(sum(a.elapsed_time(b) for a, b in evs))
    per_rank_ms = None
    if world > 1:
        t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
        every = torch.empty(world, dtype=torch.float64, device=dev)
        tdist.all_gather_into_tensor(every, t)
        per_rank_ms = [float(v) / args.steps for v in every.tolist()]
        total_ms = max(per_rank_ms) * args.steps
    ms_per_step = total_ms / args.steps

    # gather-inclusive: each step followed by the all-gather of every rank's output
    gather = None
    if world > 1:
        g_steps = max(3, min(args.steps, 10))
        recv = torch.empty((world * yd.numel(),), dtype=torch.float32, device=dev)
        for _ in range(2):
            sess.run_device(xd, yd, asynchronous=True)
            dist.allgather(sess, yd.view(-1), recv)
        barrier()
        gevs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(g_steps)]
        for s in range(g_steps):
            flush.fill_(s & 0xff)
            gevs[s][0].record(stream)
            sess.run_device(xd, yd, asynchronous=True)
            dist.allgather(sess, yd.view(-1), recv)
            gevs[s][1].record(stream)
        barrier()
        g_ms = float(sum(a.elapsed_time(b) for a, b in gevs))
        t = torch.tensor([g_ms], dtype=torch.float64, device=dev)
        tdist.all_reduce(t, op=tdist.ReduceOp.MAX)
        g_ms = float(t.item()) / g_steps
        del recv
        gather = {"value": units * world / (g_ms / 1e3), "ms_per_step": g_ms, "steps": g_steps,
                  "gather_bytes_per_rank": int(yd.numel() * 4 * (world - 1)),
                  "what": "each step's outputs all-gathered to every rank over NVLink (rg_session_allgather, NCCL) "
                          "inside the timed region; compute-only `value` leaves them sharded"}

    # MACs per unit from a one-unit run, before the profiled full-batch runs below: the
    # roofline reads the last profile's per-op MACs, which must be the full batch's
    macs_sess = sess if not f32 else InferenceSession.from_module(model, ExecutionProvider.npu_int8(), device=local)
    macs_unit = program_macs(macs_sess, x.shape) if not c3 else int(np.prod(WORKLOADS[cfg]["shape"][1:]))
    # per-op CUDA-event durations (the roofline's kernel times) from profiled runs
    prof_runs = max(3, min(args.steps, 10))
    per_op_ns = np.zeros(nops)
    for s in range(prof_runs if not f32 else 0):
        flush.fill_(s & 0xff)
        sess.run_device(xd, yd)
        per_op_ns += np.array([r.duration_ns for r in sess.last_npu_profile().records], dtype=np.float64)
    per_op_ns *= args.steps / prof_runs
    units_all = units * world
    value = units_all / (ms_per_step / 1e3)
    tops = value * 2.0 * macs_unit / 1e12

    peaks = measured_peaks()
    clk = clocks.summary()
    fp32_peak = fp32_fma_peak(torch.cuda.get_device_properties(dev).multi_processor_count,
                              clk.get("sm_mhz") or 1965.0) if (fp16 or f32) else None
    traffic, traffic_src = (None, "not captured for this arm") if (fp16 or f32) else measured_traffic(cfg, units)
    if f32:
        roofline = {"kernel": "whole program (the f32 provider records no per-op times)", "bound": "fp32",
                    "achieved": tops, "peak": fp32_peak, "unit": "TFLOP/s", "frac": tops / fp32_peak,
                    "mean_launch_us": ms_per_step * 1e3, "traffic": None,
                    "peak_source": "FP32 FMA peak: SMs x 128 FMA/clk x 2 at the sampled SM clock "
                                   "(no FP32 figure in MEASURED_PEAKS.json)"}
    elif c3 and not fp16:
        roofline = gemm_kernel_roofline(sess, xd, yd, stream, flush, peaks)
        roofline["traffic"] = traffic
        roofline["op_roofline"] = op_roofline(cfg, sess, per_op_ns, args.steps, x.shape, peaks)
    else:
        roofline = op_roofline(cfg, sess, per_op_ns, args.steps, x.shape, peaks, fp32_peak=fp32_peak,
                               traffic=None if calib else traffic, i8_out=bool(calib) and cfg == "c2")
    roofline["traffic_source"] = traffic_src

    # end to end through the public host-buffer call, pinned host memory
    xh = torch.from_numpy(x).pin_memory().numpy()
    yh = torch.empty(oshape, dtype=torch.float32).pin_memory().numpy()
    sess.run(xh, out=yh)
    barrier()
    e2e_steps = max(3, min(args.steps, 10))
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        sess.run(xh, out=yh)
    e2e_s = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
        tdist.all_reduce(t, op=tdist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_value = units_all * e2e_steps / e2e_s

    sharded = None
    if world > 1:
        per_rank = min(units, {"c4": 2, "c5": 1}.get(cfg, 64))
        ok, n_global = sharded_parity(sess, model, prov, x, args.weight_quant, rank, world, dev, tdist, per_rank,
                                      scales=sess.calibration() if calib else None)
        sharded = {"sharded_bit_exact": ok, "global_batch": n_global,
                   "how": "the batch sharded over the ranks through the library's NCCL path (per-Linear max "
                          "all-reduce), outputs all-gathered by rg_session_allgather, compared bit for bit with "
                          "one device running the whole batch"}

    unit = "samples/s (GEMM rows)" if c3 else "samples/s"
    line = {
        "metric": METRIC_FP16 if fp16 else METRIC_F32 if f32 else METRIC, "value": value, "unit": unit,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp16 (round_fp16 operands, f32 FMA sums)" if fp16 else "f32" if f32 else "int8",
        "data": "synthetic (reference generator, manual_seed(42))",
        "config": workload_config(cfg, units, world, args.weight_quant),
        "tops": tops, "tops_frac_of_nominal_int8": None if (fp16 or f32) else tops / NOMINAL_INT8_TOPS,
        "int8_macs_per_unit": macs_unit,
        "roofline": roofline,
        "e2e": {"value": e2e_value, "unit": unit,
                "h2d_bytes_per_step": int(xh.nbytes), "d2h_bytes_per_step": int(yh.nbytes),
                "api": "InferenceSession.run (rg_session_run), pinned host buffers", "steps": e2e_steps},
        "gpu_launches": launches,
        "clocks": clk,
    }
    if per_rank_ms is not None:
        line["per_rank_ms_per_step"] = per_rank_ms   # device time of each rank's timed steps
    if gather is not None:
        line["gather_inclusive"] = gather
    if sharded is not None:
        line["sharded_bit_exact"] = sharded["sharded_bit_exact"]
        line["sharded_check"] = sharded
    if args.no_fusion:
        line["config"]["fusion"] = "off (RG_SESSION_NO_FUSION: every op on its own kernel)"
    if calib:
        line["config"]["calibration"] = calib
        line["roofline"]["traffic_source"] = "no capture of the calibrated workload"
    if fp16:
        line["config"]["precision"] = "Npu(Fp16)"
    if f32:
        line["config"]["precision"] = "Cpu provider (f32 run_standard)"
    if cfg == "c5":
        line["roofline_int8_projections"] = line["roofline"]
        line["roofline"] = attention_roofline(x.shape, dev, line["clocks"])
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg, model, x, units, precision=1 if fp16 else 2 if f32 else 0)
    if rank == 0:
        print(json.dumps(line), flush=True)
    del sess
    if world > 1:
        tdist.destroy_process_group()


if __name__ == "__main__":
    main()
