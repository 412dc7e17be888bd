"""Benchmark of the int8 GEMM path (BASELINE.json metric: Int8Gemm TOPS at 8192^3 s8 x s8 -> s32).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c3|c2|c4|c5|conv|dequant|quant]
                    [--impl ours|reference] [--no-extra]

One step is one Int8Gemm.EncodeInt32 + Submit of the workload (config 3 by default: A int8 [8192 x 8192] x B int8
[8192 x 8192], zero points absent, int32 C) with inputs resident in HBM; L2 is left cold and clean before every step
(a 512 MB write, then a 256 MB read of other data, stream-ordered) and the step itself is timed with CUDA events on
the device stream. With N > 1 (torchrun, one process per GPU) the product is sharded by onegpu_cuda.shard with no
collective in its data path ("strong" scaling: the total work is fixed): a batched workload by batch (rank g computes
its batches from its batches of A and the shared B), the others by 256-column slabs of B (rank g computes its columns
from the full A and its slab of B); times are the max over ranks. The default line also carries, measured in the
same run at the same N, config 5 (`c5`: decode, N-sharded, GB/s against HBM) and config 4 (`c4`: batched QKV,
batch-sharded), and at N > 1 the gather of the sharded result onto rank 0 over NVLink (`gather`, og_comm_gather_columns,
outside `value`). `e2e` runs the same product through the C ABI from pinned host buffers (uploads of the step's inputs
- at N > 1 each rank only its 1/N of the replicated operand, all-gathered over NVLink -, the product, readback of the
rank's result), pipelined over two buffer sets. `--impl reference` times the CPU restatement of the reference's int8
product (oracle/, all host threads) on a bounded row sample of the same workload. Each line also reports
`event_floor_us` (one 1-element kernel flushed and timed like a step: the part of every step no kernel work removes)
and `host` (each rank runs on the CPUs NVML names as nearest its GPU; the CPU baselines get every host thread back).
"""
from __future__ import annotations

import argparse
import contextlib
import functools
import json
import os
import re
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "onegpu-csharp_b200"))

METRIC = "Int8Gemm TOPS at 8192³ s8×s8→s32, % int8 tensor peak, 1/2/4/8 B200"

WORKLOADS = {
    # a: how A is made (s8 / u8 uniform bytes, or DynamicQuantizeLinear of N(0, sigma) floats); zb: the range of the
    # per-column zero points of B (None: no zero points); out: i32 sums, or f32 dequantized by a_scale * b_scale[col]
    "c3": dict(m=8192, n=8192, k=8192, batch=1, a="s8", zb=None, b_lo=-128, out="i32",
               desc="square s8 x s8 -> s32, 8192^3, both operands uniform -128..127, zero points absent"),
    "c2": dict(m=4096, n=4096, k=4096, batch=1, a="dql", sigma=1.0, zb=8, b_lo=-127, out="f32", dql_in_step=True,
               desc="DynamicQuantizeLinear of f32 [4096 x 4096] ~ N(0,1) to u8, then u8 x s8 (per-column zp -8..8) -> "
                    "f32 dequantized by a_scale * b_scale[col], 4096^3; one step = both"),
    "c4": dict(m=2048, n=12288, k=4096, batch=8, a="dql", sigma=0.5, zb=8, b_lo=-127, out="i32",
               desc="batched QKV: u8 A = DynamicQuantizeLinear of N(0, 0.5) over the whole [8, 2048, 4096] tensor (its "
                    "zero point) x shared s8 B [4096 x 12288] -127..127 (per-column zp -8..8) -> s32"),
    "c5": dict(m=16, n=28672, k=8192, batch=1, a="u8", za=128, zb=4, b_lo=-127, out="f32",
               desc="decode: u8 A [16 x 8192] (zp 128) x s8 B [8192 x 28672] -127..127 (per-column zp -4..4), int32 "
                    "sums dequantized to f32 by a_scale 0.02 * b_scale[col] (0.001..0.02) in the product's epilogue"),
}

# The other kernel families of the path (not BASELINE configs): measured the same way, one JSON line each.
FAMILIES = {
    "conv": dict(metric="ConvInteger TOPS", unit="TOPS", bound="tensor",
                 desc="ConvInteger, Whisper-small encoder conv2 at batch 8: u8 x [8, 768, 3000] (zp) * s8 "
                      "[768, 768, 3] (per-channel zp), stride 2, pad 1 -> int32 [8, 768, 1500]",
                 batch=8, cin=768, length=3000, cout=768, kernel=3, stride=2, pad=1),
    "dequant": dict(metric="DequantizeLinear GB/s", unit="GB/s", bound="hbm",
                    desc="DequantizeLinear int8 [8192, 8192] per axis 1 (scale + int8 zero point per column) -> "
                         "float32", shape=[8192, 8192], axis=1),
    "quant": dict(metric="QuantizeLinear GB/s", unit="GB/s", bound="hbm",
                  desc="QuantizeLinear float32 [8192, 8192] ~ N(0, 30) per tensor -> uint8 with zero point 128",
                  shape=[8192, 8192], axis=0),
}


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"bf16_tflops": p.get("bf16_tflops"), "bf16_tflops_sustained": p.get("bf16_tflops_sustained"),
                "hbm_gbs": p.get("hbm_gbs"), "source": "measured"}
    return {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0, "source": "fallback"}


PROFILES = {"c3": "int8_gemm_tc2_c3.md", "c2": "dql_int8_gemm_chain_c2.md", "c4": "int8_gemm_tc2_c4.md",
            "c5": "int8_gemm_rows_c5.md", "dequant": "dequantize_linear_dequant.md",
            "quant": "quantize_linear_quant.md", "conv": "conv_integer_conv.md"}


def profile_traffic(workload: str):
    """Per-launch DRAM bytes (read + write) of the workload's dominant kernel from its committed ncu summary, or
    None when there is no full capture for it."""
    if workload not in PROFILES:
        return None
    path = os.path.join(ROOT, "profiles", PROFILES[workload])
    if not os.path.exists(path):
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", open(path).read())
    return float(m.group(1)) if m else None


def nvml_index(local_rank: int):
    """The NVML handle argument of this rank's GPU (CUDA_VISIBLE_DEVICES may renumber or name them by UUID)."""
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        items = [v.strip() for v in vis.split(",") if v.strip()]
        if local_rank < len(items):
            return items[local_rank]
    return local_rank


class HostBinding:
    """Binds this process's threads to the CPUs NVML names as nearest the rank's GPU (nvmlDeviceSetCpuAffinity, which
    sets the calling thread's CPU affinity and nothing on the GPU), so that the page-locked buffers of the e2e leg are
    allocated on the GPU's own socket. `everywhere()` lends the process all of its original CPUs back for the CPU
    baselines, which use every host thread."""

    def __init__(self, local_rank: int):
        self.original = os.sched_getaffinity(0)
        self.cpus = None
        try:
            import pynvml
            pynvml.nvmlInit()
            idx = nvml_index(local_rank)
            h = (pynvml.nvmlDeviceGetHandleByUUID(idx) if isinstance(idx, str) and idx.startswith(("GPU-", "MIG-"))
                 else pynvml.nvmlDeviceGetHandleByIndex(int(idx)))
            pynvml.nvmlDeviceSetCpuAffinity(h)
            self.bound = os.sched_getaffinity(0)
            self.cpus = len(self.bound)
        except Exception:  # noqa: BLE001 - no NVML or no affinity: the process stays where it was
            self.bound = self.original

    @contextlib.contextmanager
    def everywhere(self):
        os.sched_setaffinity(0, self.original)
        try:
            yield
        finally:
            os.sched_setaffinity(0, self.bound)

    def summary(self):
        return {"cpus_near_gpu": self.cpus, "cpus_total": len(self.original)}


class ClockSampler:
    """SM clock, power and clock-event (throttle) reasons of one GPU, read through NVML every 5 ms while the timed
    region runs (read-only queries; nothing is set)."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4,
               "hw_power_brake_slowdown": 0x80}

    def __init__(self, local_rank: int):
        self.rank = local_rank
        self.samples = []
        self.stop = threading.Event()
        self.ok = False

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            idx = nvml_index(self.rank)
            self.h = (pynvml.nvmlDeviceGetHandleByUUID(idx) if isinstance(idx, str) and idx.startswith(("GPU-", "MIG-"))
                      else pynvml.nvmlDeviceGetHandleByIndex(int(idx)))
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.nv = pynvml
            self.ok = True
            self.thread = threading.Thread(target=self._run, daemon=True)
            self.thread.start()
            t0 = time.time()
            while not self.samples and time.time() - t0 < 2.0:
                time.sleep(0.005)
        except Exception:  # noqa: BLE001 - no NVML: the line says "unsampled"
            self.ok = False
        return self

    def _run(self):
        nv = self.nv
        while not self.stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                watts = nv.nvmlDeviceGetPowerUsage(self.h) / 1000.0
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((mhz, watts, reasons))
            except Exception:  # noqa: BLE001
                pass
            time.sleep(0.005)

    def __exit__(self, *exc):
        self.stop.set()
        if self.ok:
            self.thread.join(timeout=1.0)

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        reasons = sorted({name for _, _, r in self.samples for name, bit in self.REASONS.items() if r & bit})
        return {"sm_mhz": statistics.median(s[0] for s in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.samples),
                "power_w_max": round(max(s[1] for s in self.samples), 1)}


def cpu_gemm_tops(n: int, k: int, threads: int, target_s: float, max_rows: int, seed: int = 0, tiled: bool = False):
    """Times the oracle's threaded restatement of the reference's int8 product (Int8Tests.Reference; with `tiled`, the
    same sums through the reference portable kernel's 64 x 64 x 16 blocking, Int8GemmKernel.hlsl) on a sample of rows
    of A against the whole B, sized to about `target_s` seconds; returns (TOPS, seconds, rows)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import og_oracle as oracle

    b = oracle.bytes_(k * n, seed + 31)
    rows = 64 if tiled else 4  # the tiled form computes whole 64-row tiles
    while True:
        a = oracle.bytes_(rows * k, seed + 30)
        t0 = time.perf_counter()
        oracle.int8_gemm(a, True, b, True, m=rows, n=n, k=k, threads=threads, tiled=tiled)
        dt = time.perf_counter() - t0
        if dt >= 0.5 * target_s or rows >= max_rows:
            return 2.0 * rows * n * k / dt / 1e12, dt, rows
        rows = int(min(max_rows, max(rows * 2, rows * target_s / max(dt, 1e-3) * 0.9)))
        if tiled:
            rows = max(64, rows // 64 * 64)


class L2Flush:
    """Leaves L2 cold and clean before a timed step: a 512 MB write evicts the workload's lines, then a 256 MB read
    of other data evicts the write's dirty lines (their write-back happens here, outside the timed region, instead of
    inside the first kernel of the step). Runs on the library device's own stream, so it is stream-ordered before
    the step without host synchronisation."""

    def __init__(self, dev, local_rank: int):
        import torch

        self.torch = torch
        d = torch.device(f"cuda:{local_rank}")
        self.stream = torch.cuda.ExternalStream(dev.stream, device=d)
        self.write = torch.empty(512 << 20, dtype=torch.uint8, device=d)
        self.read = torch.ones((256 << 20) // 4, dtype=torch.float32, device=d)
        self.sink = torch.empty((), dtype=torch.float32, device=d)
        torch.cuda.synchronize(d)

    def __call__(self, i: int = 0) -> None:
        with self.torch.cuda.stream(self.stream):
            self.write.fill_(i & 0xFF)
            self.torch.sum(self.read, dim=0, out=self.sink)

    DESCRIPTION = "flushed before every step (512 MB write, then a 256 MB read of other data so that no dirty line " \
                  "remains), steps timed by CUDA events"


@functools.lru_cache(maxsize=None)
def family_inputs(name: str):
    """Seeded synthetic inputs of a family workload (host arrays, made once) and its algorithmic work per step."""
    f = FAMILIES[name]
    rng = np.random.default_rng(77)
    if name == "conv":
        B, C, L, O, Kw = f["batch"], f["cin"], f["length"], f["cout"], f["kernel"]
        ow = (L + 2 * f["pad"] - Kw) // f["stride"] + 1
        x = rng.integers(0, 256, size=B * C * L, dtype=np.int16).astype(np.uint8)
        w = rng.integers(-127, 128, size=O * C * Kw, dtype=np.int16).astype(np.int8)
        wz = rng.integers(-8, 9, size=O, dtype=np.int16).astype(np.int8)
        return dict(x=x, w=w, xz=np.array([128, 0, 0, 0], np.uint8), wz=wz, ow=ow,
                    work=2.0 * B * O * ow * C * Kw, y_elems=B * O * ow)
    shape = f["shape"]
    count = int(np.prod(shape))
    if name == "dequant":
        x = rng.integers(-128, 128, size=count, dtype=np.int16).astype(np.int8)
        scale = rng.uniform(0.001, 0.02, size=shape[1]).astype(np.float32)
        zp = rng.integers(-8, 9, size=shape[1], dtype=np.int16).astype(np.int8)
        return dict(x=x, scale=scale, zp=zp, count=count, work=5.0 * count)
    x = (rng.standard_normal(count, dtype=np.float32) * np.float32(30.0))
    return dict(x=x, scale=np.array([0.25], np.float32), zp=np.array([128, 0, 0, 0], np.uint8), count=count,
                work=5.0 * count)


_CONV_SAMPLE = {}  # target seconds -> output channels of the ConvInteger sample


def cpu_family(name: str, threads: int, target_s: float):
    """The oracle's restatement of the reference's CPU definition on a bounded sample: (value, cores, sample)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import og_oracle as oracle

    f = FAMILIES[name]
    d = family_inputs(name)
    if name == "conv":
        # One image; as many output channels as fit the target time (found once by doubling from 8).
        one = d["x"][: f["cin"] * f["length"]]
        cout = _CONV_SAMPLE.get(target_s, 8)
        while True:
            p = dict(batch=1, cin=f["cin"], h=1, w=f["length"], cout=cout, kh=1, kw=f["kernel"], stride_h=1,
                     stride_w=f["stride"], pad_left=f["pad"], pad_right=f["pad"])
            t0 = time.perf_counter()
            oracle.conv_integer(p, one, False, d["w"][: cout * f["cin"] * f["kernel"]], True, d["xz"][:1],
                                d["wz"][:cout], True, threads=threads)
            dt = time.perf_counter() - t0
            if dt >= 0.5 * target_s or cout >= f["cout"] or target_s in _CONV_SAMPLE:
                break
            cout = min(f["cout"], cout * 2)
        _CONV_SAMPLE[target_s] = cout
        work = d["work"] / f["batch"] * cout / f["cout"]
        return work / dt / 1e12, threads, f"{cout} of {f['cout']} output channels of 1 of {f['batch']} images " \
            f"({dt:.2f} s), direct convolution og_oracle_conv_integer (restates ConvIntegerTests.Reference) on " \
            f"{threads} threads"
    n = min(d["count"], 1 << 23)
    t0 = time.perf_counter()
    reps = 0
    while True:
        if name == "dequant":
            oracle.dequantize(d["x"][:n], [n // f["shape"][1], f["shape"][1]], 1, True, d["scale"], d["zp"])
        else:
            oracle.quantize(d["x"][:n], [n], 0, False, d["scale"], d["zp"][:1])
        reps += 1
        dt = time.perf_counter() - t0
        if dt >= target_s:
            break
    return 5.0 * n * reps / dt / 1e9, 1, f"{reps} x {n} elements ({dt:.1f} s) through the oracle's scalar " \
        f"restatement of the reference's CPU definition, 1 thread"


def run_family_reference(args, rank: int, world: int):
    if rank != 0:
        return
    f = FAMILIES[args.workload]
    threads = os.cpu_count() or 1
    values, cores, sample = [], 1, ""
    for _ in range(args.warmup):
        cpu_family(args.workload, threads, 0.05)
    per_step = min(args.cpu_seconds, max(0.01, REFERENCE_SECONDS / max(args.steps, 1)))
    for _ in range(args.steps):
        v, cores, sample = cpu_family(args.workload, threads, per_step)
        values.append(v)
    v = statistics.median(values)
    d = family_inputs(args.workload)
    line = {"metric": f["metric"], "impl": "reference", "value": round(v, 6), "unit": f["unit"], "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(d["work"] / (v * (1e12 if f["unit"] == "TOPS" else 1e9)) * 1e3, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "data": "synthetic",
            "dtype": "int8" if args.workload == "conv" else "f32/u8",
            "config": {"workload": f"{args.workload}: {f['desc']}", "parallelism": "host threads"},
            "cpu_baseline": {"value": round(v, 6), "unit": f["unit"], "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(v, 6), "unit": f["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_family(args, rank: int, world: int, local_rank: int):
    """One step = one encode + submit of the family's operation on inputs resident in HBM, L2 flushed before it."""
    import ctypes

    import onegpu_cuda as og

    if world > 1:
        raise SystemExit(f"{args.workload} is measured on one GPU")
    f = FAMILIES[args.workload]
    d = family_inputs(args.workload)
    host = HostBinding(local_rank)
    dev = og.GpuDevice(local_rank)
    bufs = []

    def buf(dtype, data_or_len):
        b = dev.create_buffer(dtype, data_or_len)
        bufs.append(b)
        return b

    if args.workload == "conv":
        problem = og.ConvProblem.conv1d(f["batch"], f["cin"], f["length"], f["cout"], f["kernel"], stride=f["stride"],
                                        pad_begin=f["pad"], pad_end=f["pad"])
        x, w = buf(np.uint8, d["x"]), buf(np.int8, d["w"])
        xz, wz = buf(np.uint8, d["xz"]), buf(np.int8, d["wz"])
        y = buf(np.int32, d["y_elems"])
        op = og.ConvIntegerKernels(dev)
        inputs, outputs = [(x, d["x"])], [(y, d["y_elems"] * 4)]

        def encode(enc):
            op.encode(enc, problem, x, w, y, og.Int8Operand(xz, 0), og.Int8Operand(wz, 0, True))
    else:
        op = og.DequantizeKernels(dev)
        shape = f["shape"]
        if args.workload == "dequant":
            x, s, z = buf(np.int8, d["x"]), buf(np.float32, d["scale"]), buf(np.int8, d["zp"])
            y = buf(np.float32, d["count"])
            outputs = [(y, d["count"] * 4)]

            def encode(enc):
                op.encode(enc, x, 0, shape, f["axis"], True, s, 0, z, 0, y, 0)
        else:
            x, s, z = buf(np.float32, d["x"]), buf(np.float32, d["scale"]), buf(np.uint8, d["zp"])
            y = buf(np.uint8, d["count"])
            outputs = [(y, d["count"])]

            def encode(enc):
                op.encode_quantize(enc, x, 0, shape, f["axis"], False, s, 0, z, 0, y, 0)
        inputs = [(x, d["x"])]

    flush = L2Flush(dev, local_rank)
    stamps = og.GpuTimestampSet(dev, 2 * args.steps)

    def step(i=None):
        flush(i if i is not None else 0)
        enc = dev.begin_commands()
        if i is not None:
            enc.write_timestamp(stamps, 2 * i)
        encode(enc)
        if i is not None:
            enc.write_timestamp(stamps, 2 * i + 1)
        n = enc.dispatch_count
        dev.submit(enc)
        return n

    for _ in range(args.warmup):
        step()
    dev.wait_idle()
    launches = 0
    with ClockSampler(local_rank) as clocks:
        t0 = time.perf_counter()
        for i in range(args.steps):
            launches += step(i)
        dev.wait_idle()
        wall = time.perf_counter() - t0
    ts = stamps.read(0)
    per_step = [ts[2 * i + 1] - ts[2 * i] for i in range(args.steps)]
    total_ns = sum(per_step)
    floor_us = event_floor_us(dev, og, flush)
    scale_unit = 1e12 if f["unit"] == "TOPS" else 1e9
    value = d["work"] * args.steps / (total_ns * 1e-9) / scale_unit

    # e2e: the same operation through the C ABI from pinned host memory, inputs uploaded and outputs read back.
    h2d = sum(a.nbytes for _, a in inputs)
    d2h = sum(n for _, n in outputs)
    pin = ctypes.c_void_p()
    og._check(og._lib.og_host_alloc(h2d + d2h, ctypes.byref(pin)))
    off = 0
    for _, a in inputs:
        ctypes.memmove(pin.value + off, a.ctypes.data, a.nbytes)
        off += a.nbytes
    e2e_steps = min(args.steps, 20)
    e2e_stamps = og.GpuTimestampSet(dev, 2 * e2e_steps)
    for i in range(-1, e2e_steps):
        if i >= 0:
            dev.timestamp(e2e_stamps, 2 * i)
        off = 0
        for b, a in inputs:
            og._check(og._lib.og_buffer_write(dev.handle, b.ptr, pin.value + off, a.nbytes))
            off += a.nbytes
        enc = dev.begin_commands()
        encode(enc)
        dev.submit(enc)
        for b, n in outputs:
            og._check(og._lib.og_buffer_read(dev.handle, pin.value + h2d, b.ptr, n))
        if i >= 0:
            dev.timestamp(e2e_stamps, 2 * i + 1)
    ets = e2e_stamps.read(0)
    e2e_ns = sum(ets[2 * i + 1] - ets[2 * i] for i in range(e2e_steps)) / e2e_steps
    og._check(og._lib.og_host_free(pin))

    peaks = load_peaks()
    sustained = total_ns * 1e-9 > 1.0 or wall > 1.0
    if f["bound"] == "tensor":
        peak = 2.0 * (peaks["bf16_tflops_sustained"] if sustained else peaks["bf16_tflops"])
        roof = {"bound": "tensor", "unit": "TOPS", "peak_source": f"2 x {peaks['source']} dense bf16 "
                f"{'sustained' if sustained else 'burst'}: the int8 dense rate is twice bf16 on B200"}
    else:
        peak = peaks["hbm_gbs"]
        roof = {"bound": "hbm", "unit": "GB/s", "peak_source": f"{peaks['source']} HBM copy bandwidth"}
    achieved = d["work"] / (statistics.mean(per_step) * 1e-9) / scale_unit
    roof.update({"achieved": round(achieved, 3), "peak": round(peak, 1), "frac": round(achieved / peak, 4),
                 "traffic": profile_traffic(args.workload)})
    cpu = None
    if not args.no_cpu:
        with host.everywhere():
            v, cores, sample = cpu_family(args.workload, os.cpu_count() or 1, args.cpu_seconds)
        cpu = {"value": round(v, 6), "unit": f["unit"], "cores": cores, "kind": "port", "sample": sample}
    line = {"metric": f["metric"], "value": round(value, 3), "unit": f["unit"], "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(total_ns / args.steps / 1e6, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8" if args.workload == "conv" else "f32/u8",
            "data": "synthetic",
            "config": {"workload": f"{args.workload}: {f['desc']}", "parallelism": "single GPU",
                       "l2": L2Flush.DESCRIPTION},
            "roofline": roof, "cpu_baseline": cpu,
            "e2e": {"value": round(d["work"] / (e2e_ns * 1e-9) / scale_unit, 3), "unit": f["unit"],
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h)},
            "gpu_launches": int(launches), "event_floor_us": floor_us, "clocks": clocks.summary(),
            "host": host.summary(), "wall_s": round(wall, 3)}
    print(json.dumps(line), flush=True)
    op.dispose()
    stamps.dispose()
    e2e_stamps.dispose()
    for b in bufs:
        b.dispose()
    dev.dispose()


def run_reference(args, rank: int, world: int):
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import og_oracle as oracle

    w = WORKLOADS[args.workload]
    threads = os.cpu_count() or 1
    n, k = w["n"], w["k"]
    # Every step is the same bounded sample (rows of A against the whole B), sized so that the K steps together take
    # about REFERENCE_SECONDS (at most args.cpu_seconds each); B and the rows are made once.
    per_step = min(args.cpu_seconds, max(0.01, REFERENCE_SECONDS / max(args.steps, 1)))
    b = oracle.bytes_(k * n, 31)
    rows = 4
    for _ in range(6):  # calibration (part of the warm-up)
        a = oracle.bytes_(rows * k, 30)
        t0 = time.perf_counter()
        oracle.int8_gemm(a, True, b, True, m=rows, n=n, k=k, threads=threads)
        dt = time.perf_counter() - t0
        if 0.7 * per_step <= dt <= 1.4 * per_step or rows >= w["m"]:
            break
        rows = int(min(w["m"], max(1, rows * per_step / max(dt, 1e-4))))
    a = oracle.bytes_(rows * k, 30)
    for _ in range(args.warmup):
        oracle.int8_gemm(a, True, b, True, m=rows, n=n, k=k, threads=threads)
    values = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        oracle.int8_gemm(a, True, b, True, m=rows, n=n, k=k, threads=threads)
        values.append(2.0 * rows * n * k / (time.perf_counter() - t0) / 1e12)
    tops = statistics.median(values)
    full_ms = 2.0 * w["batch"] * w["m"] * w["n"] * w["k"] / (tops * 1e12) * 1e3
    sample = (f"{rows} of {w['m']} rows of A against the full B ({w['n']} x K {w['k']}) per step, extrapolated; "
              f"oracle og_oracle_int8_gemm (restates Int8Tests.Reference) on {threads} threads")
    line = {"metric": METRIC, "impl": "reference", "value": round(tops, 6), "unit": "TOPS", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(full_ms, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": f"{args.workload}: {w['desc']}", "m": w["m"], "n": w["n"], "k": w["k"],
                       "batch": w["batch"], "parallelism": "host threads", "sample": sample},
            "cpu_baseline": {"value": round(tops, 6), "unit": "TOPS", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(tops, 6), "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


REFERENCE_SECONDS = 120.0  # the reference arm's timed steps together, whatever --steps is


class Workload:
    """One rank's part of a BASELINE config, resident in HBM: its shard of the operands (batched products by batch with
    B shared; the others by 256-column slabs of B, A replicated), the output, and how to record one step."""

    def __init__(self, og, sh, dev, name: str, world: int, rank: int, seed: int = 1234):
        w = WORKLOADS[name]
        self.name, self.w = name, w
        self.M, self.N, self.K, self.B = M, N, K, B = w["m"], w["n"], w["k"], w["batch"]
        self.by_batch = B > 1
        extent, align = (B, 1) if self.by_batch else (N, sh.TILE_COLUMNS)
        self.shards = sh.split(extent, world, align)
        if min(s.width for s in self.shards) == 0:  # decided alike on every rank
            raise SystemExit(f"{name} has fewer shards than the {world} ranks")
        self.part = part = self.shards[rank]
        self.shard_n = N if self.by_batch else part.width
        self.B_local = part.width if self.by_batch else B
        self.dev = dev
        rng = np.random.default_rng(seed)
        self.bufs, self.extra = {}, []
        self.dq = None
        a_kind = w["a"]
        self.a_dtype = np.int8 if a_kind == "s8" else np.uint8
        # B (K x N, row-major): every rank draws the whole operand from one seed and keeps its shard.
        b_full = rng.integers(w["b_lo"], 128, size=(K, N), dtype=np.int16)
        self.b_host = (b_full if self.by_batch else sh.column_slab(b_full, part)).astype(np.int8).reshape(-1)
        del b_full
        self.bufs["b"] = dev.create_buffer(np.int8, self.b_host)
        zp = None
        if a_kind == "dql":
            # float activations ~ N(0, sigma) quantized by this library's DynamicQuantizeLinear over the whole tensor
            x = (rng.standard_normal(size=B * M * K, dtype=np.float32) * np.float32(w["sigma"]))
            self.x_host = x
            self.bufs["x"] = dev.create_buffer(np.float32, x)
            self.bufs["a"] = dev.create_buffer(np.uint8, B * M * K)
            self.a_scale = dev.create_buffer(np.float32, 1)
            self.za = dev.create_buffer(np.uint8, 4)
            self.extra += [self.a_scale, self.za]
            self.dq = og.DynamicQuantizeKernels(dev)
            enc = dev.begin_commands()
            self.dq.encode(enc, self.bufs["x"], 0, B * M * K, self.bufs["a"], 0, self.a_scale, 0, self.za, 0)
            dev.submit(enc)
            dev.wait_idle()
            self.a_zero_point = int(self.za.read()[0])
            if not w.get("dql_in_step"):
                self.a_host = self.bufs["a"].read()  # what the e2e leg uploads
                if self.by_batch:
                    self.a_host = self.a_host.reshape(B, M * K)[part.start:part.stop].reshape(-1)
                    self.bufs["a"].dispose()
                    self.bufs["a"] = dev.create_buffer(np.uint8, self.a_host)
                self.bufs["x"].dispose()
                del self.bufs["x"]
                self.x_host = None
        else:
            lo, hi = (-128, 128) if a_kind == "s8" else (0, 256)
            a_full = rng.integers(lo, hi, size=(B, M, K), dtype=np.int16).astype(self.a_dtype)
            self.a_host = (sh.batch_slab(a_full, part) if self.by_batch else a_full).reshape(-1)
            del a_full
            self.bufs["a"] = dev.create_buffer(self.a_dtype, self.a_host)
            self.x_host = None
            if "za" in w:
                self.za = dev.create_buffer(np.uint8, np.array([w["za"], 0, 0, 0], np.uint8))
                self.extra.append(self.za)
                self.a_zero_point = w["za"]
        self.zpa = og.Int8Operand(self.za, 0) if (a_kind == "dql" or "za" in w) else None
        self.zpb = None
        if w["zb"] is not None:
            zb_full = rng.integers(-w["zb"], w["zb"] + 1, size=N).astype(np.int8)
            zb = zb_full if self.by_batch else sh.column_vector(zb_full, part)
            self.zb = dev.create_buffer(np.int8, zb)
            self.extra.append(self.zb)
            self.zpb = og.Int8Operand(self.zb, 0, True)
        self.count = self.B_local * M * self.shard_n
        self.out_dtype = np.float32 if w["out"] == "f32" else np.int32
        self.bufs["c"] = dev.create_buffer(self.out_dtype, self.count)
        if w["out"] == "f32":
            if a_kind != "dql":
                self.a_scale = dev.create_buffer(np.float32, np.array([0.02], np.float32))
                self.extra.append(self.a_scale)
            bs_full = rng.uniform(0.001, 0.02, size=N).astype(np.float32)
            self.b_scale = dev.create_buffer(np.float32, bs_full if self.by_batch else sh.column_vector(bs_full, part))
            self.extra.append(self.b_scale)
        self.problem = og.Int8GemmProblem(M, self.shard_n, K, batch=self.B_local,
                                          stride_a=M * K if self.B_local > 1 else 0, stride_b=0)
        self.gemm = og.Int8Gemm(dev)
        self.og = og
        self.ops_total = 2.0 * B * M * N * K
        self.ops_shard = 2.0 * self.B_local * M * self.shard_n * K
        # Bytes one launch must move at least: A, the B slab, C, and the zero-point / scale vectors (plus, for the
        # config-2 step, x read and A written by DynamicQuantizeLinear and read again by the product).
        self.algo_bytes = (self.B_local * M * K + K * self.shard_n + self.count * np.dtype(self.out_dtype).itemsize
                           + (self.shard_n if w["zb"] is not None else 0)
                           + (4 * self.shard_n if w["out"] == "f32" else 0)
                           + (4 * M * K + 2 * M * K if w.get("dql_in_step") else 0))

    @property
    def first_host(self):
        """What a step's upload starts with: x for the config-2 chain, A otherwise."""
        return self.x_host if self.w.get("dql_in_step") else self.a_host

    def encode(self, enc, a=None, b=None, c=None, x=None):
        og = self.og
        a = a or self.bufs["a"]
        b = b or self.bufs["b"]
        c = c or self.bufs["c"]
        if self.w.get("dql_in_step"):
            self.dq.encode(enc, x or self.bufs["x"], 0, self.M * self.K, a, 0, self.a_scale, 0, self.za, 0)
        if self.w["out"] == "f32":
            self.gemm.encode_dequantize(enc, self.problem, a, b, c, og.Int8Operand(self.a_scale, 0),
                                        og.Int8Operand(self.b_scale, 0, True), self.zpa, self.zpb)
        else:
            self.gemm.encode_int32(enc, self.problem, a, b, c, self.zpa, self.zpb)

    def dispose(self):
        for v in list(self.bufs.values()) + self.extra:
            v.dispose()
        if self.dq is not None:
            self.dq.dispose()
        self.gemm.dispose()


def event_floor_us(dev, og, flush, reps: int = 12) -> float:
    """The part of every timed step that no kernel work removes: one 1-element torch kernel, flushed and bracketed by
    CUDA events exactly like a step, median over `reps` (on B200 an event pair alone is ~2.6 us and the first kernel
    after an event adds ~3.5 us more)."""
    stamps = og.GpuTimestampSet(dev, 2 * reps)
    for i in range(reps):
        flush(i)
        dev.timestamp(stamps, 2 * i)
        with flush.torch.cuda.stream(flush.stream):
            flush.sink.zero_()
        dev.timestamp(stamps, 2 * i + 1)
    ts = stamps.read(0)
    stamps.dispose()
    return round(statistics.median(ts[2 * i + 1] - ts[2 * i] for i in range(reps)) / 1e3, 2)


def timed_steps(dev, og, flush, wl: Workload, steps: int, warmup: int, barrier=None):
    """Runs `warmup` untimed and `steps` timed steps (L2 flushed before each, CUDA events around the step on the
    device stream); returns the per-step nanoseconds and the number of kernel launches recorded in the timed steps."""
    stamps = og.GpuTimestampSet(dev, 2 * steps)

    def step(i=None):
        flush(i if i is not None else 0)
        enc = dev.begin_commands()
        if i is not None:
            enc.write_timestamp(stamps, 2 * i)
        wl.encode(enc)
        if i is not None:
            enc.write_timestamp(stamps, 2 * i + 1)
        n = enc.dispatch_count
        dev.submit(enc)
        return n

    for _ in range(warmup):
        step()
    dev.wait_idle()
    if barrier is not None:
        barrier()
    launches = 0
    t0 = time.perf_counter()
    for i in range(steps):
        launches += step(i)
    dev.wait_idle()
    wall = time.perf_counter() - t0
    if barrier is not None:
        barrier()
    ts = stamps.read(0)
    stamps.dispose()
    return [ts[2 * i + 1] - ts[2 * i] for i in range(steps)], launches, wall


def roofline_peaks(clk: dict, sustained_time: bool):
    """The int8 tensor denominator: twice the measured dense bf16 rate, the sustained figure when the run's own clock
    record shows the power cap (or the timed region is long enough to reach it), the burst figure otherwise."""
    peaks = load_peaks()
    capped = "sw_power_cap" in (clk.get("reasons") or [])
    sustained = capped or sustained_time
    burst, sust = 2.0 * peaks["bf16_tflops"], 2.0 * peaks["bf16_tflops_sustained"]
    return peaks, (sust if sustained else burst), ("sustained" if sustained else "burst"), burst, sust, capped


def run_ours(args, rank: int, world: int, local_rank: int, dist):
    import onegpu_cuda as og

    from onegpu_cuda import shard as sh

    host = HostBinding(local_rank)
    dev = og.GpuDevice(local_rank)
    flush = L2Flush(dev, local_rank)

    def barrier():
        if dist is not None:
            import torch
            dist.barrier(device_ids=[local_rank])
            torch.cuda.synchronize(local_rank)

    wl = Workload(og, sh, dev, args.workload, world, rank)
    with ClockSampler(local_rank) as clocks:
        per_step_ns, launches, wall = timed_steps(dev, og, flush, wl, args.steps, args.warmup, barrier)
    kernel, variant = wl.gemm.last_kernel, wl.gemm.variant
    floor_us = event_floor_us(dev, og, flush)
    gemm_ns = sum(per_step_ns)

    # Decode also as a CUDA graph: the step (the product alone) captured once and replayed back to back. B (235 MB)
    # exceeds L2, so the replays read it from HBM without a flush between them.
    graph_replay = None
    if args.workload == "c5":
        replays = 200
        dev.capture_begin()
        genc = dev.begin_commands()
        wl.encode(genc)
        dev.submit(genc)
        graph = dev.capture_end()
        gstamps = og.GpuTimestampSet(dev, 2)
        for _ in range(5):
            graph.launch()
        dev.timestamp(gstamps, 0)
        for _ in range(replays):
            graph.launch()
        dev.timestamp(gstamps, 1)
        gts = gstamps.read(0)
        graph_replay = {"us_per_step": round((gts[1] - gts[0]) / replays / 1e3, 3), "replays": replays,
                        "l2": "not flushed between replays (B exceeds L2)"}
        graph.dispose()
        gstamps.dispose()

    # Communicator for N > 1 (NCCL over NVLink): the id made on rank 0 and handed out through the process group.
    comm = None
    if dist is not None:
        box = [og.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        comm = og.Communicator(dev, world, rank, box[0])

    # The gather of the sharded result onto rank 0 over NVLink, timed apart from `value` (every rank takes part).
    gather = None
    if comm is not None:
        full = dev.create_buffer(wl.out_dtype, wl.B * wl.M * wl.N) if rank == 0 else None
        esize = np.dtype(wl.out_dtype).itemsize
        if wl.by_batch:  # batch shards are contiguous: one row of each rank's whole shard
            widths, gb, gm = [s.width * wl.M * wl.N for s in wl.shards], 1, 1
        else:
            widths, gb, gm = [s.width for s in wl.shards], wl.B, wl.M
        gst = og.GpuTimestampSet(dev, 2 * 6)
        for i in range(-2, 6):
            if i >= 0:
                dev.timestamp(gst, 2 * i)
            comm.gather_columns(wl.bufs["c"].ptr, esize, gb, gm, widths, full.ptr if full is not None else 0, 0)
            if i >= 0:
                dev.timestamp(gst, 2 * i + 1)
        gts = gst.read(0)
        gst.dispose()
        g_ns = statistics.median(gts[2 * i + 1] - gts[2 * i] for i in range(6))
        if full is not None:
            full.dispose()
        received = (wl.B * wl.M * wl.N - wl.count) * esize
        gather = {"ns": g_ns, "bytes_into_root": int(received)}

    # e2e through the C ABI from page-locked host memory, pipelined over two sets of device buffers: every step
    # uploads its inputs on the copy engine (at N > 1 each rank only its 1/N of the replicated operand, which the
    # ranks then all-gather over NVLink), runs the product, and reads its shard of the result back, while the next
    # step's upload and the previous step's readback overlap it. Timed by the host clock from the first upload to
    # the last readback; the max over ranks.
    first_host, b_host = wl.first_host, wl.b_host
    # A replicated (column shards) or B replicated (batch shards): each rank uploads its rows of it.
    split_a = comm is not None and not wl.by_batch and first_host.nbytes % world == 0
    split_b = comm is not None and wl.by_batch and b_host.nbytes % world == 0
    up_first = first_host.nbytes // world if split_a else first_host.nbytes
    up_b = b_host.nbytes // world if split_b else b_host.nbytes
    h2d = up_first + up_b
    d2h = wl.count * np.dtype(wl.out_dtype).itemsize
    pin_in = og.PinnedHost(up_first + up_b)
    pin_out = og.PinnedHost(2 * d2h)
    fv = first_host.view(np.uint8)
    bv = b_host.view(np.uint8)
    pin_in.view(np.uint8, up_first)[:] = fv[rank * up_first:(rank + 1) * up_first] if split_a else fv
    pin_in.view(np.uint8, up_b, up_first)[:] = bv[rank * up_b:(rank + 1) * up_b] if split_b else bv
    first_key = "x" if wl.w.get("dql_in_step") else "a"
    first_dtype = np.float32 if first_key == "x" else wl.a_dtype
    spare = dict(a=dev.create_buffer(wl.a_dtype, wl.bufs["a"].length), b=dev.create_buffer(np.int8, b_host.size),
                 c=dev.create_buffer(wl.out_dtype, wl.count))
    if first_key == "x":
        spare["x"] = dev.create_buffer(np.float32, wl.bufs["x"].length)
    part_first = [dev.create_buffer(np.uint8, up_first) for _ in range(2)] if split_a else None
    part_b = [dev.create_buffer(np.uint8, up_b) for _ in range(2)] if split_b else None
    sets = [dict(wl.bufs), spare]

    def e2e_step(i, tickets):
        bs = sets[i % 2]
        if len(tickets) >= 2:
            tickets[-2].wait()  # the step that last used this buffer set has been read back, so it has finished
        dst_first = bs[first_key]
        if split_a:
            dev.write_async(part_first[i % 2].ptr, pin_in.ptr, up_first)
            comm.all_gather(part_first[i % 2].ptr, up_first, dst_first.ptr)
        else:
            dev.write_async(dst_first.ptr, pin_in.ptr, up_first)
        if split_b:
            dev.write_async(part_b[i % 2].ptr, pin_in.ptr + up_first, up_b)
            comm.all_gather(part_b[i % 2].ptr, up_b, bs["b"].ptr)
        else:
            dev.write_async(bs["b"].ptr, pin_in.ptr + up_first, up_b)
        enc = dev.begin_commands()
        wl.encode(enc, **{k: v for k, v in bs.items() if k in ("a", "b", "c", "x")})
        dev.submit(enc)
        tickets.append(dev.read_async(pin_out.ptr + (i % 2) * d2h, bs["c"].ptr, d2h))

    tickets = []
    for i in range(2):  # warm-up: each buffer set once
        e2e_step(i, tickets)
    for t in tickets[-2:]:
        t.wait()
    barrier()
    tickets = []
    e2e_steps = min(args.steps, 20)
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        e2e_step(i, tickets)
    for t in tickets[-2:]:
        t.wait()
    e2e_ns = (time.perf_counter() - t0) * 1e9 / e2e_steps * args.steps
    barrier()
    pin_in.dispose()
    pin_out.dispose()
    for v in list(spare.values()) + (part_first or []) + (part_b or []):
        v.dispose()

    # cuBLAS (torch._int_mm) on the same shard for context: library int8 throughput on this GPU.
    lib_tops = None
    if args.workload == "c3" and not args.no_library:
        try:
            import torch
            ta = torch.from_numpy(wl.a_host.reshape(wl.M, wl.K)).cuda(local_rank)
            tb = torch.from_numpy(wl.b_host.reshape(wl.K, wl.shard_n)).cuda(local_rank)
            for _ in range(3):
                torch._int_mm(ta, tb)
            torch.cuda.synchronize(local_rank)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(5):
                torch._int_mm(ta, tb)
            e1.record()
            torch.cuda.synchronize(local_rank)
            lib_tops = 2.0 * wl.M * wl.shard_n * wl.K * 5 / (e0.elapsed_time(e1) * 1e-3) / 1e12
            del ta, tb
        except Exception as exc:  # noqa: BLE001 - context only
            lib_tops = f"unavailable: {type(exc).__name__}"

    # The other multi-GPU configs at this N, measured in the same run (a few steps each): config 5 (decode,
    # N-sharded, HBM-bound) and config 4 (batched QKV, batch-sharded).
    subs = {}
    if args.workload == "c3" and not args.no_extra:
        for name in ("c5", "c4"):
            sub = Workload(og, sh, dev, name, world, rank, seed=4321)
            ns, sub_launches, _ = timed_steps(dev, og, flush, sub, min(args.steps, 20), 3, barrier)
            subs[name] = dict(ns=statistics.mean(ns), total=sum(ns), steps=len(ns), kernel=sub.gemm.last_kernel,
                              ops_total=sub.ops_total, ops_shard=sub.ops_shard, algo_bytes=sub.algo_bytes,
                              launches=sub_launches, desc=sub.w["desc"],
                              parallelism=("batch" if sub.by_batch else "N") + f"-shard x{world}")
            sub.dispose()

    wl.dispose()
    # Max over ranks of every time (the slowest rank sets the step).
    keys = ["gemm", "e2e"] + (["gather"] if gather else []) + [f"{k}_total" for k in subs] + [f"{k}_ns" for k in subs]
    vals = [gemm_ns, e2e_ns] + ([gather["ns"]] if gather else []) + [subs[k]["total"] for k in subs] + \
           [subs[k]["ns"] for k in subs]
    if dist is not None:
        vals = sh.max_over_ranks(dist, vals, device=f"cuda:{local_rank}")
    mx = dict(zip(keys, vals))
    gemm_ns, e2e_ns = mx["gemm"], mx["e2e"]

    ms_per_step = gemm_ns / args.steps / 1e6
    value = wl.ops_total / (ms_per_step * 1e-3) / 1e12
    per_launch_s = statistics.mean(per_step_ns) * 1e-9
    achieved = wl.ops_shard / per_launch_s / 1e12
    if rank == 0:
        clk = clocks.summary()
        peaks, peak, peak_kind, burst, sust, capped = roofline_peaks(clk, gemm_ns * 1e-9 > 1.0 or wall > 1.0)
        cpu = None
        if world == 1 and not args.no_cpu:
            with host.everywhere():  # the CPU baselines use every host thread
                threads = os.cpu_count() or 1
                tops, dt, rows = cpu_gemm_tops(wl.shard_n, wl.K, threads, args.cpu_seconds, wl.M)
                sample = (f"{rows} of {wl.M} rows x {wl.shard_n} x K {wl.K} on {threads} threads ({dt:.1f} s), "
                          f"extrapolated to TOPS")
                if wl.w.get("dql_in_step"):
                    # Config 2's step also quantizes the activations: the oracle's DynamicReference over the whole x
                    # (one thread), added to the product's extrapolated time.
                    sys.path.insert(0, os.path.join(ROOT, "oracle"))
                    import og_oracle as oracle

                    t0 = time.perf_counter()
                    oracle.dynamic_quantize(wl.x_host)
                    dq_s = time.perf_counter() - t0
                    gemm_s = 2.0 * wl.M * wl.shard_n * wl.K / (tops * 1e12)
                    tops = 2.0 * wl.M * wl.shard_n * wl.K / (gemm_s + dq_s) / 1e12
                    sample += (f"; plus DynamicQuantizeLinear of all {wl.x_host.size} elements on 1 thread "
                               f"({dq_s:.2f} s)")
                cpu = {"value": round(tops, 6), "unit": "TOPS", "cores": threads, "kind": "port", "sample": sample}
                # The second CPU baseline: the reference's portable GPU kernel's blocking restated for the host's
                # cores.
                t_tops, t_dt, t_rows = cpu_gemm_tops(wl.shard_n, wl.K, threads, min(args.cpu_seconds, 6.0), wl.M,
                                                     tiled=True)
                cpu["tiled"] = {"value": round(t_tops, 6), "unit": "TOPS", "cores": threads, "kind": "port",
                                "sample": f"{t_rows} of {wl.M} rows x {wl.shard_n} x K {wl.K} on {threads} threads "
                                          f"({t_dt:.1f} s), extrapolated; og_oracle_int8_gemm_tiled restates "
                                          f"Int8GemmKernel.hlsl's 64 x 64 tiles, K chunks of 16, float sums folded "
                                          f"into int32 every 128 k"}
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "TOPS", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": f"{args.workload}: {wl.w['desc']}", "m": wl.M, "n": wl.N, "k": wl.K,
                       "batch": wl.B,
                       "parallelism": (f"{'batch' if wl.by_batch else 'N'}-shard x{world}" if world > 1
                                       else "single GPU"),
                       "l2": L2Flush.DESCRIPTION,
                       "kernel": kernel, "variant": variant},
            "roofline": {"bound": "tensor", "achieved": round(achieved, 3), "peak": round(peak, 1), "unit": "TOPS",
                         "frac": round(achieved / peak, 4), "traffic": profile_traffic(args.workload),
                         "peak_source": f"2 x {peaks['source']} dense bf16 {peak_kind} ({peak / 2.0} TF/s): the int8 "
                                        f"dense rate is twice bf16 on B200"
                                        + ("; sw_power_cap seen during the timed steps" if capped else ""),
                         "peak_burst": round(burst, 1), "frac_of_burst": round(achieved / burst, 4),
                         "peak_sustained": round(sust, 1), "frac_of_sustained": round(achieved / sust, 4)},
            "hbm": {"algorithmic_bytes_per_launch": int(wl.algo_bytes),
                    "achieved_gbs": round(wl.algo_bytes / per_launch_s / 1e9, 1), "peak_gbs": peaks["hbm_gbs"],
                    "frac": round(wl.algo_bytes / per_launch_s / 1e9 / peaks["hbm_gbs"], 4)},
            "cpu_baseline": cpu,
            "e2e": {"value": round(wl.ops_total / (e2e_ns / args.steps * 1e-9) / 1e12, 3), "unit": "TOPS",
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                    "replicated_operand": ("A uploaded 1/N per rank, all-gathered over NVLink" if split_a else
                                           "B uploaded 1/N per rank, all-gathered over NVLink" if split_b else None)},
            "gpu_launches": int(launches),
            "event_floor_us": floor_us,
            "host": host.summary(),
            "clocks": clk,
            "library_int8_tops": round(lib_tops, 3) if isinstance(lib_tops, float) else lib_tops,
            "graph_replay": graph_replay,
            "wall_s": round(wall, 3),
        }
        if gather:
            line["gather"] = {"us": round(mx["gather"] / 1e3, 2),
                              "gbs": round(gather["bytes_into_root"] / mx["gather"], 1),
                              "bytes_into_root": gather["bytes_into_root"], "root": 0,
                              "how": "NCCL send/recv over NVLink into staging, placed by one kernel "
                                     "(og_comm_gather_columns); not part of value"}
        for name, d in subs.items():
            ms = mx[f"{name}_total"] / d["steps"] / 1e6
            per_launch = mx[f"{name}_ns"] * 1e-9
            if name == "c5":
                total_bytes = d["algo_bytes"] * world  # every rank moves its own slab
                line["c5"] = {"workload": d["desc"], "parallelism": d["parallelism"], "kernel": d["kernel"],
                              "us_per_step": round(ms * 1e3, 2), "value": round(total_bytes / (ms * 1e-3) / 1e9, 1),
                              "unit": "GB/s", "per_gpu_gbs": round(d["algo_bytes"] / per_launch / 1e9, 1),
                              "frac": round(d["algo_bytes"] / per_launch / 1e9 / peaks["hbm_gbs"], 4),
                              "peak_gbs": peaks["hbm_gbs"], "algorithmic_bytes_per_gpu": int(d["algo_bytes"]),
                              "steps": d["steps"], "gpu_launches": d["launches"]}
            else:
                line["c4"] = {"workload": d["desc"], "parallelism": d["parallelism"], "kernel": d["kernel"],
                              "us_per_step": round(ms * 1e3, 2),
                              "value": round(d["ops_total"] / (ms * 1e-3) / 1e12, 1), "unit": "TOPS",
                              "per_gpu_tops": round(d["ops_shard"] / per_launch / 1e12, 1),
                              "frac": round(d["ops_shard"] / per_launch / 1e12 / peak, 4), "peak": round(peak, 1),
                              "steps": d["steps"], "gpu_launches": d["launches"]}
        print(json.dumps(line), flush=True)
    if comm is not None:
        comm.dispose()
    flush_dispose = getattr(flush, "dispose", None)
    if flush_dispose:
        flush_dispose()
    dev.dispose()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c3", choices=sorted(WORKLOADS) + sorted(FAMILIES))
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-library", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the c4 / c5 measurements of the default line")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.workload in FAMILIES:
        if args.impl == "reference":
            run_family_reference(args, rank, world)
        else:
            run_family(args, rank, world, local_rank)
        return
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    dist = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as tdist
        torch.cuda.set_device(local_rank)
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                 device_id=torch.device(f"cuda:{local_rank}"))
        dist = tdist
    try:
        run_ours(args, rank, world, local_rank, dist)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
