"""Benchmark of the int8 GEMM path (BASELINE.json metric: Int8Gemm TOPS at 8192^3 s8 x s8 -> s32).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c3|c2|c4|c5|conv|dequant|quant]
                    [--impl ours|reference]

One step is one Int8Gemm.EncodeInt32 + Submit of the workload (config 3 by default: A int8 [8192 x 8192] x B int8
[8192 x 8192], zero points absent, int32 C) with inputs resident in HBM; L2 is left cold and clean before every step
(a 512 MB write, then a 256 MB read of other data, stream-ordered) and the step itself is timed with CUDA events on
the device stream. With N > 1 (torchrun, one process per GPU,
NCCL only for the barrier and the max-over-ranks of the times) the product is sharded by onegpu_cuda.shard with no
collective in the data path ("strong" scaling: the total work is fixed): a batched workload by batch (rank g computes
its batches from its batches of A and the shared B), the others by 256-column slabs of B (rank g computes its columns
from the full A and its slab of B). `e2e` runs the same product through the C ABI from pinned host buffers (uploads of A and the B
slab, the product, readback of C), timed on the device. `--impl reference` times the CPU restatement of the
reference's int8 product (oracle/, all host threads) on a bounded row sample of the same workload.
"""
from __future__ import annotations

import argparse
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
    # name: (M, N, K, batch, a_signed, za, zb, out, description)
    "c3": dict(m=8192, n=8192, k=8192, batch=1, a_signed=True, zp=False, out="i32",
               desc="square s8 x s8 -> s32, 8192^3, zero points absent"),
    "c2": dict(m=4096, n=4096, k=4096, batch=1, a_signed=False, zp=True, out="f32", dql=True,
               desc="DynamicQuantizeLinear of f32 [4096 x 4096] ~ N(0,1) to u8, then u8 x s8 (per-column zp) -> f32 "
                    "dequantized by a_scale * b_scale[col], 4096^3; one step = both"),
    "c4": dict(m=2048, n=12288, k=4096, batch=8, a_signed=False, zp=True, out="i32",
               desc="batched QKV u8 (zp) x shared s8 (per-column zp) -> s32, 8 x 2048 x 12288 x 4096"),
    "c5": dict(m=16, n=28672, k=8192, batch=1, a_signed=False, zp=True, out="i32",
               desc="decode u8 (zp 128) x s8 (per-column zp) -> s32, 16 x 28672 x 8192"),
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


class ClockSampler:
    """SM clock, power and clock-event (throttle) reasons of one GPU, read through NVML every 20 ms while the timed
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
            time.sleep(0.02)

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


def cpu_gemm_tops(n: int, k: int, threads: int, target_s: float, max_rows: int, seed: int = 0):
    """Times the oracle's threaded restatement of the reference's int8 product (Int8Tests.Reference) on a sample of
    rows of A against the whole B, sized to about `target_s` seconds; returns (TOPS, seconds, rows)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import og_oracle as oracle

    b = oracle.bytes_(k * n, seed + 31)
    rows = 4
    while True:
        a = oracle.bytes_(rows * k, seed + 30)
        t0 = time.perf_counter()
        oracle.int8_gemm(a, True, b, True, m=rows, n=n, k=k, threads=threads)
        dt = time.perf_counter() - t0
        if dt >= 0.5 * target_s or rows >= max_rows:
            return 2.0 * rows * n * k / dt / 1e12, dt, rows
        rows = int(min(max_rows, max(rows * 2, rows * target_s / max(dt, 1e-3) * 0.9)))


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
            "gpu_launches": int(launches), "clocks": clocks.summary(), "wall_s": round(wall, 3)}
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
            "config": {"workload": f"{args.workload}: {w['desc']}", "parallelism": "host threads",
                       "sample": sample},
            "cpu_baseline": {"value": round(tops, 6), "unit": "TOPS", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(tops, 6), "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


REFERENCE_SECONDS = 120.0  # the reference arm's timed steps together, whatever --steps is


def run_ours(args, rank: int, world: int, local_rank: int, dist):
    import onegpu_cuda as og

    from onegpu_cuda import shard as sh

    w = WORKLOADS[args.workload]
    dev = og.GpuDevice(local_rank)
    M, N, K, B = w["m"], w["n"], w["k"], w["batch"]
    # Batched products are split by batch (B shared), the others by 256-column slabs of B.
    by_batch = B > 1
    extent, align = (B, 1) if by_batch else (N, sh.TILE_COLUMNS)
    if min(s.width for s in sh.split(extent, world, align)) == 0:  # decided alike on every rank
        raise SystemExit(f"{args.workload} has fewer shards than the {world} ranks")
    part = sh.shard_of(extent, world, rank, align)
    shard_n = N if by_batch else part.width
    B_local = part.width if by_batch else B
    rng = np.random.default_rng(1234)
    a_dtype = np.int8 if w["a_signed"] else np.uint8
    # Synthetic inputs with the config's distributions, generated on the host once (each rank draws the whole
    # operands from the same seed and keeps its shard).
    a_full = rng.integers(-128 if w["a_signed"] else 0, 128 if w["a_signed"] else 256, size=(B, M, K),
                          dtype=np.int16).astype(a_dtype)
    a_host = (sh.batch_slab(a_full, part) if by_batch else a_full).reshape(-1)
    del a_full
    b_full_cols = rng.integers(-128 if args.workload == "c3" else -127, 128, size=(K, N), dtype=np.int16)
    b_host = (b_full_cols if by_batch else sh.column_slab(b_full_cols, part)).astype(np.int8).reshape(-1)
    del b_full_cols
    a = dev.create_buffer(a_dtype, a_host)
    b = dev.create_buffer(np.int8, b_host)
    count = B_local * M * shard_n
    out_dtype = {"i32": np.int32, "f32": np.float32}[w["out"]]
    c = dev.create_buffer(out_dtype, count)
    zpa = zpb = scale = None
    extra = []
    if w["zp"]:
        za = dev.create_buffer(a_dtype, np.array([128 if not w["a_signed"] else 0], a_dtype))
        zb = dev.create_buffer(np.int8, rng.integers(-8, 9, size=shard_n).astype(np.int8))
        zpa, zpb = og.Int8Operand(za, 0), og.Int8Operand(zb, 0, True)
        extra += [za, zb]
    dq = x_dev = None
    if w.get("dql"):
        # Config 2: the activations arrive as float32 ~ N(0, 1); DynamicQuantizeLinear turns them into A (u8) with a
        # scale and zero point on the device, and the product dequantizes with a_scale * b_scale[col].
        x_host = rng.standard_normal(size=M * K, dtype=np.float32)
        x_dev = dev.create_buffer(np.float32, x_host)
        a_scale = dev.create_buffer(np.float32, 1)
        za = dev.create_buffer(np.uint8, 1)
        zb = dev.create_buffer(np.int8, rng.integers(-8, 9, size=shard_n).astype(np.int8))
        b_scale = dev.create_buffer(np.float32, rng.uniform(0.001, 0.02, size=shard_n).astype(np.float32))
        zpa, zpb = og.Int8Operand(za, 0), og.Int8Operand(zb, 0, True)
        dq = og.DynamicQuantizeKernels(dev)
        extra += [x_dev, a_scale, za, zb, b_scale]
        a_host = x_host  # what the e2e leg uploads
    elif w["out"] == "f32":
        s = dev.create_buffer(np.float32, rng.uniform(0.001, 0.02, size=shard_n).astype(np.float32) * 0.02)
        scale = og.Int8Operand(s, 0, True)
        extra.append(s)
    flush = L2Flush(dev, local_rank)
    prob = og.Int8GemmProblem(M, shard_n, K, batch=B_local, stride_a=M * K if B_local > 1 else 0, stride_b=0)
    gemm = og.Int8Gemm(dev)

    def encode(enc, a=a, b=b, c=c, x_dev=x_dev):
        if dq is not None:
            dq.encode(enc, x_dev, 0, M * K, a, 0, a_scale, 0, za, 0)
            gemm.encode_dequantize(enc, prob, a, b, c, og.Int8Operand(a_scale, 0), og.Int8Operand(b_scale, 0, True),
                                   zpa, zpb)
        elif w["out"] == "f32":
            gemm.encode_float(enc, prob, a, b, c, scale, zpa, zpb)
        else:
            gemm.encode_int32(enc, prob, a, b, c, zpa, zpb)

    stamps = og.GpuTimestampSet(dev, 2 * args.steps)

    def step(i=None):
        flush(i if i is not None else 0)
        enc = dev.begin_commands()
        if i is not None:
            enc.write_timestamp(stamps, 2 * i)
        encode(enc)
        if i is not None:
            enc.write_timestamp(stamps, 2 * i + 1)
        launches = enc.dispatch_count
        dev.submit(enc)
        return launches

    for _ in range(args.warmup):
        step()
    dev.wait_idle()
    kernel = gemm.last_kernel
    launches = 0

    def barrier():
        if dist is not None:
            import torch
            dist.barrier(device_ids=[local_rank])
            torch.cuda.synchronize(local_rank)

    barrier()
    with ClockSampler(local_rank) as clocks:
        t0 = time.perf_counter()
        for i in range(args.steps):
            launches += step(i)
        dev.wait_idle()
        wall = time.perf_counter() - t0
    barrier()
    ts = stamps.read(0)
    per_step_ns = [ts[2 * i + 1] - ts[2 * i] for i in range(args.steps)]
    gemm_ns = sum(per_step_ns)

    # Decode also as a CUDA graph: the step (the product alone) captured once and replayed back to back. B (235 MB)
    # exceeds L2, so the replays read it from HBM without a flush between them.
    graph_replay = None
    if args.workload == "c5":
        replays = 200
        dev.capture_begin()
        genc = dev.begin_commands()
        encode(genc)
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

    # e2e through the C ABI from page-locked host memory, pipelined over two sets of device buffers: every step
    # uploads its inputs (A and the B slab; x for c2) on the copy engine, runs the product, and reads its whole result
    # back, while the next step's upload and the previous step's readback overlap it. Timed by the host clock from the
    # first upload to the last readback.
    first_host = x_host if dq is not None else a_host
    h2d = first_host.nbytes + b_host.nbytes
    d2h = count * np.dtype(out_dtype).itemsize
    pin_in = og.PinnedHost(h2d)
    pin_out = og.PinnedHost(2 * d2h)
    pin_in.view(np.uint8, first_host.nbytes)[:] = first_host.view(np.uint8)
    pin_in.view(np.uint8, b_host.nbytes, first_host.nbytes)[:] = b_host.view(np.uint8)
    spare = dict(a=dev.create_buffer(a_dtype, B_local * M * K), b=dev.create_buffer(np.int8, b_host.size),
                 c=dev.create_buffer(out_dtype, count),
                 x_dev=dev.create_buffer(np.float32, M * K) if dq is not None else None)
    sets = [dict(a=a, b=b, c=c, x_dev=x_dev), spare]

    def e2e_step(i, tickets):
        bs = sets[i % 2]
        if len(tickets) >= 2:
            tickets[-2].wait()  # the step that last used this buffer set has been read back, so it has finished
        dst_first = bs["x_dev"] if dq is not None else bs["a"]
        dev.write_async(dst_first.ptr, pin_in.ptr, first_host.nbytes)
        dev.write_async(bs["b"].ptr, pin_in.ptr + first_host.nbytes, b_host.nbytes)
        enc = dev.begin_commands()
        encode(enc, **bs)
        dev.submit(enc)
        tickets.append(dev.read_async(pin_out.ptr + (i % 2) * d2h, bs["c"].ptr, d2h))

    tickets = []
    for i in range(2):  # warm-up: each buffer set once
        e2e_step(i, tickets)
    for t in tickets[-2:]:
        t.wait()
    tickets = []
    e2e_steps = min(args.steps, 20)
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        e2e_step(i, tickets)
    for t in tickets[-2:]:
        t.wait()
    e2e_ns = (time.perf_counter() - t0) * 1e9 / e2e_steps * args.steps
    pin_in.dispose()
    pin_out.dispose()
    for v in spare.values():
        if v is not None:
            v.dispose()

    # cuBLAS (torch._int_mm) on the same shard for context: library int8 throughput on this GPU.
    lib_tops = None
    if args.workload == "c3" and not args.no_library:
        try:
            import torch
            ta = torch.from_numpy(a_host.reshape(M, K)).cuda(local_rank)
            tb = torch.from_numpy(b_host.reshape(K, shard_n)).cuda(local_rank)
            for _ in range(3):
                torch._int_mm(ta, tb)
            torch.cuda.synchronize(local_rank)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(5):
                torch._int_mm(ta, tb)
            e1.record()
            torch.cuda.synchronize(local_rank)
            lib_tops = 2.0 * M * shard_n * K * 5 / (e0.elapsed_time(e1) * 1e-3) / 1e12
            del ta, tb
        except Exception as exc:  # noqa: BLE001 - context only
            lib_tops = f"unavailable: {type(exc).__name__}"

    if dist is not None:
        gemm_ns, e2e_ns = sh.max_over_ranks(dist, [gemm_ns, e2e_ns], device=f"cuda:{local_rank}")

    total_ops = 2.0 * B * M * N * K
    ms_per_step = gemm_ns / args.steps / 1e6
    value = total_ops / (ms_per_step * 1e-3) / 1e12
    per_launch_s = statistics.mean(per_step_ns) * 1e-9
    shard_ops = 2.0 * B_local * M * shard_n * K
    achieved = shard_ops / per_launch_s / 1e12
    # Bytes one launch must move at least: A, the B slab, C, and the zero-point / scale vectors.
    algo_bytes = (a_host.nbytes + b_host.nbytes + count * np.dtype(out_dtype).itemsize
                  + (shard_n + 1 if w["zp"] else 0) + (4 * shard_n if w["out"] == "f32" else 0)
                  + (2 * M * K if w.get("dql") else 0))  # the quantized A written by DQL and read by the product
    peaks = load_peaks()
    # A timed region of back-to-back launches longer than a second settles at the power-capped clock: compare with
    # the sustained figure then, with the burst figure for short runs.
    sustained = gemm_ns * 1e-9 > 1.0 or wall > 1.0
    peak_kind = "sustained" if sustained else "burst"
    peak = 2.0 * (peaks["bf16_tflops_sustained"] if sustained else peaks["bf16_tflops"])
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu:
            threads = os.cpu_count() or 1
            tops, dt, rows = cpu_gemm_tops(shard_n, K, threads, args.cpu_seconds, M)
            sample = f"{rows} of {M} rows x {shard_n} x K {K} on {threads} threads ({dt:.1f} s), extrapolated to TOPS"
            if dq is not None:
                # Config 2's step also quantizes the activations: the oracle's DynamicReference over the whole x
                # (one thread), added to the product's extrapolated time.
                sys.path.insert(0, os.path.join(ROOT, "oracle"))
                import og_oracle as oracle

                t0 = time.perf_counter()
                oracle.dynamic_quantize(x_host)
                dq_s = time.perf_counter() - t0
                gemm_s = 2.0 * M * shard_n * K / (tops * 1e12)
                tops = 2.0 * M * shard_n * K / (gemm_s + dq_s) / 1e12
                sample += f"; plus DynamicQuantizeLinear of all {x_host.size} elements on 1 thread ({dq_s:.2f} s)"
            cpu = {"value": round(tops, 6), "unit": "TOPS", "cores": threads, "kind": "port", "sample": sample}
        clk = clocks.summary()
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "TOPS", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": f"{args.workload}: {w['desc']}", "m": M, "n": N, "k": K, "batch": B,
                       "parallelism": (f"{'batch' if by_batch else 'N'}-shard x{world}" if world > 1
                                       else "single GPU"),
                       "l2": L2Flush.DESCRIPTION,
                       "kernel": kernel, "variant": gemm.variant},
            "roofline": {"bound": "tensor", "achieved": round(achieved, 3), "peak": round(peak, 1), "unit": "TOPS",
                         "frac": round(achieved / peak, 4), "traffic": profile_traffic(args.workload),
                         "peak_source": f"2 x {peaks['source']} dense bf16 {peak_kind} "
                                        f"({peak / 2.0} TF/s): the int8 dense rate is twice bf16 on B200"},
            "hbm": {"algorithmic_bytes_per_launch": int(algo_bytes),
                    "achieved_gbs": round(algo_bytes / per_launch_s / 1e9, 1), "peak_gbs": peaks["hbm_gbs"],
                    "frac": round(algo_bytes / per_launch_s / 1e9 / peaks["hbm_gbs"], 4)},
            "cpu_baseline": cpu,
            "e2e": {"value": round(total_ops / (e2e_ns / args.steps * 1e-9) / 1e12, 3), "unit": "TOPS",
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h)},
            "gpu_launches": int(launches),
            "clocks": clk,
            "library_int8_tops": round(lib_tops, 3) if isinstance(lib_tops, float) else lib_tops,
            "graph_replay": graph_replay,
            "wall_s": round(wall, 3),
        }
        print(json.dumps(line), flush=True)
    for v in [a, b, c] + extra:
        v.dispose()
    if dq is not None:
        dq.dispose()
    gemm.dispose()
    stamps.dispose()
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
