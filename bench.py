#!/usr/bin/env python
"""Benchmark of the FP8/FP4 hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload NAME] [--weak] [--size S] [--shape I] ...

Default run (no --workload): four JSON lines, one per workload, in this order
  1. fp8_roundtrip  4096x4096 float32 -> e4m3fn -> float32 (planted edges)
  2. fp8_roundtrip  the same input as bfloat16 -> e4m3fn -> bfloat16
  3. scaled_mm      torch._scaled_mm e4m3 x e4m3, per-tensor scales, bf16
                    out, M = N = K = 8192
  4. fp4_decode     16384x8192 float4_e2m1fn_x2 -> 16384x16384 bf16 x 0.37
The last line (FP4 decode) is the headline. `--impl reference` prints the
matching lines of the CPU implementation in the same order, with the same
config dicts.

Other workloads (`--workload`, one line each): fp8_roundtrip (--src, --fmt,
--elems), scaled_mm (--size), scaled_mm_rowwise (--shape 0|1|2 of
(16384,4096,4096), (16384,14336,4096), (16384,4096,14336)), fp4_scaled_mm
(packed FP4 x FP4, --size), scaled_mm_small_m (--m, --shape), linear_fp8w
(--m, --shape), llama_fp8 (--layers), fp8_quantize, fp8_quantize_noalloc,
quantize_rows, fp4_quantize.

Timing: W untimed warm-up steps, then a timed region of exactly K steps
(device time, CUDA events on the launching stream, barrier + synchronize on
both sides, max over ranks). The region is repeated until the repeats span
at least 200 ms (at least 3 repeats) so the clock sampler sees the load;
ms_per_step is the median region time / K, with the spread alongside.
Launch-bound workloads (round trip, quantisers, Llama stack) replay their K
steps from one CUDA graph. Working sets rotate through buffer sets until one
step's bytes times the sets exceed 400 MB, so no step is served from L2.

Multi-GPU (torchrun, one process per GPU): the workload's rows are split
across the ranks (converters: contiguous row blocks; GEMMs: rows of A with B
replicated; the Llama stack: sequences) with no collective on the data path:
strong scaling, `value` = the whole workload's bytes or flops / the max over
ranks of the step time. `--weak` runs a full-size replica per rank instead.
Workloads that do not split by rows (per-tensor quantisation, decode-sized
GEMMs and linears) always run as replicas.

`value` is device-resident throughput of the whole job; `e2e` is the same
metric through the package's public API with pinned host buffers (host to
device copy of the step's inputs, kernels, device to host copy of the result
inside the timed region, pipelined over chunks on three streams for the
converters).

`--impl reference` times the CPU implementation of the path on the host cores
with all threads, on rank 0 only: the reference's own kernels are Metal
compute for Apple GPUs and cannot run here, so the CPU oracle (a C
restatement of the same conversions) stands in for the converters and a
float32 dequantise-and-matmul stands in for the GEMM.
"""
from __future__ import annotations

import argparse
import copy
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.join(ROOT, "mps-fp8-for-torch-and-comfyui-python-package_b200")
for _p in (ROOT, PKG_ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

from fp4_fp8_for_torch_mps.parallel import shard_rows  # noqa: E402

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
ROTATE_BYTES = 400_000_000   # bytes touched between two uses of one buffer set (> 126 MB L2)
MIN_REGION_MS = 200.0        # timed regions repeat until they span this much device time
MIN_REPEATS, MAX_REPEATS = 3, 2000

DEFAULT_SUITE = [
    ("fp8_roundtrip", {"src": "f32", "fmt": "e4m3"}),
    ("fp8_roundtrip", {"src": "bf16", "fmt": "e4m3"}),
    ("scaled_mm", {"size": 8192}),
    ("fp4_decode", {}),
]


# ---------------------------------------------------------------- environment
def rank_info():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0")),
            int(os.environ.get("WORLD_SIZE", "1")))


class Ctx:
    """Rank, world size and split mode of one bench process."""

    def __init__(self, rank=0, local=0, ws=1, weak=False):
        self.rank, self.local, self.ws, self.weak = rank, local, ws, weak
        self.dist_on = ws > 1

    @property
    def sharded(self) -> bool:
        return self.ws > 1 and not self.weak

    def rows(self, total: int, splits: bool = True) -> tuple[int, int]:
        """This rank's [start, stop) block of `total` rows (everything when the
        workload runs as replicas)."""
        if splits and self.sharded:
            return shard_rows(total, self.ws, self.rank)
        return 0, total

    def parallelism(self, splits: bool = True) -> str:
        if self.ws == 1:
            return "single"
        return f"rows/{self.ws}" if (splits and not self.weak) else f"replicas{self.ws}"

    def scaling(self, splits: bool = True) -> str:
        return "strong" if (splits and self.sharded) else "weak"

    def seed(self) -> int:
        """Input seed: one global input split by rows, or a different input per replica."""
        return self.rank if (self.weak and self.ws > 1) else 0


_CPU_INPUTS: dict = {}


def cpu_input(key, make):
    """Host inputs of the CPU baseline, built once per process (the reference
    arm times `steps` samples of the same input)."""
    if key not in _CPU_INPUTS:
        _CPU_INPUTS[key] = make()
    return _CPU_INPUTS[key]


def rotating_sets(step_bytes: float, cap: int = 64) -> int:
    return 1 if step_bytes >= ROTATE_BYTES else min(cap, -(-int(ROTATE_BYTES) // max(1, int(step_bytes))))


def l2_note(sets: int, step_bytes: float) -> str:
    if sets > 1:
        return f"{sets} rotating buffer sets ({sets * step_bytes / 2**20:.0f} MiB) > L2"
    return f"{step_bytes / 2**20:.0f} MiB per step > L2, no flush"


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def profile_traffic(name: str):
    """DRAM bytes per launch from an ncu capture summarised in
    profiles/<name>.md (a line `dram_bytes_per_launch: <int>`), or None."""
    if not name:
        return None
    p = os.path.join(ROOT, "profiles", name + ".md")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        for line in f:
            if line.strip().startswith("dram_bytes_per_launch:"):
                try:
                    return int(float(line.split(":", 1)[1].strip().split()[0]))
                except ValueError:
                    return None
    return None


class ClockSampler:
    """SM clock and clock-event (throttle) reasons during the timed region:
    NVML polled every 2 ms from a background thread (the device is matched by
    PCI bus id), falling back to `nvidia-smi -lms 100`."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, cuda_index: int):
        self.cuda_index = cuda_index
        self.samples, self.reason_bits, self.max_mhz = [], 0, None
        self.thread, self.stop_flag, self.proc, self.err = None, False, None, None

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        p = torch.cuda.get_device_properties(self.cuda_index)
        bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)

    def start(self):
        import threading
        try:
            nv, h = self._nvml_handle()
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)

            def loop():
                while not self.stop_flag:
                    try:
                        self.samples.append(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                        self.reason_bits |= nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                    except Exception:  # noqa: BLE001 - keep sampling
                        pass
                    time.sleep(0.002)

            self.thread = threading.Thread(target=loop, daemon=True)
            self.thread.start()
        except Exception as e:  # noqa: BLE001 - fall back to nvidia-smi
            self.err = f"nvml: {e}"
            try:
                fd, self.path = tempfile.mkstemp(suffix=".csv")
                os.close(fd)
                self.proc = subprocess.Popen(
                    ["nvidia-smi", f"--id={self.cuda_index}",
                     "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.sw_power_cap,"
                     "clocks_event_reasons.hw_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                     "clocks_event_reasons.hw_thermal_slowdown", "--format=csv,noheader,nounits", "-lms", "100"],
                    stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
                time.sleep(0.3)
            except OSError as e2:
                self.err += f"; nvidia-smi: {e2}"

    def stop(self):
        if self.thread is not None:
            self.stop_flag = True
            self.thread.join(timeout=2)
            if not self.samples:
                return {"error": "no NVML samples"}
            reasons = sorted(v for k, v in self.REASONS.items() if self.reason_bits & k)
            return {"sm_mhz": statistics.median(self.samples), "sm_min_mhz": min(self.samples),
                    "sm_max_mhz": self.max_mhz, "reasons": reasons, "samples": len(self.samples),
                    "source": "nvml"}
        if self.proc is None:
            return {"error": self.err or "no sampler"}
        self.proc.terminate()
        self.proc.wait(timeout=5)
        rows = [[x.strip() for x in line.split(",")] for line in open(self.path) if line.count(",") >= 5]
        os.unlink(self.path)
        if not rows:
            return {"error": "no nvidia-smi samples"}
        names = ["sw_power_cap", "hw_slowdown", "sw_thermal_slowdown", "hw_thermal_slowdown"]
        sm = [float(r[0]) for r in rows if r[0].replace(".", "").isdigit()]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": float(rows[0][1]),
                "reasons": sorted({names[i] for r in rows for i in range(4) if r[2 + i].lower() == "active"}),
                "samples": len(rows), "source": "nvidia-smi"}


def timed_region(region, stream, dist_on: bool) -> float:
    """One call of `region` between barrier + synchronize; device ms, max over ranks."""
    import torch.distributed as dist
    if dist_on:
        dist.barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    region()
    end.record(stream)
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    if dist_on:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    return ms


def repeated_regions(region, stream, dist_on: bool) -> list[float]:
    """Repeat the K-step region until the repeats span MIN_REGION_MS of device
    time (and at least MIN_REPEATS). Every rank sees the same max-reduced
    times, so every rank stops after the same repeat."""
    out = []
    while True:
        out.append(timed_region(region, stream, dist_on))
        if len(out) >= MAX_REPEATS or (len(out) >= MIN_REPEATS and sum(out) >= MIN_REGION_MS):
            return out


def all_true(ok: bool, ctx: Ctx) -> bool:
    if not ctx.dist_on:
        return bool(ok)
    import torch.distributed as dist
    t = torch.tensor([1 if ok else 0], dtype=torch.int32, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return bool(t.item())


def gather_line(w, ctx: Ctx, reps=10):
    """Replicated-output mode of the row-sharded GEMM, timed on its own: each
    rank contributes its block of output rows and parallel.gather_rows (one
    NCCL all_gather_into_tensor over NVLink/NVSwitch) assembles the full
    M x N result on every rank."""
    from fp4_fp8_for_torch_mps.parallel import gather_rows
    M = w.M_total
    local = w.out
    for _ in range(3):
        full = gather_rows(local, M)
    torch.cuda.synchronize()

    def region():
        for _ in range(reps):
            gather_rows(local, M)
    ms = timed_region(region, torch.cuda.current_stream(), True) / reps
    nbytes = full.numel() * full.element_size()
    return {"ms": round(ms, 4), "bytes_per_rank": local.numel() * local.element_size(), "bytes_total": nbytes,
            "algbw_GBps": round(nbytes / (ms * 1e-3) / 1e9, 1),
            "busbw_GBps": round(nbytes * (ctx.ws - 1) / ctx.ws / (ms * 1e-3) / 1e9, 1),
            "op": "parallel.gather_rows -> NCCL all_gather_into_tensor", "timed": "separately, not in value"}


def chunk_bounds(n: int, chunks: int) -> list[tuple[int, int]]:
    chunks = max(1, min(chunks, n))
    step = -(-n // chunks)
    return [(i, min(n, i + step)) for i in range(0, n, step)]


def chunked_e2e(bounds, streams, body):
    """Run body(i, lo, hi, stream_index) for every chunk on rotating streams,
    joined to the current stream (so events on it bracket the whole pipeline)."""
    cur = torch.cuda.current_stream()
    ev = torch.cuda.Event()
    ev.record(cur)
    for s in streams:
        s.wait_event(ev)
    for i, (lo, hi) in enumerate(bounds):
        j = i % len(streams)
        with torch.cuda.stream(streams[j]):
            body(i, lo, hi, j)
    for s in streams:
        cur.wait_stream(s)


# ---------------------------------------------------------------- workloads
# Every workload class has
#   describe(args, ctx) -> dict(metric, unit, dtype, config, splits, bound)
#       the line's identity, shared by the GPU arm and the reference arm;
#   __init__(ctx, args), step(), e2e_step(), check(), and cpu_run(args) ->
#       (value, cores, sample description) for the host baseline.
class Fp4Decode:
    name = "fp4_decode"
    bound, kernels_per_step = "hbm", 1
    profile = "fp4_decode_16384x8192_bf16"

    @staticmethod
    def describe(args, ctx):
        from fp4_fp8_for_torch_mps.workloads import FP4_DECODE_SCALE, FP4_DECODE_SHAPE
        rows, cols = FP4_DECODE_SHAPE
        s, e = ctx.rows(rows)
        step = (e - s) * cols * 5
        sets = rotating_sets(step)
        return {"metric": "fp4_decode_GBps", "unit": "GB/s", "dtype": "u8->bf16", "splits": True, "bound": "hbm",
                "config": {"workload": "fp4_decode", "shape": [rows, cols], "out": f"bf16[{rows},{2 * cols}]",
                           "scale": FP4_DECODE_SCALE, "l2": l2_note(sets, step),
                           "launch": "K steps (one decode kernel each) replayed as one CUDA graph",
                           "parallelism": ctx.parallelism()}}

    def __init__(self, ctx, args):
        from fp4_fp8_for_torch_mps import _lib as L
        from fp4_fp8_for_torch_mps import fp8_mps_native as nat
        from fp4_fp8_for_torch_mps.workloads import FP4_DECODE_SCALE, fp4_decode_input
        self.L, self.nat, self.scale_v = L, nat, FP4_DECODE_SCALE
        full = fp4_decode_input(seed=ctx.seed())
        s, e = ctx.rows(full.shape[0])
        self.x_host = full[s:e].contiguous()
        del full
        rows, cols = self.x_host.shape
        self.rows, self.cols = rows, cols
        self.sets = rotating_sets(rows * cols * 5)
        self.xs = [self.x_host.cuda() for _ in range(self.sets)]
        self.outs = [torch.empty(rows, 2 * cols, dtype=torch.bfloat16, device="cuda") for _ in range(self.sets)]
        self.scale = torch.tensor([FP4_DECODE_SCALE], dtype=torch.float32, device="cuda")
        self.work = rows * cols * 5            # bytes read + written per step on this rank
        self.h2d, self.d2h = rows * cols, rows * cols * 4
        self.stream = torch.cuda.current_stream()
        self.lib = L.lib()
        self.i = 0
        # end-to-end buffers: pinned host in/out, row chunks on 3 streams
        self.h_in = self.x_host.pin_memory()
        self.h_out = torch.empty(rows, 2 * cols, dtype=torch.bfloat16).pin_memory()
        self.bounds = chunk_bounds(rows, 16)
        crow = self.bounds[0][1] - self.bounds[0][0]
        self.streams = [torch.cuda.Stream() for _ in range(3)]
        self.d_in = [torch.empty(crow, cols, dtype=torch.uint8, device="cuda") for _ in self.streams]
        self.d_out = [torch.empty(crow, 2 * cols, dtype=torch.bfloat16, device="cuda") for _ in self.streams]

    graph = None
    graph_launches = 0  # kernels in the captured graph

    def _launch(self, k, st):
        x, out = self.xs[k], self.outs[k]
        rc = self.lib.fp8b200_decode_fp4(x.data_ptr(), x.numel(), out.data_ptr(), self.L.BF16,
                                         self.scale.data_ptr(), self.L.SCALE_F32, st)
        if rc:
            self.L.check(rc, "fp4 decode")

    def capture(self, steps):
        """The K timed steps (one decode launch each, cycling through the
        buffer sets) as one CUDA graph, replayed once per timed region, so
        that consecutive launches overlap through programmatic dependent
        launch with no host launch gap (a row block on 8 GPUs is a ~13 us
        launch)."""
        side = torch.cuda.Stream()
        self.graph = torch.cuda.CUDAGraph()
        n0 = self.L.launch_count()
        with torch.cuda.stream(side):
            with torch.cuda.graph(self.graph, stream=side):
                for j in range(steps):
                    self._launch((self.i + j) % self.sets, side.cuda_stream)
        self.graph_launches = self.L.launch_count() - n0
        torch.cuda.synchronize()

    def replay(self):
        self.graph.replay()

    def step(self):
        k = self.i % self.sets
        self.i += 1
        self._launch(k, self.stream.cuda_stream)

    def e2e_step(self):
        def body(i, lo, hi, j):
            n = hi - lo
            self.d_in[j][:n].copy_(self.h_in[lo:hi], non_blocking=True)
            self.nat.fp4_decode(self.d_in[j][:n].view(torch.float4_e2m1fn_x2), torch.bfloat16,
                                scale=self.scale, out=self.d_out[j][:n])
            self.h_out[lo:hi].copy_(self.d_out[j][:n], non_blocking=True)
        chunked_e2e(self.bounds, self.streams, body)

    def check(self):
        import numpy as np
        from oracle import oracle as O
        sl = slice(max(0, self.rows - 64), self.rows)
        ref = O.fp4_decode(self.x_host[sl].numpy(), 1, self.scale_v)
        return bool(np.array_equal(ref, self.h_out[sl].view(torch.int16).numpy().view(np.uint16)))

    @staticmethod
    def cpu_run(args=None, reps=3, rows=16384):
        from oracle import oracle as O
        from fp4_fp8_for_torch_mps.workloads import FP4_DECODE_SCALE, fp4_decode_input
        x = cpu_input(("fp4_decode", rows), lambda: fp4_decode_input(seed=0, rows=rows).numpy())
        threads = os.cpu_count() or 1
        O.fp4_decode(x, 1, FP4_DECODE_SCALE, threads=threads)
        t0 = time.perf_counter()
        for _ in range(reps):
            O.fp4_decode(x, 1, FP4_DECODE_SCALE, threads=threads)
        dt = (time.perf_counter() - t0) / reps
        return x.size * 5 / dt / 1e9, threads, f"{rows}x{x.shape[1]} bytes -> bf16 x 0.37 per pass (oracle, C)", dt


class Fp8RoundTrip:
    """FP8 round trip: encode `--src` (f32, bf16 or f16) to `--fmt` (e4m3fn
    or e5m2), decode back to the source dtype. Default 4096x4096 f32 ->
    e4m3fn -> f32; `--elems` sets the element count (the 4096x4096 planted
    input is tiled; e.g. 1073741824 for a 1 Gi-element sweep). Rows of 4096
    elements split across ranks."""
    name = "fp8_roundtrip"
    bound, kernels_per_step = "hbm", 2
    SRC = {"f32": (torch.float32, 0, 4), "bf16": (torch.bfloat16, 1, 2), "f16": (torch.float16, 2, 2)}
    FMT = {"e4m3": ("e4m3fn", 0, torch.float8_e4m3fn), "e5m2": ("e5m2", 1, torch.float8_e5m2)}

    @staticmethod
    def _n(args):
        from fp4_fp8_for_torch_mps.workloads import FP8_ROUNDTRIP_SHAPE
        base = FP8_ROUNDTRIP_SHAPE[0] * FP8_ROUNDTRIP_SHAPE[1]
        return (getattr(args, "elems", 0) or base), base

    @staticmethod
    def describe(args, ctx):
        n, base = Fp8RoundTrip._n(args)
        src, fmt = args.src, args.fmt
        _, _, eb = Fp8RoundTrip.SRC[src]
        rows = -(-n // 4096)
        s, e = ctx.rows(rows)
        local = min(n, e * 4096) - s * 4096
        step = local * (2 * eb + 2)
        sets = rotating_sets(step)
        fmt_name = Fp8RoundTrip.FMT[fmt][0]
        return {"metric": "fp8_roundtrip_GBps", "unit": "GB/s", "dtype": f"{src}->{fmt_name}->{src}",
                "splits": True, "bound": "hbm",
                "config": {"workload": "fp8_roundtrip", "shape": [4096, 4096] if n == base else [n],
                           "src": src, "fp8": fmt_name, "l2": l2_note(sets, step),
                           "launch": "K steps (encode + decode kernels each) replayed as one CUDA graph",
                           "parallelism": ctx.parallelism()}}

    def __init__(self, ctx, args):
        from fp4_fp8_for_torch_mps import _lib as L
        from fp4_fp8_for_torch_mps import fp8_mps_native as nat
        from fp4_fp8_for_torch_mps.workloads import fp8_roundtrip_input
        self.L, self.nat = L, nat
        src, fmt = args.src, args.fmt
        self.src, self.fmt_key = src, fmt
        self.tdt, self.sdt, eb = self.SRC[src]
        self.fmt_name, self.fmt, self.fp8 = self.FMT[fmt]
        self.l_sdt = (L.F32, L.BF16, L.F16)[self.sdt]
        self.l_fmt = (L.E4M3, L.E5M2)[self.fmt]
        n, base_n = self._n(args)
        base = fp8_roundtrip_input(seed=ctx.seed())
        flat = base.view(-1)
        if n > flat.numel():
            flat = flat.repeat((n + flat.numel() - 1) // flat.numel())
        rows = -(-n // 4096)
        s, e = ctx.rows(rows)
        lo, hi = s * 4096, min(n, e * 4096)
        self.x_host = flat[lo:hi].to(self.tdt).contiguous()
        del base, flat
        nl = self.x_host.numel()
        self.profile = "fp8_encode_decode_4096x4096" if (src, fmt, n, ctx.sharded) == ("f32", "e4m3", base_n,
                                                                                       False) else None
        step_bytes = nl * (2 * eb + 2)
        self.SETS = rotating_sets(step_bytes)
        self.xs = [self.x_host.cuda() for _ in range(self.SETS)]
        self.codes = [torch.empty(nl, dtype=torch.uint8, device="cuda") for _ in range(self.SETS)]
        self.back = [torch.empty(nl, dtype=self.tdt, device="cuda") for _ in range(self.SETS)]
        self.i = 0
        self.work = step_bytes                   # encode (eb + 1) B/elt + decode (1 + eb) B/elt
        self.h2d, self.d2h = nl * eb, nl * eb
        self.stream = torch.cuda.current_stream()
        self.lib = L.lib()
        self.h_in = self.x_host.pin_memory()
        self.h_out = torch.empty_like(self.x_host).pin_memory()
        self.bounds = chunk_bounds(nl, 8)
        cn = self.bounds[0][1] - self.bounds[0][0]
        self.streams = [torch.cuda.Stream() for _ in range(3)]
        self.d_in = [torch.empty(cn, dtype=self.tdt, device="cuda") for _ in self.streams]
        self.d_mid = [torch.empty(cn, dtype=torch.uint8, device="cuda") for _ in self.streams]
        self.d_out = [torch.empty(cn, dtype=self.tdt, device="cuda") for _ in self.streams]

    graph = None
    graph_launches = 0  # kernels in the captured graph

    def _launch(self, k, s):
        n = self.codes[k].numel()
        rc = self.lib.fp8b200_encode_fp8(self.xs[k].data_ptr(), self.l_sdt, self.codes[k].data_ptr(),
                                         self.l_fmt, n, None, s)
        rc = rc or self.lib.fp8b200_decode_fp8(self.codes[k].data_ptr(), self.l_fmt, self.back[k].data_ptr(),
                                               self.l_sdt, n, None, 0, s)
        if rc:
            self.L.check(rc, "fp8 round trip")

    def capture(self, steps):
        """One CUDA graph holding `steps` consecutive steps (each an encode
        and a decode launch, cycling through the buffer sets), replayed once
        per timed region: the two 13-16 us kernels of a step are otherwise
        bound by host launch cost, and one graph per step still leaves a
        graph-launch gap between steps."""
        side = torch.cuda.Stream()
        self.graph = torch.cuda.CUDAGraph()
        n0 = self.L.launch_count()
        with torch.cuda.stream(side):
            with torch.cuda.graph(self.graph, stream=side):
                for j in range(steps):
                    self._launch((self.i + j) % self.SETS, side.cuda_stream)
        self.graph_launches = self.L.launch_count() - n0
        torch.cuda.synchronize()

    def replay(self):
        self.graph.replay()

    def step(self):
        k = self.i % self.SETS
        self.i += 1
        self._launch(k, self.stream.cuda_stream)

    def e2e_step(self):
        hin, hout = self.h_in.view(-1), self.h_out.view(-1)

        def body(i, lo, hi, j):
            n = hi - lo
            self.d_in[j][:n].copy_(hin[lo:hi], non_blocking=True)
            self.nat.encode_fp8(self.d_in[j][:n], self.fp8, out=self.d_mid[j][:n])
            self.nat.decode_fp8(self.d_mid[j][:n], self.fp8, self.tdt, out=self.d_out[j][:n])
            hout[lo:hi].copy_(self.d_out[j][:n], non_blocking=True)
        chunked_e2e(self.bounds, self.streams, body)

    def check(self):
        import numpy as np
        from oracle import oracle as O
        npu = np.uint32 if self.sdt == 0 else np.uint16
        ity = torch.int32 if self.sdt == 0 else torch.int16
        m = min(1 << 16, self.x_host.numel())
        xb = self.x_host.view(-1)[:m].view(ity).numpy().view(npu)
        ref = O.decode_fp8(O.encode_fp8(xb, self.sdt, self.fmt), self.fmt, self.sdt)
        got = self.h_out.view(-1)[:m].view(ity).numpy().view(npu)
        return bool(np.array_equal(ref, got))

    @staticmethod
    def cpu_run(args, reps=3, rows=4096):
        import numpy as np
        from oracle import oracle as O
        from fp4_fp8_for_torch_mps.workloads import fp8_roundtrip_input
        src, fmt = args.src, args.fmt
        tdt, sdt, eb = Fp8RoundTrip.SRC[src]
        f = Fp8RoundTrip.FMT[fmt][1]
        x = cpu_input(("fp8_roundtrip", rows, src), lambda: fp8_roundtrip_input(0).view(-1)[: rows * 4096].to(tdt))
        xb = x.view(torch.int32 if sdt == 0 else torch.int16).numpy().view(np.uint32 if sdt == 0 else np.uint16)
        threads = os.cpu_count() or 1
        t0 = time.perf_counter()
        for _ in range(reps):
            O.decode_fp8(O.encode_fp8(xb, sdt, f, threads=threads), f, sdt, threads=threads)
        dt = (time.perf_counter() - t0) / reps
        return xb.size * (2 * eb + 2) / dt / 1e9, threads, \
            f"{rows}x4096 {src} encode to {Fp8RoundTrip.FMT[fmt][0]} + decode per pass (oracle, C)", dt


class Quantize:
    """Dynamic quantisation rows of the path, each one bench line:
    fp8_quantize  -- per-tensor e4m3 (amax pass, scale, encode pass) of the
                     4096x4096 f32 FP8 round-trip input; bytes = in + out;
    fp8_quantize_noalloc -- the same through the allocation-free entry point
                     (scratch in the library's own device memory);
    quantize_rows -- per-token e4m3 of 16384x4096 bf16 activations (the
                     Llama-shaped stack's linear inputs); bytes = in + out +
                     scales; rows split across ranks;
    fp4_quantize  -- per-tensor FP4 (amax pass, scale, nibble encode) of
                     16384x16384 bf16 (the FP4 decode output's shape)."""
    bound = "hbm"
    profile = None
    SHAPES = {"fp8_quantize": (4096, 4096), "fp8_quantize_noalloc": (4096, 4096), "quantize_rows": (16384, 4096),
              "fp4_quantize": (16384, 16384)}
    DTYPES = {"fp8_quantize": "f32->e4m3 (per tensor)", "fp8_quantize_noalloc": "f32->e4m3 (per tensor)",
              "quantize_rows": "bf16->e4m3 (per row)", "fp4_quantize": "bf16->fp4 e2m1 (per tensor)"}

    @staticmethod
    def _bytes(kind, rows, cols):
        n = rows * cols
        eb = 4 if kind.startswith("fp8_quantize") else 2
        out_n = n // 2 if kind == "fp4_quantize" else n
        return n * eb + out_n + (4 * rows if kind == "quantize_rows" else 0), n * eb, out_n

    @staticmethod
    def describe_kind(kind, args, ctx):
        rows, cols = Quantize.SHAPES[kind]
        splits = kind == "quantize_rows"
        s, e = ctx.rows(rows, splits)
        work, _, _ = Quantize._bytes(kind, e - s, cols)
        sets = rotating_sets(work)
        return {"metric": f"{kind}_GBps", "unit": "GB/s", "dtype": Quantize.DTYPES[kind], "splits": splits,
                "bound": "hbm",
                "config": {"workload": kind, "shape": [rows, cols],
                           "src": "float32" if kind.startswith("fp8_quantize") else "bfloat16",
                           "l2": l2_note(sets, work), "launch": "K steps replayed as one CUDA graph",
                           "parallelism": ctx.parallelism(splits)}}

    def __init__(self, ctx, args, kind):
        from fp4_fp8_for_torch_mps import _lib as L
        from fp4_fp8_for_torch_mps.workloads import fp8_roundtrip_input
        self.L, self.kind = L, kind
        self.name = kind
        g = torch.Generator().manual_seed(ctx.seed())
        if kind.startswith("fp8_quantize"):
            x = fp8_roundtrip_input(seed=ctx.seed())
        elif kind == "quantize_rows":
            x = torch.randn(16384, 4096, generator=g).to(torch.bfloat16)
            s, e = ctx.rows(x.shape[0])
            x = x[s:e].contiguous()
        else:
            x = (torch.randn(16384, 16384, generator=g) * 3).to(torch.bfloat16)
        self.x_host = x
        rows, cols = x.shape
        self.work, in_b, out_n = self._bytes(kind, rows, cols)
        # a per-tensor scale needs the whole input's amax before the first code can be written, so the
        # input is read twice (amax pass, encode pass): the line also reports that two-read bound
        self.two_read_bytes = self.work + in_b if kind != "quantize_rows" else None
        n = x.numel()
        self.n = n
        self.sets = sets = rotating_sets(self.work)
        self.xs = [x.cuda() for _ in range(sets)]
        self.outs = [torch.empty(out_n, dtype=torch.uint8, device="cuda") for _ in range(sets)]
        self.scales = torch.empty(rows if kind == "quantize_rows" else 2, dtype=torch.float32, device="cuda")
        self.scratch = torch.zeros(1, dtype=torch.int32, device="cuda")
        self.h2d, self.d2h = in_b, out_n + 4 * (rows if kind == "quantize_rows" else 1)
        self.stream = torch.cuda.current_stream()
        self.lib = L.lib()
        self.i = 0
        n0 = L.launch_count()
        self.step()
        torch.cuda.synchronize()
        self.kernels_per_step = L.launch_count() - n0
        self.h_in = x.pin_memory()
        self.d_in = torch.empty_like(self.xs[0])
        self.h_out = torch.empty(out_n, dtype=torch.uint8).pin_memory()
        self.h_scales = torch.empty(self.scales.numel(), dtype=torch.float32).pin_memory()

    graph = None
    graph_launches = 0  # kernels in the captured graph

    def capture(self, steps):
        """One CUDA graph holding `steps` consecutive quantisations (cycling
        through the buffer sets), replayed once per timed region: a step is
        up to three kernels of a few to 25 us (clear, amax, encode for the
        per-tensor rows), which host launches one by one cannot keep fed; the
        host-launched path is what `e2e` measures."""
        side = torch.cuda.Stream()
        self.graph = torch.cuda.CUDAGraph()
        n0 = self.L.launch_count()
        with torch.cuda.stream(side):
            with torch.cuda.graph(self.graph, stream=side):
                for j in range(steps):
                    self._launch((self.i + j) % self.sets, side.cuda_stream)
        self.graph_launches = self.L.launch_count() - n0
        torch.cuda.synchronize()

    def replay(self):
        self.graph.replay()

    def step(self):
        k = self.i % self.sets
        self.i += 1
        self._launch(k, self.stream.cuda_stream)

    def _launch(self, k, st):
        L, x, o = self.L, self.xs[k], self.outs[k]
        if self.kind == "fp8_quantize":
            rc = self.lib.fp8b200_quantize_fp8(x.data_ptr(), L.F32, o.data_ptr(), L.E4M3, self.n,
                                               self.scales.data_ptr(), self.scratch.data_ptr(), st)
        elif self.kind == "fp8_quantize_noalloc":
            rc = self.lib.fp8b200_quantize_fp8_noalloc(x.data_ptr(), L.F32, o.data_ptr(), L.E4M3, self.n,
                                                       self.scales.data_ptr(), st)
        elif self.kind == "quantize_rows":
            r, c = x.shape
            rc = self.lib.fp8b200_quantize_rows_fp8(x.data_ptr(), L.BF16, r, c, c, o.data_ptr(), c, L.E4M3,
                                                    self.scales.data_ptr(), st)
        else:
            rc = self.lib.fp8b200_quantize_fp4(x.data_ptr(), L.BF16, o.data_ptr(), self.n,
                                               self.scales.data_ptr(), self.scratch.data_ptr(), st)
        if rc:
            L.check(rc, self.kind)

    def e2e_step(self):
        # public API on an input copied from pinned host memory, results read back
        self.d_in.copy_(self.h_in, non_blocking=True)
        if self.kind == "fp8_quantize":
            q, s = torch.ops.fp8_mps.quantize(self.d_in)
        elif self.kind == "fp8_quantize_noalloc":
            q = torch.empty(self.n, dtype=torch.uint8, device="cuda")
            s = torch.empty(2, dtype=torch.float32, device="cuda")
            self.L.check(self.lib.fp8b200_quantize_fp8_noalloc(self.d_in.data_ptr(), self.L.F32, q.data_ptr(),
                                                               self.L.E4M3, self.n, s.data_ptr(),
                                                               torch.cuda.current_stream().cuda_stream),
                         "quantize noalloc")
            s = s[1:]
        elif self.kind == "quantize_rows":
            from fp4_fp8_for_torch_mps import fp8_mps_native as nat
            q, s = nat.quantize_rows_fp8(self.d_in)
        else:
            q, s = torch.ops.fp8_mps.fp4_quantize(self.d_in)
        self.h_out.copy_(q.reshape(-1).view(torch.uint8), non_blocking=True)
        self.h_scales[:s.numel()].copy_(s.reshape(-1), non_blocking=True)

    def check(self):
        import numpy as np
        from oracle import oracle as O
        got = self.h_out.numpy()
        if self.kind == "quantize_rows":
            xf = self.x_host[:16].float().numpy()
            cols = xf.shape[1]
            for r in range(16):
                amax = np.float64(np.max(np.abs(xf[r])))
                sd = 448.0 / amax if amax > 0 else 1.0
                if self.h_scales[r].item() != np.float32(1.0 / sd):
                    return False
                if not np.array_equal(got[r * cols:(r + 1) * cols], O.encode_fp8_scaled(xf[r], np.float32(sd), 0)):
                    return False
            return True
        amax = float(self.x_host.float().abs().max())
        m = 1 << 16
        xf = self.x_host.reshape(-1)[:m].float().numpy()
        # the reference's rule: scale = fmax / amax if amax > 0 else 1 (a NaN amax gives 1)
        if self.kind.startswith("fp8_quantize"):
            scale = 448.0 / amax if amax > 0 else 1.0
            ok = np.array_equal(got[:m], O.encode_fp8_scaled(xf, scale, 0))
        else:
            scale = 6.0 / amax if amax > 0 else 1.0
            ok = np.array_equal(got[:m // 2], O.fp4_encode_ref(xf, scale))
        return bool(ok and self.h_scales[0].item() == np.float32(1.0 / scale))

    @staticmethod
    def cpu_run_kind(kind, reps=1):
        """The oracle (C, one thread) on a 1024-row sample: amax, scale, encode."""
        import numpy as np
        from oracle import oracle as O
        from fp4_fp8_for_torch_mps.workloads import fp8_roundtrip_input
        g = torch.Generator().manual_seed(0)
        if kind.startswith("fp8_quantize"):
            x = cpu_input(("fp8_quantize",), lambda: fp8_roundtrip_input(0)[:1024].numpy())
            eb, outb = 4, 1.0
        elif kind == "quantize_rows":
            x = cpu_input((kind,), lambda: torch.randn(1024, 4096, generator=g).to(torch.bfloat16).float().numpy())
            eb, outb = 2, 1.0
        else:
            x = cpu_input((kind,), lambda: (torch.randn(1024, 16384, generator=g) * 3).to(torch.bfloat16)
                          .float().numpy())
            eb, outb = 2, 0.5
        t0 = time.perf_counter()
        for _ in range(reps):
            if kind == "quantize_rows":
                for r in range(x.shape[0]):
                    a = float(np.max(np.abs(x[r])))
                    O.encode_fp8_scaled(x[r], np.float32(448.0 / a if a > 0 else 1.0), 0)
            elif kind.startswith("fp8_quantize"):
                O.encode_fp8_scaled(x, 448.0 / float(np.max(np.abs(x))), 0)
            else:
                O.fp4_encode_ref(x, 6.0 / float(np.max(np.abs(x))))
        dt = (time.perf_counter() - t0) / reps
        return x.size * (eb + outb) / dt / 1e9, 1, \
            f"{x.shape[0]}x{x.shape[1]} {kind} per pass (oracle, C, 1 thread)", dt


class GraphSteps:
    """Launch-bound workloads (decode-sized GEMMs and linears, a few to 40 us
    per call): the K timed steps are captured once as a CUDA graph (each step
    one C-ABI call, rotating through the weight sets) and replayed per timed
    region; `e2e` keeps the host-launched public API."""
    graph = None
    graph_launches = 0

    def capture(self, steps):
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        self.graph = torch.cuda.CUDAGraph()
        n0 = self.L.launch_count()
        saved = self.stream
        with torch.cuda.stream(side):
            self.stream = side
            with torch.cuda.graph(self.graph, stream=side):
                for _ in range(steps):
                    self.step()
        self.stream = saved
        self.graph_launches = self.L.launch_count() - n0
        torch.cuda.synchronize()

    def replay(self):
        self.graph.replay()


def _quantize_factory(kind):
    class _K(Quantize):
        name = kind

        @staticmethod
        def describe(args, ctx):
            return Quantize.describe_kind(kind, args, ctx)

        @staticmethod
        def cpu_run(args=None):
            return Quantize.cpu_run_kind(kind)

        def __init__(self, ctx, args):
            Quantize.__init__(self, ctx, args, kind)
    _K.__name__ = f"Quantize_{kind}"
    return _K


def gemm_check(w, rows):
    """Oracle check of `rows` output rows (all columns) of a GEMM line: the
    tolerance of the GEMM tests (one output ulp plus the float32 accumulation
    bound; FP4 x FP4 accumulates exactly, so one ulp alone), and the largest
    error in bf16 ulps of the float64 reference."""
    import numpy as np
    from oracle import oracle as O
    fa = O.FP4 if w.fp4 else O.E4M3
    ref, S = O.scaled_mm_ref(w.a_host.view(torch.uint8).numpy(), w.b_host.view(torch.uint8).numpy(),
                             w.sa_host.numpy().reshape(-1), w.sb_host.numpy().reshape(-1), fmt_a=fa, fmt_b=fa,
                             rows=rows)
    got = w.h_out[torch.from_numpy(rows)].float().double().numpy()
    u = O.bf16_ulp(ref)
    err = np.abs(got - ref)
    acc = (0.0 if w.fp4 else 2.0 ** -20) * S
    ok = bool(np.all(err <= u + acc))
    # outputs whose float32 accumulation bound is below half an output ulp (no cancellation)
    well = acc <= 0.5 * u
    return ok, {"rows_checked": int(len(rows)), "cols_checked": int(ref.shape[1]),
                "max_err_bf16_ulp": round(float((err / u).max()), 4),
                "max_err_bf16_ulp_well_conditioned": round(float((err / u)[well].max()), 4) if well.any() else None,
                "frac_well_conditioned": round(float(well.mean()), 6),
                "frac_over_1_ulp": float((err > u).mean()),
                "reference": "float64 dequantised product"}


class ScaledMM:
    """torch._scaled_mm e4m3 x e4m3 (per-tensor: M = N = K = --size; rowwise:
    the LLM shape --shape), or the packed FP4 x FP4 GEMM (fp4_scaled_mm,
    per-tensor, M = N = K = --size), bf16 out. Rows of A split across ranks,
    B replicated."""
    bound, kernels_per_step = "tensor", 1

    @staticmethod
    def _mnk(args, rowwise):
        from fp4_fp8_for_torch_mps.workloads import ROWWISE_SHAPES
        return ROWWISE_SHAPES[args.shape] if rowwise else (args.size,) * 3

    @staticmethod
    def describe_mode(args, ctx, rowwise, fp4):
        M, N, K = ScaledMM._mnk(args, rowwise)
        name = "fp4_scaled_mm" if fp4 else ("scaled_mm_rowwise" if rowwise else "scaled_mm")
        s, e = ctx.rows(M)
        kb = K // 2 if fp4 else K
        foot = (e - s) * kb + N * kb + 2 * (e - s) * N
        metric = {"scaled_mm": "scaled_mm_TFLOPS", "scaled_mm_rowwise": "scaled_mm_rowwise_TFLOPS",
                  "fp4_scaled_mm": "fp4_scaled_mm_TFLOPS"}[name]
        # packed FP4 x FP4 with K a multiple of 256 runs as tcgen05 kind::mxf4: four times the bf16 rate
        bound = "tensor_fp4" if (fp4 and K % 256 == 0) else "tensor"
        return {"metric": metric, "unit": "TFLOP/s", "splits": True, "bound": bound,
                "dtype": "e2m1xe2m1->bf16 (f32 acc)" if fp4 else "e4m3xe4m3->bf16 (f32 acc)",
                "config": {"workload": name, "M": M, "N": N, "K": K,
                           "scales": "rowwise" if rowwise else "tensorwise", "out": "bf16",
                           "operands": "packed float4_e2m1fn_x2, uniform bytes" if fp4 else "e4m3",
                           "l2": "A+B+D {:.0f} MiB".format(foot / 2**20) + (
                               " > L2, no flush" if foot > 126e6 else
                               " (one GEMM reads each operand tile from L2 repeatedly by design)"),
                           "parallelism": ctx.parallelism()}}

    def __init__(self, ctx, args, rowwise=False, fp4=False):
        from fp4_fp8_for_torch_mps import _lib as L
        from fp4_fp8_for_torch_mps.workloads import fp4_gemm_operands, rowwise_operands, scaled_mm_operands
        self.L, self.fp4, self.rowwise = L, fp4, rowwise
        M, N, K = self._mnk(args, rowwise)
        if fp4:
            aq, bq, sa, sb = fp4_gemm_operands(M, N, K, seed=ctx.seed())
        elif rowwise:
            aq, bq, sa, sb = rowwise_operands(M, N, K, seed=ctx.seed())
        else:
            aq, bq, sa, sb = scaled_mm_operands(M, N, K, seed=ctx.seed())
        self.name = "fp4_scaled_mm" if fp4 else ("scaled_mm_rowwise" if rowwise else "scaled_mm")
        s, e = ctx.rows(M)
        self.M_total = M
        aq = aq[s:e].contiguous()
        if sa.numel() > 1:
            sa = sa[s:e].contiguous()
        M = e - s
        self.M, self.N, self.K = M, N, K
        self.profile = f"{self.name}_{M}x{N}x{K}"
        self.a_host, self.b_host, self.sa_host, self.sb_host = aq, bq, sa, sb
        self.a, self.b = aq.cuda(), bq.cuda()
        self.sa, self.sb = sa.cuda(), sb.cuda()
        self.out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        self.work = 2.0 * M * N * K
        self.h2d = aq.numel() + bq.numel()
        self.d2h = M * N * 2
        self.stream = torch.cuda.current_stream()
        self.lib = L.lib()
        self.la = L.SCALE_ROWWISE if rowwise else L.SCALE_TENSOR
        self.code = L.E2M1 if fp4 else L.E4M3
        self.ld = K // 2 if fp4 else K
        self.h_a, self.h_b = aq.view(torch.uint8).pin_memory(), bq.view(torch.uint8).pin_memory()
        self.h_out = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()
        self.d_a = torch.empty_like(self.a.view(torch.uint8))
        self.d_b = torch.empty_like(self.b.view(torch.uint8))

    def step(self):
        L = self.L
        rc = self.lib.fp8b200_scaled_mm(self.a.data_ptr(), self.code, self.ld, self.b.data_ptr(), self.code, self.ld,
                                        self.M, self.N, self.K, self.sa.data_ptr(), self.la, self.sb.data_ptr(),
                                        self.la, None, 0, None, self.out.data_ptr(), L.BF16, self.N,
                                        self.stream.cuda_stream)
        if rc:
            L.check(rc, self.name)

    def e2e_step(self):
        # public API (torch._scaled_mm, or fp8_mps::fp4_scaled_mm for FP4) on
        # operands copied from pinned host memory, result read back
        self.d_a.copy_(self.h_a, non_blocking=True)
        self.d_b.copy_(self.h_b, non_blocking=True)
        if self.fp4:
            r = torch.ops.fp8_mps.fp4_scaled_mm(self.d_a, self.d_b, self.sa, self.sb, out_dtype=torch.bfloat16)
        else:
            r = torch._scaled_mm(self.d_a.view(torch.float8_e4m3fn), self.d_b.view(torch.float8_e4m3fn).t(),
                                 self.sa, self.sb, out_dtype=torch.bfloat16)
        self.h_out.copy_(r, non_blocking=True)

    def check(self):
        import numpy as np
        rows = np.sort(np.random.default_rng(1).choice(self.M, min(256, self.M), replace=False))
        ok, self.accuracy = gemm_check(self, rows)
        return ok

    @staticmethod
    def cpu_run_mode(args, rowwise, fp4, reps=1):
        """float32 dequantise-and-matmul on the host (the CPU path for this
        GEMM; CPU torch._scaled_mm is per-tensor only and ~0.1 GFLOP/s), on a
        256-row slice of A; FP4 operands are decoded to float first."""
        from fp4_fp8_for_torch_mps.workloads import fp4_gemm_operands, rowwise_operands, scaled_mm_operands
        M, N, K = ScaledMM._mnk(args, rowwise)
        rows = 256
        threads = torch.get_num_threads()
        def make():
            if fp4:
                from oracle import oracle as O
                a, b, sa, sb = fp4_gemm_operands(rows, N, K)
                return (torch.from_numpy(O.fp4_unpack_f64(a.numpy())).float() * sa,
                        torch.from_numpy(O.fp4_unpack_f64(b.numpy())).float() * sb)
            a, b, sa, sb = (rowwise_operands if rowwise else scaled_mm_operands)(rows, N, K)
            return (a.float() * (sa.reshape(-1, 1) if sa.numel() > 1 else sa),
                    b.float() * (sb.reshape(-1, 1) if sb.numel() > 1 else sb))
        A, B = cpu_input(("gemm", M, N, K, rowwise, fp4), make)
        t0 = time.perf_counter()
        for _ in range(reps):
            (A @ B.t()).to(torch.bfloat16)
        dt = (time.perf_counter() - t0) / reps
        return 2.0 * rows * N * K / dt / 1e12, threads, \
            f"{rows}x{N}x{K} f32 dequantised matmul (CPU torch, {threads} threads)", dt


def _gemm_factory(rowwise, fp4):
    class _G(ScaledMM):
        @staticmethod
        def describe(args, ctx):
            return ScaledMM.describe_mode(args, ctx, rowwise, fp4)

        @staticmethod
        def cpu_run(args):
            return ScaledMM.cpu_run_mode(args, rowwise, fp4)

        def __init__(self, ctx, args):
            ScaledMM.__init__(self, ctx, args, rowwise, fp4)
    return _G


class ScaledMMSmallM(GraphSteps):
    """Decode-sized rowwise GEMM: M (--m, default 16) activation rows against
    Llama-shaped e4m3 weights (N, K from --shape). The weights dominate the
    bytes, so the bound is HBM: work = N*K + M*K bytes read + 2*M*N written.
    Weight sets rotate (>= 300 MB in total) so that every step reads its
    weights from HBM, not L2. Replicas across ranks."""
    name = "scaled_mm_small_m"
    bound, kernels_per_step = "hbm", 1

    @staticmethod
    def describe(args, ctx):
        from fp4_fp8_for_torch_mps.workloads import ROWWISE_SHAPES
        _, N, K = ROWWISE_SHAPES[args.shape]
        M = args.m or 16
        nsets = max(2, min(32, -(-300_000_000 // (N * K))))
        return {"metric": "scaled_mm_small_m_GBps", "unit": "GB/s", "dtype": "e4m3xe4m3->bf16 (f32 acc)",
                "splits": False, "bound": "hbm",
                "config": {"workload": "scaled_mm_small_m", "M": M, "N": N, "K": K, "scales": "rowwise",
                           "out": "bf16", "l2": f"{nsets} rotating weight sets, {nsets * N * K / 2**20:.0f} MiB > L2",
                           "launch": "K steps replayed as one CUDA graph",
                           "parallelism": ctx.parallelism(False)}}

    def __init__(self, ctx, args):
        from fp4_fp8_for_torch_mps import _lib as L
        from fp4_fp8_for_torch_mps.workloads import ROWWISE_SHAPES, rowwise_operands
        self.L = L
        _, N, K = ROWWISE_SHAPES[args.shape]
        M = args.m or 16
        aq, bq, sa, sb = rowwise_operands(M, N, K, seed=ctx.rank)
        self.M, self.N, self.K = M, N, K
        self.profile = f"{self.name}_{M}x{N}x{K}"
        self.a_host, self.b_host, self.sa_host, self.sb_host = aq, bq, sa, sb
        self.nsets = max(2, min(32, -(-300_000_000 // (N * K))))
        self.a, self.sa, self.sb = aq.cuda(), sa.cuda(), sb.cuda()
        b = bq.cuda()
        self.bs = [b] + [b.clone() for _ in range(self.nsets - 1)]
        self.out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        self.work = float(N * K + M * K + 2 * M * N)
        self.h2d = M * K
        self.d2h = M * N * 2
        self.stream = torch.cuda.current_stream()
        self.lib = L.lib()
        self.i = 0
        self.h_a = aq.view(torch.uint8).pin_memory()
        self.h_out = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()
        self.d_a = torch.empty_like(self.a.view(torch.uint8))

    def step(self):
        L = self.L
        b = self.bs[self.i % self.nsets]
        self.i += 1
        rc = self.lib.fp8b200_scaled_mm(self.a.data_ptr(), L.E4M3, self.K, b.data_ptr(), L.E4M3, self.K,
                                        self.M, self.N, self.K, self.sa.data_ptr(), L.SCALE_ROWWISE,
                                        self.sb.data_ptr(), L.SCALE_ROWWISE, None, 0, None, self.out.data_ptr(),
                                        L.BF16, self.N, self.stream.cuda_stream)
        if rc:
            L.check(rc, "scaled_mm")

    def e2e_step(self):
        # public API: torch._scaled_mm on activations copied from pinned host
        # memory (the weights stay resident, as in decoding), result read back
        b = self.bs[self.i % self.nsets]
        self.i += 1
        self.d_a.copy_(self.h_a, non_blocking=True)
        r = torch._scaled_mm(self.d_a.view(torch.float8_e4m3fn), b.t(), self.sa, self.sb,
                             out_dtype=torch.bfloat16)
        self.h_out.copy_(r, non_blocking=True)

    def check(self):
        import numpy as np
        from oracle import oracle as O
        ref, S = O.scaled_mm_ref(self.a_host.view(torch.uint8).numpy(), self.b_host.view(torch.uint8).numpy(),
                                 self.sa_host.numpy().reshape(-1), self.sb_host.numpy().reshape(-1))
        got = self.h_out.float().double().numpy()
        return bool(np.all(np.abs(got - ref) <= O.bf16_ulp(ref) + 2.0 ** -20 * S))

    @staticmethod
    def cpu_run(args, reps=3):
        """float32 dequantise-and-matmul of the same M rows on the host."""
        from fp4_fp8_for_torch_mps.workloads import ROWWISE_SHAPES, rowwise_operands
        _, N, K = ROWWISE_SHAPES[args.shape]
        M = args.m or 16
        def make():
            a, b, sa, sb = rowwise_operands(M, N, K)
            return a.float() * sa.reshape(-1, 1), b.float() * sb.reshape(-1, 1)
        A, B = cpu_input(("small_m", M, N, K), make)
        threads = torch.get_num_threads()
        t0 = time.perf_counter()
        for _ in range(reps):
            (A @ B.t()).to(torch.bfloat16)
        dt = (time.perf_counter() - t0) / reps
        return float(N * K + M * K + 2 * M * N) / dt / 1e9, threads, \
            f"{M}x{N}x{K} f32 dequantised matmul (CPU torch, {threads} threads; weights pre-dequantised)", dt


class LinearFp8W(GraphSteps):
    """FP8-weight linear with dequant-on-load: y = x @ (w * s)^T, x bf16
    (M, K) N(0,1), w e4m3 quantised per output channel from N(0, 0.02),
    Llama shapes (N, K from --shape, M from --m, default 16384). Compute in
    bf16 on the tensor cores: the roofline peak is the measured bf16 rate;
    for M <= 256 the weight bytes bound it and the line reports GB/s (weights
    + x + y) against HBM. Replicas across ranks."""
    name = "linear_fp8w"
    kernels_per_step = 1

    @staticmethod
    def _dims(args):
        from fp4_fp8_for_torch_mps.workloads import ROWWISE_SHAPES
        _, N, K = ROWWISE_SHAPES[args.shape]
        M = args.m or 16384
        foot = M * K * 2 + N * K + M * N * 2
        nsets = 1 if foot > 300_000_000 else max(2, min(32, -(-300_000_000 // (N * K))))
        return M, N, K, foot, nsets

    @staticmethod
    def describe(args, ctx):
        M, N, K, foot, nsets = LinearFp8W._dims(args)
        small = M <= 256
        return {"metric": "linear_fp8w_GBps" if small else "linear_fp8w_TFLOPS",
                "unit": "GB/s" if small else "TFLOP/s", "splits": False, "bound": "hbm" if small else "tensor_bf16",
                "dtype": "bf16 x e4m3 (dequantised on load) -> bf16, f32 acc",
                "config": {"workload": "linear_fp8w", "M": M, "N": N, "K": K, "weights": "e4m3, per-channel scale",
                           "activations": "bf16", "out": "bf16",
                           "l2": ("x+w+y {:.0f} MiB > L2".format(foot / 2**20) if nsets == 1 else
                                  f"{nsets} rotating weight sets, {nsets * N * K / 2**20:.0f} MiB > L2"),
                           "launch": "K steps replayed as one CUDA graph" if small else "host-launched",
                           "parallelism": ctx.parallelism(False)}}

    def __init__(self, ctx, args):
        from fp4_fp8_for_torch_mps import _lib as L
        from fp4_fp8_for_torch_mps import fp8_mps_native as nat
        from fp4_fp8_for_torch_mps.workloads import rowwise_operands
        self.L, self.nat = L, nat
        M, N, K, foot, nsets = self._dims(args)
        g = torch.Generator().manual_seed(ctx.rank)
        self.x_host = torch.randn(M, K, generator=g).to(torch.bfloat16)
        _, wq, _, sw = rowwise_operands(1, N, K, seed=ctx.rank)
        self.w_host, self.s_host = wq, sw.reshape(-1)
        self.M, self.N, self.K = M, N, K
        self.profile = f"{self.name}_{M}x{N}x{K}"
        self.x, self.w, self.s = self.x_host.cuda(), wq.cuda(), self.s_host.cuda()
        self.nsets = nsets
        self.ws = [self.w] + [self.w.clone() for _ in range(self.nsets - 1)]
        self.i = 0
        self.out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        self.work = 2.0 * M * N * K
        if M <= 256:
            self.work = float(N * K + M * K * 2 + M * N * 2)
        self.h2d, self.d2h = M * K * 2, M * N * 2
        self.stream = torch.cuda.current_stream()
        self.lib = L.lib()
        self.h_x = self.x_host.pin_memory()
        self.h_out = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()
        self.d_x = torch.empty_like(self.x)

    def capture(self, steps):
        if self.M <= 256:
            GraphSteps.capture(self, steps)
        else:
            self.steps = steps

    def replay(self):
        if self.graph is not None:
            self.graph.replay()
        else:
            for _ in range(self.steps):
                self.step()

    def step(self):
        L = self.L
        w = self.ws[self.i % self.nsets]
        self.i += 1
        rc = self.lib.fp8b200_linear_fp8w(self.x.data_ptr(), L.BF16, self.K, w.data_ptr(), L.E4M3, self.K,
                                          self.M, self.N, self.K, self.s.data_ptr(), L.SCALE_ROWWISE, None, 0,
                                          self.out.data_ptr(), L.BF16, self.N, self.stream.cuda_stream)
        if rc:
            L.check(rc, "linear_fp8w")

    def e2e_step(self):
        self.d_x.copy_(self.h_x, non_blocking=True)
        w = self.ws[self.i % self.nsets]
        self.i += 1
        y = torch.ops.fp8_mps.fp8_linear(self.d_x, w, self.s)
        self.h_out.copy_(y, non_blocking=True)

    def check(self):
        import numpy as np
        from oracle import oracle as O
        rows = np.arange(0, self.M, max(1, self.M // 16))[:16]
        xv = self.x_host[torch.from_numpy(rows)].double().numpy()
        W = O.fp8_table_f64(O.E4M3)[self.w_host.view(torch.uint8).numpy()] * self.s_host.double().numpy()[:, None]
        ref = xv @ W.T
        S = np.abs(xv) @ np.abs(W).T
        got = self.h_out[torch.from_numpy(rows)].double().numpy()
        return bool(np.all(np.abs(got - ref) <= O.bf16_ulp(ref) + 2.0 ** -20 * S))

    @staticmethod
    def cpu_run(args, reps=1):
        """float32 matmul of a (at most) 256-row slice against the dequantised
        weights (CPU torch); in GB/s of the step's bytes for M <= 256."""
        from fp4_fp8_for_torch_mps.workloads import rowwise_operands
        M, N, K, _, _ = LinearFp8W._dims(args)
        threads = torch.get_num_threads()
        rows = min(256, M)

        def make():
            _, w, _, sw = rowwise_operands(1, N, K)
            return (w.float() * sw.reshape(-1, 1),
                    torch.randn(rows, K, generator=torch.Generator().manual_seed(0)).to(torch.bfloat16).float())
        W, A = cpu_input(("linear", M, N, K), make)
        t0 = time.perf_counter()
        for _ in range(reps):
            (A @ W.t()).to(torch.bfloat16)
        dt = (time.perf_counter() - t0) / reps
        sample = f"{rows}x{N}x{K} f32 matmul, weights dequantised beforehand (CPU torch, {threads} threads)"
        if M <= 256:
            return (N * K + rows * K * 2 + rows * N * 2) / dt / 1e9, threads, sample, dt
        return 2.0 * rows * N * K / dt / 1e12, threads, sample, dt


class LlamaFp8:
    """32 Llama-3-8B-shaped layers, e4m3 weights, per-token e4m3 activations,
    every linear through torch._scaled_mm; batch 8 x 2048 tokens split across
    the ranks (strong scaling). Metric: tokens/s."""
    name = "llama_fp8"
    bound, kernels_per_step = "tensor", 1
    profile = "scaled_mm_llama_fp8"
    sustained = True  # a step is ~0.1 s of GEMMs at the power cap

    @staticmethod
    def describe(args, ctx):
        layers = args.layers or 32
        return {"metric": "llama_fp8_tokens_per_s", "unit": "tokens/s", "splits": True, "bound": "tensor",
                "dtype": "e4m3 linears (f32 acc), bf16 attention/norms",
                "config": {"workload": "llama_fp8", "layers": layers, "hidden": 4096, "intermediate": 14336,
                           "heads": 32, "kv_heads": 8, "global_batch": 8, "seq_len": 2048,
                           "l2": "activations and weights per step >> L2",
                           "launch": ("every kernel launched from Python" if args.eager else
                                      "forward pass captured once as a CUDA graph, replayed per step"),
                           "parallelism": f"batch/{ctx.ws}" if ctx.ws > 1 else "single"}}

    def __init__(self, ctx, args):
        from fp4_fp8_for_torch_mps.workloads import LLAMA, Fp8LlamaStack, llama_input
        ws = ctx.ws
        total_batch, self.seq = 8, 2048
        if total_batch % ws:
            raise SystemExit(f"llama_fp8: batch {total_batch} does not split over {ws} ranks")
        self.batch = total_batch // ws
        self.layers = args.layers or LLAMA["layers"]
        self.model = Fp8LlamaStack(torch.device("cuda"), layers=self.layers, seed=0)
        x = llama_input(total_batch, self.seq, seed=0)
        t = self.batch * self.seq
        self.x_host = x[ctx.rank * t:(ctx.rank + 1) * t].contiguous()
        self.x = self.x_host.cuda()
        self.work = float(t)                       # tokens per step on this rank
        self.h2d = self.d2h = self.x_host.numel() * 2
        self.stream = torch.cuda.current_stream()
        self.h_in = self.x_host.pin_memory()
        self.h_out = torch.empty_like(self.x_host).pin_memory()
        self.gemm_flops = self.model.gemm_flops(t)
        from fp4_fp8_for_torch_mps import _lib as L
        self.L = L
        self.eager = bool(getattr(args, "eager", False))

    def step(self):
        self.y = self.model.forward(self.x, self.batch, self.seq)

    graph = None
    graph_launches = 0

    def capture(self, steps):
        """The forward pass (32 layers, ~500 kernels) captured once as a CUDA
        graph; each timed step replays it, so no host dispatch gap sits
        between kernels. Every kernel of the eager step runs in the replay."""
        self.steps = steps
        if self.eager:
            return
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        self.graph = torch.cuda.CUDAGraph()
        n0 = self.L.launch_count()
        with torch.cuda.stream(side):
            with torch.cuda.graph(self.graph, stream=side):
                self.y = self.model.forward(self.x, self.batch, self.seq)
        self.per_forward = self.L.launch_count() - n0
        self.graph_launches = self.per_forward * steps
        torch.cuda.synchronize()

    def replay(self):
        for _ in range(self.steps):
            if self.graph is None:
                self.step()
            else:
                self.graph.replay()

    def e2e_step(self):
        x = self.h_in.to("cuda", non_blocking=True)
        y = self.model.forward(x, self.batch, self.seq)
        self.h_out.copy_(y, non_blocking=True)

    def gemm_roofline(self):
        """Average achieved TFLOP/s of the _scaled_mm launches in one
        instrumented step (CUDA events on the launching stream)."""
        ev = []
        for l in self.model.layers:
            l.gemm_events = ev
        torch.cuda.synchronize()
        self.step()
        torch.cuda.synchronize()
        for l in self.model.layers:
            l.gemm_events = None
        ms = sum(a.elapsed_time(b) for a, b, _ in ev)
        flops = sum(f for _, _, f in ev)
        return flops / (ms * 1e-3) / 1e12, ms, len(ev)

    def check(self):
        y = self.h_out.float()
        return bool(torch.isfinite(y).all().item()) and y.std().item() > 0

    @staticmethod
    def cpu_run(args, reps=1):
        return llama_cpu_tokens_per_s(args.layers or 32, reps)


def llama_cpu_tokens_per_s(layers: int, reps: int = 1, seq: int = 256):
    """One Llama-shaped layer on the host in float32 with e4m3-dequantised
    random weights over one `seq`-token sequence; tokens/s extrapolated to
    `layers` layers."""
    import torch.nn.functional as F
    from fp4_fp8_for_torch_mps.workloads import LLAMA, _rope, quantize_per_tensor, rope_tables
    c = LLAMA
    h, f, hd, nkv = c["hidden"], c["intermediate"], c["head_dim"], c["kv_heads"]
    g = torch.Generator().manual_seed(0)

    def w(n, k):
        q, sc = quantize_per_tensor(torch.randn(n, k, generator=g) * 0.02)
        return q.float() * sc

    wqkv, wo, wgu, wd = w(h + 2 * nkv * hd, h), w(h, h), w(2 * f, h), w(h, f)
    x = torch.randn(seq, h, generator=g)
    cos, sin = (t.float() for t in rope_tables(seq, "cpu"))
    threads = torch.get_num_threads()
    t0 = time.perf_counter()
    for _ in range(reps):
        r = F.rms_norm(x, (h,), None, c["eps"])
        q, k, v = (r @ wqkv.t()).split([h, nkv * hd, nkv * hd], dim=1)
        q = _rope(q.view(1, seq, 32, hd), cos, sin).transpose(1, 2)
        k = _rope(k.view(1, seq, nkv, hd), cos, sin).transpose(1, 2)
        v = v.view(1, seq, nkv, hd).transpose(1, 2)
        a = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
        y = x + a.transpose(1, 2).reshape(seq, h) @ wo.t()
        gg, u = (F.rms_norm(y, (h,), None, c["eps"]) @ wgu.t()).chunk(2, dim=1)
        y = y + (F.silu(gg) * u) @ wd.t()
    dt = (time.perf_counter() - t0) / reps
    return seq / (dt * layers), threads, \
        f"one layer, 1x{seq} tokens, float32 e4m3-dequantised weights (CPU torch, {threads} threads), " \
        f"x{layers} layers", dt * layers * (8 * 2048 / seq)


WORKLOADS = {"fp4_decode": Fp4Decode, "fp8_roundtrip": Fp8RoundTrip, "llama_fp8": LlamaFp8,
             "scaled_mm": _gemm_factory(False, False), "scaled_mm_rowwise": _gemm_factory(True, False),
             "fp4_scaled_mm": _gemm_factory(False, True),
             "scaled_mm_small_m": ScaledMMSmallM, "linear_fp8w": LinearFp8W,
             "fp8_quantize": _quantize_factory("fp8_quantize"),
             "fp8_quantize_noalloc": _quantize_factory("fp8_quantize_noalloc"),
             "quantize_rows": _quantize_factory("quantize_rows"),
             "fp4_quantize": _quantize_factory("fp4_quantize")}


# ---------------------------------------------------------------- the two arms
def base_line(desc, ctx, args):
    return {"metric": desc["metric"], "unit": desc["unit"], "n_gpus": ctx.ws, "steps": args.steps,
            "warmup": max(args.warmup, 3), "higher_is_better": True, "vs_baseline": None,
            "data": "synthetic", "scaling": ctx.scaling(desc["splits"]), "config": desc["config"]}


def reference_line(args, ctx):
    """The CPU implementation of the path on the host cores, on the GPU arm's
    metric, unit and config: `steps` samples, median value."""
    cls = WORKLOADS[args.workload]
    desc = cls.describe(args, ctx)
    vals = [cls.cpu_run(args) for _ in range(max(1, min(args.steps, 3 if args.workload == "llama_fp8" else 50)))]
    v = statistics.median(x[0] for x in vals)
    line = base_line(desc, ctx, args)
    line.update({"value": round(v, 4), "ms_per_step": round(statistics.median(x[3] for x in vals) * 1e3, 3),
                 "dtype": "cpu", "impl": "reference",
                 "cpu_baseline": {"value": round(v, 4), "unit": desc["unit"], "cores": vals[0][1], "kind": "port",
                                  "sample": vals[0][2]},
                 "e2e": {"value": round(v, 4), "unit": desc["unit"], "h2d_bytes_per_step": 0,
                         "d2h_bytes_per_step": 0}})
    return line


def gpu_line(args, ctx):
    """One workload on this rank's GPU; returns the JSON line on rank 0."""
    import torch.distributed as dist
    from fp4_fp8_for_torch_mps import _lib as L
    cls = WORKLOADS[args.workload]
    desc = cls.describe(args, ctx)
    w = cls(ctx, args)
    warm = max(args.warmup, 3)
    for _ in range(warm):
        w.step()
    torch.cuda.synchronize()
    graphed = hasattr(w, "capture")
    if graphed:  # launch-bound workloads: the K timed steps replay as one CUDA graph
        w.capture(args.steps)
        w.replay()  # warm replay of the captured steps
        torch.cuda.synchronize()
        region = w.replay
    else:
        def region():
            for _ in range(args.steps):
                w.step()

    sampler = ClockSampler(ctx.local)
    sampler.start()
    n0 = L.launch_count()
    regions = repeated_regions(region, w.stream, ctx.dist_on)
    launches = L.launch_count() - n0 + getattr(w, "graph_launches", 0) * len(regions)
    clocks = sampler.stop()

    for _ in range(2):
        w.e2e_step()
    torch.cuda.synchronize()
    e2e_steps = max(3, min(args.steps, 10))

    def e2e_region():
        for _ in range(e2e_steps):
            w.e2e_step()
    e2e_ms = timed_region(e2e_region, torch.cuda.current_stream(), ctx.dist_on)
    ok = all_true(w.check(), ctx)
    gather = gather_line(w, ctx) if (args.gather and ctx.sharded and hasattr(w, "M_total")) else None

    # the whole job's work per step: summed over ranks
    total = torch.tensor([float(w.work)], dtype=torch.float64, device="cuda")
    if ctx.dist_on:
        dist.all_reduce(total)
    total_work = total.item()

    pk, pk_kind = peaks()
    ms_step = statistics.median(regions) / args.steps
    scale = {"GB/s": 1e9, "TFLOP/s": 1e12}.get(desc["unit"], 1.0)
    value = total_work / (ms_step * 1e-3) / scale
    e2e_value = total_work / (e2e_ms / e2e_steps * 1e-3) / scale
    achieved = total_work / ctx.ws / (ms_step * 1e-3) / scale  # per GPU, per launch-averaged step
    extra = {}
    if hasattr(w, "gemm_roofline"):
        achieved, gemm_ms, n_gemm = w.gemm_roofline()
        extra = {"gemm_ms_per_step": round(gemm_ms, 3), "gemm_launches_per_step": n_gemm,
                 "gemm_share": round(gemm_ms / ms_step, 4)}
    # Tensor-core lines: the timed repeats run the GEMM back to back for at
    # least MIN_REGION_MS, long enough for the 1000 W power cap to lower the
    # clocks, so they are held against the sustained GEMM peak (measured the
    # same way, back to back); the fastest repeat (burst clocks) is reported
    # beside it against the burst peak.
    bound = desc["bound"]
    long_run = bound in ("tensor", "tensor_bf16", "tensor_fp4") and sum(regions) >= 100.0
    bf16_key = "bf16_tflops_sustained" if (getattr(w, "sustained", False) or long_run) \
        and "bf16_tflops_sustained" in pk else "bf16_tflops"
    if long_run and not extra:
        burst = total_work / ctx.ws / (min(regions) / args.steps * 1e-3) / scale
        burst_peak = {"tensor": 2.0, "tensor_fp4": 4.0}.get(bound, 1.0) * pk["bf16_tflops"]
        extra = {"burst": {"achieved": round(burst, 2), "peak": burst_peak, "frac": round(burst / burst_peak, 4),
                           "from": "fastest timed repeat, against the burst peak"}}
    if bound == "hbm":
        peak, punit, psrc = pk["hbm_gbs"], "GB/s", f"{pk_kind} hbm_gbs"
        if getattr(w, "two_read_bytes", None):
            moved = w.two_read_bytes / w.work * achieved
            extra["two_read_bound"] = {
                "bytes_per_step": int(w.two_read_bytes), "achieved": round(moved, 2),
                "frac": round(moved / peak, 4),
                "note": "bytes a per-tensor quantisation must move (input read twice: amax, then encode; "
                        "output written once) over the step time, against the same HBM peak"}
    elif bound == "tensor_bf16":
        peak, punit, psrc = pk[bf16_key], "TFLOP/s", f"{pk_kind} {bf16_key}"
    elif bound == "tensor_fp4":
        peak, punit = 4.0 * pk[bf16_key], "TFLOP/s"
        psrc = f"4 x {pk_kind} {bf16_key} (dense fp4 kind::mxf4 issue rate is four times bf16 on tcgen05)"
    else:
        peak, punit = 2.0 * pk[bf16_key], "TFLOP/s"
        psrc = f"2 x {pk_kind} {bf16_key} (dense fp8/fp6/fp4 kind::f8f6f4 issue rate is twice bf16 on tcgen05)"
    cpu = None
    if ctx.rank == 0 and ctx.ws == 1:
        v, cores, sample, _ = cls.cpu_run(args)
        cpu = {"value": round(v, 4), "unit": desc["unit"], "cores": cores, "kind": "port", "sample": sample}
    line = None
    if ctx.rank == 0:
        line = base_line(desc, ctx, args)
        line.update({
            "value": round(value, 3), "ms_per_step": round(ms_step, 4),
            "ms_per_step_spread": [round(min(regions) / args.steps, 4), round(max(regions) / args.steps, 4)],
            "timed_repeats": len(regions), "timed_ms_total": round(sum(regions), 1),
            "dtype": desc["dtype"],
            "e2e": {"value": round(e2e_value, 3), "unit": desc["unit"], "h2d_bytes_per_step": int(w.h2d),
                    "d2h_bytes_per_step": int(w.d2h)},
            "roofline": {"bound": "tensor" if bound.startswith("tensor") else bound, "achieved": round(achieved, 2),
                         "peak": peak, "unit": punit, "frac": round(achieved / peak, 4), "peak_source": psrc,
                         "per": "GPU" if ctx.ws > 1 else "launch-averaged step",
                         "traffic": profile_traffic(getattr(w, "profile", None)), **extra},
            "cpu_baseline": cpu,
            "gpu_launches": int(launches),
            "clocks": clocks,
            "result_check": ok,
        })
        if hasattr(w, "accuracy"):
            line["accuracy"] = w.accuracy
        if gather is not None:
            line["gather"] = gather
    del w
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return line


# ---------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default=None, choices=sorted(WORKLOADS),
                    help="one workload (default: the four-line suite ending with fp4_decode)")
    ap.add_argument("--weak", action="store_true",
                    help="N > 1: a full-size replica per rank instead of splitting the workload's rows")
    ap.add_argument("--size", type=int, default=8192)
    ap.add_argument("--shape", type=int, default=0, choices=[0, 1, 2])
    ap.add_argument("--layers", type=int, default=0, help="llama_fp8: number of layers (default 32)")
    ap.add_argument("--elems", type=int, default=0,
                    help="fp8_roundtrip: elements per step (default 4096x4096; 1073741824 for the 1 Gi sweep)")
    ap.add_argument("--src", default="f32", choices=["f32", "bf16", "f16"], help="fp8_roundtrip: source dtype")
    ap.add_argument("--fmt", default="e4m3", choices=["e4m3", "e5m2"], help="fp8_roundtrip: fp8 format")
    ap.add_argument("--eager", action="store_true",
                    help="llama_fp8: launch every kernel from Python instead of replaying a captured graph")
    ap.add_argument("--gather", action="store_true",
                    help="GEMMs at N > 1: also time the replicated-output all-gather of the row-split result")
    ap.add_argument("--m", type=int, default=0,
                    help="rows of A / x: scaled_mm_small_m (default 16), linear_fp8w (default 16384)")
    args = ap.parse_args()
    rank, local, ws = rank_info()
    ctx = Ctx(rank, local, ws, args.weak)

    if args.workload is None:
        plan = []
        for wl, over in DEFAULT_SUITE:
            a = copy.copy(args)
            a.workload = wl
            for k, v in over.items():
                setattr(a, k, v)
            plan.append(a)
    else:
        plan = [args]

    if args.impl == "reference":
        if rank != 0:
            return 0
        for a in plan:
            print(json.dumps(reference_line(a, ctx)), flush=True)
        return 0

    torch.cuda.set_device(local)
    if ctx.dist_on:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    import fp4_fp8_for_torch_mps  # noqa: F401  (registers the overrides used by e2e)
    try:
        for a in plan:
            line = gpu_line(a, ctx)
            if line is not None:
                print(json.dumps(line), flush=True)
    finally:
        if ctx.dist_on:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
