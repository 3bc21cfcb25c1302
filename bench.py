#!/usr/bin/env python
"""Benchmark of the FP8/FP4 hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload fp4_decode|fp8_roundtrip|scaled_mm|scaled_mm_rowwise]
                    [--size S] [--shape I]

Default workload (the one the headline metric is quoted on): FP4 decode of a
16384x8192 float4_e2m1fn_x2 tensor (uniform bytes, arange(256) prefix) to a
16384x16384 bf16 tensor times a per-tensor fp32 scale 0.37. One step = one
decode of the whole tensor. Inputs (128 MiB) plus outputs (512 MiB) exceed the
126 MB L2, so no flush is needed between steps.

Other workloads (one JSON line each, same keys):
  fp8_roundtrip      4096x4096 f32 -> e4m3 -> f32 (two kernels per step), four
                     rotating buffer sets so the 144 MB working set of one
                     step is not served from L2
  scaled_mm          torch._scaled_mm e4m3 x e4m3, per-tensor scales, bf16
                     out, M=N=K=--size (default 8192)
  scaled_mm_rowwise  rowwise scales, LLM shape --shape 0|1|2 of
                     (16384,4096,4096), (16384,14336,4096), (16384,4096,14336)

Multi-GPU (torchrun, one process per GPU): every rank runs its own full-size
workload (weak scaling, no collective on the data path); the time is the max
over ranks of the device-timed region.

`value` is device-resident throughput summed over ranks; `e2e` is the same
metric through the package's public API with pinned host buffers (host to
device copy, kernel, device to host copy inside the timed region, pipelined
over chunks on three streams for the converters).

`--impl reference` times the CPU implementation of the path on the host cores
with all threads, on rank 0 only: the reference's own kernels are Metal
compute for Apple GPUs and cannot run here, so the CPU oracle (a C
restatement of the same conversions) stands in for the converters and a
float32 dequantise-and-matmul stands in for the GEMM.
"""
from __future__ import annotations

import argparse
import datetime
import json
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

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


# ---------------------------------------------------------------- environment
def rank_info():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0")),
            int(os.environ.get("WORLD_SIZE", "1")))


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
                    ["nvidia-smi", f"--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.sw_power_cap,"
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


def timed_region(step, steps: int, stream, dist_on: bool):
    """`steps` steps between barrier + synchronize; device ms, max over ranks."""
    import torch.distributed as dist
    if dist_on:
        dist.barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        step()
    end.record(stream)
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    if dist_on:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    return ms


def gather_line(w, ws, rank, reps=10):
    """Replicated-output mode of the row-sharded GEMM, timed on its own: each
    rank contributes its block of M/ws output rows and
    parallel.gather_rows (one NCCL all_gather_into_tensor over
    NVLink/NVSwitch) assembles the full M x N result on every rank."""
    from fp4_fp8_for_torch_mps.parallel import gather_rows, shard_rows
    M = w.out.shape[0]
    s, e = shard_rows(M, ws, rank)
    local = w.out[s:e]
    for _ in range(3):
        full = gather_rows(local, M)
    torch.cuda.synchronize()
    ms = timed_region(lambda: gather_rows(local, M), reps, torch.cuda.current_stream(), True) / reps
    nbytes = full.numel() * full.element_size()
    return {"ms": round(ms, 4), "bytes_per_rank": local.numel() * local.element_size(), "bytes_total": nbytes,
            "algbw_GBps": round(nbytes / (ms * 1e-3) / 1e9, 1),
            "busbw_GBps": round(nbytes * (ws - 1) / ws / (ms * 1e-3) / 1e9, 1),
            "op": "parallel.gather_rows -> NCCL all_gather_into_tensor", "timed": "separately, not in value"}


def chunked_e2e(chunks, streams, body):
    """Run body(i, stream_index) for every chunk on rotating streams, joined
    to the current stream (so events on it bracket the whole pipeline)."""
    cur = torch.cuda.current_stream()
    ev = torch.cuda.Event()
    ev.record(cur)
    for s in streams:
        s.wait_event(ev)
    for i in range(chunks):
        j = i % len(streams)
        with torch.cuda.stream(streams[j]):
            body(i, j)
    for s in streams:
        cur.wait_stream(s)


# ---------------------------------------------------------------- workloads
class Fp4Decode:
    name = "fp4_decode"
    metric = "fp4_decode_GBps"
    unit, bound, kernels_per_step = "GB/s", "hbm", 1
    profile = "fp4_decode_16384x8192_bf16"
    dtype = "u8->bf16"

    def __init__(self, rank, args):
        from fp4_fp8_for_torch_mps import _lib as L
        from fp4_fp8_for_torch_mps import fp8_mps_native as nat
        from fp4_fp8_for_torch_mps.workloads import FP4_DECODE_SCALE, fp4_decode_input
        self.L, self.nat, self.scale_v = L, nat, FP4_DECODE_SCALE
        self.x_host = fp4_decode_input(seed=rank)
        rows, cols = self.x_host.shape
        self.rows, self.cols = rows, cols
        self.x = self.x_host.cuda()
        self.out = torch.empty(rows, 2 * cols, dtype=torch.bfloat16, device="cuda")
        self.scale = torch.tensor([FP4_DECODE_SCALE], dtype=torch.float32, device="cuda")
        self.work = self.x.numel() * 5            # bytes read + written per step
        self.h2d, self.d2h = self.x.numel(), self.x.numel() * 4
        self.config = {"workload": "fp4_decode", "shape": [rows, cols], "out": f"bf16[{rows},{2 * cols}]",
                       "scale": FP4_DECODE_SCALE, "l2": "640 MiB per step > L2, no flush"}
        self.stream = torch.cuda.current_stream()
        self.lib = L.lib()
        # end-to-end buffers: pinned host in/out, 16 row chunks on 3 streams
        self.h_in = self.x_host.pin_memory()
        self.h_out = torch.empty(rows, 2 * cols, dtype=torch.bfloat16).pin_memory()
        self.chunks = 16
        self.crow = rows // self.chunks
        self.streams = [torch.cuda.Stream() for _ in range(3)]
        self.d_in = [torch.empty(self.crow, cols, dtype=torch.uint8, device="cuda") for _ in self.streams]
        self.d_out = [torch.empty(self.crow, 2 * cols, dtype=torch.bfloat16, device="cuda") for _ in self.streams]

    def step(self):
        rc = self.lib.fp8b200_decode_fp4(self.x.data_ptr(), self.x.numel(), self.out.data_ptr(), self.L.BF16,
                                         self.scale.data_ptr(), self.L.SCALE_F32, self.stream.cuda_stream)
        if rc:
            self.L.check(rc, "fp4 decode")

    def e2e_step(self):
        c = self.crow

        def body(i, j):
            self.d_in[j].copy_(self.h_in[i * c:(i + 1) * c], non_blocking=True)
            self.nat.fp4_decode(self.d_in[j].view(torch.float4_e2m1fn_x2), torch.bfloat16,
                                scale=self.scale, out=self.d_out[j])
            self.h_out[i * c:(i + 1) * c].copy_(self.d_out[j], non_blocking=True)
        chunked_e2e(self.chunks, self.streams, body)

    def check(self):
        import numpy as np
        from oracle import oracle as O
        ref = O.fp4_decode(self.x_host[-64:].numpy(), 1, self.scale_v)
        return bool(np.array_equal(ref, self.h_out[-64:].view(torch.int16).numpy().view(np.uint16)))

    @staticmethod
    def cpu_run(rows=16384, reps=3):
        from oracle import oracle as O
        from fp4_fp8_for_torch_mps.workloads import FP4_DECODE_SCALE, fp4_decode_input
        x = fp4_decode_input(seed=0, rows=rows).numpy()
        threads = os.cpu_count() or 1
        O.fp4_decode(x, 1, FP4_DECODE_SCALE, threads=threads)
        t0 = time.perf_counter()
        for _ in range(reps):
            O.fp4_decode(x, 1, FP4_DECODE_SCALE, threads=threads)
        dt = (time.perf_counter() - t0) / reps
        return x.size * 5 / dt / 1e9, threads, f"{rows}x{x.shape[1]} bytes -> bf16 x 0.37 per pass (oracle, C)"


class Fp8RoundTrip:
    """FP8 round trip: encode `--src` (f32, bf16 or f16) to `--fmt` (e4m3fn
    or e5m2), decode back to the source dtype. Default 4096x4096 f32 ->
    e4m3fn -> f32; `--elems` sets the element count (the 4096x4096 planted
    input is tiled; e.g. 1073741824 for a 1 Gi-element sweep)."""
    name = "fp8_roundtrip"
    metric = "fp8_roundtrip_GBps"
    unit, bound, kernels_per_step = "GB/s", "hbm", 2
    profile = "fp8_encode_decode_4096x4096"
    SRC = {"f32": (torch.float32, 0, 4), "bf16": (torch.bfloat16, 1, 2), "f16": (torch.float16, 2, 2)}
    FMT = {"e4m3": ("e4m3fn", 0, torch.float8_e4m3fn), "e5m2": ("e5m2", 1, torch.float8_e5m2)}

    def __init__(self, rank, args):
        from fp4_fp8_for_torch_mps import _lib as L
        from fp4_fp8_for_torch_mps import fp8_mps_native as nat
        from fp4_fp8_for_torch_mps.workloads import fp8_roundtrip_input
        self.L, self.nat = L, nat
        src, fmt = getattr(args, "src", "f32"), getattr(args, "fmt", "e4m3")
        self.src, self.fmt_key = src, fmt
        self.tdt, self.sdt, eb = self.SRC[src]
        self.fmt_name, self.fmt, self.fp8 = self.FMT[fmt]
        self.l_sdt = (L.F32, L.BF16, L.F16)[self.sdt]
        self.l_fmt = (L.E4M3, L.E5M2)[self.fmt]
        base = fp8_roundtrip_input(seed=rank)
        n = getattr(args, "elems", 0) or base.numel()
        flat = base.view(-1)
        if n > flat.numel():
            flat = flat.repeat((n + flat.numel() - 1) // flat.numel())
        self.x_host = flat[:n].to(self.tdt).reshape(base.shape if n == base.numel() else (n,))
        self.dtype = f"{src}->{self.fmt_name}->{src}"
        if (src, fmt, n) != ("f32", "e4m3", base.numel()):
            self.profile = None  # the committed ncu summary covers the default case only
        step_bytes = n * (2 * eb + 2)
        self.SETS = 4 if step_bytes < (1 << 30) else 1
        self.xs = [self.x_host.cuda() for _ in range(self.SETS)]
        self.codes = [torch.empty(n, dtype=torch.uint8, device="cuda") for _ in range(self.SETS)]
        self.back = [torch.empty(n, dtype=self.tdt, device="cuda") for _ in range(self.SETS)]
        self.i = 0
        self.work = step_bytes                   # encode (eb + 1) B/elt + decode (1 + eb) B/elt
        self.h2d, self.d2h = n * eb, n * eb
        self.config = {"workload": "fp8_roundtrip", "shape": list(self.x_host.shape), "src": src,
                       "fp8": self.fmt_name,
                       "l2": (f"{self.SETS} rotating buffer sets ({self.SETS * step_bytes / 2**20:.0f} MiB) > L2"
                              if self.SETS > 1 else f"one buffer set of {step_bytes / 2**20:.0f} MiB > L2")}
        self.stream = torch.cuda.current_stream()
        self.lib = L.lib()
        self.h_in = self.x_host.pin_memory()
        self.h_out = torch.empty_like(self.x_host).pin_memory()
        self.chunks = 8
        self.streams = [torch.cuda.Stream() for _ in range(3)]
        cn = n // self.chunks
        self.cn = cn
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
        for the timed region: the two 13-16 us kernels of a step are
        otherwise bound by host launch cost, and one graph per step still
        leaves a graph-launch gap between steps."""
        side = torch.cuda.Stream()
        self.graph = torch.cuda.CUDAGraph()
        n0 = self.L.launch_count()
        with torch.cuda.stream(side):
            with torch.cuda.graph(self.graph, stream=side):
                for j in range(steps):
                    self._launch((self.i + j) % self.SETS, side.cuda_stream)
        self.graph_launches = self.L.launch_count() - n0
        torch.cuda.synchronize()
        self.config["launch"] = f"one CUDA graph of {steps} steps (encode + decode kernels each)"

    def replay(self):
        self.graph.replay()

    def step(self):
        k = self.i % self.SETS
        self.i += 1
        self._launch(k, self.stream.cuda_stream)

    def e2e_step(self):
        c = self.cn
        hin, hout = self.h_in.view(-1), self.h_out.view(-1)

        def body(i, j):
            self.d_in[j].copy_(hin[i * c:(i + 1) * c], non_blocking=True)
            self.nat.encode_fp8(self.d_in[j], self.fp8, out=self.d_mid[j])
            self.nat.decode_fp8(self.d_mid[j], self.fp8, self.tdt, out=self.d_out[j])
            hout[i * c:(i + 1) * c].copy_(self.d_out[j], non_blocking=True)
        chunked_e2e(self.chunks, self.streams, body)

    def check(self):
        import numpy as np
        from oracle import oracle as O
        npu = np.uint32 if self.sdt == 0 else np.uint16
        ity = torch.int32 if self.sdt == 0 else torch.int16
        xb = self.x_host.view(-1)[:1 << 16].view(ity).numpy().view(npu)
        ref = O.decode_fp8(O.encode_fp8(xb, self.sdt, self.fmt), self.fmt, self.sdt)
        got = self.h_out.view(-1)[:1 << 16].view(ity).numpy().view(npu)
        return bool(np.array_equal(ref, got))

    def cpu_run(self):
        return Fp8RoundTrip.cpu_run_for(src=self.src, fmt=self.fmt_key)

    @staticmethod
    def cpu_run_for(rows=4096, reps=3, src="f32", fmt="e4m3"):
        import numpy as np
        from oracle import oracle as O
        from fp4_fp8_for_torch_mps.workloads import fp8_roundtrip_input
        tdt, sdt, eb = Fp8RoundTrip.SRC[src]
        f = Fp8RoundTrip.FMT[fmt][1]
        x = fp8_roundtrip_input(0).view(-1)[: rows * 4096].to(tdt)
        xb = x.view(torch.int32 if sdt == 0 else torch.int16).numpy().view(np.uint32 if sdt == 0 else np.uint16)
        threads = os.cpu_count() or 1
        t0 = time.perf_counter()
        for _ in range(reps):
            O.decode_fp8(O.encode_fp8(xb, sdt, f, threads=threads), f, sdt, threads=threads)
        dt = (time.perf_counter() - t0) / reps
        return xb.size * (2 * eb + 2) / dt / 1e9, threads, \
            f"{rows}x4096 {src} encode to {Fp8RoundTrip.FMT[fmt][0]} + decode per pass (oracle, C)"


class Quantize:
    """Dynamic quantisation rows of the path, each one bench line:
    fp8_quantize  -- per-tensor e4m3 (amax pass, scale, encode pass) of the
                     4096x4096 f32 FP8 round-trip input; bytes = in + out;
    quantize_rows -- per-token e4m3 of 16384x4096 bf16 activations (the
                     Llama-shaped stack's linear inputs); bytes = in + out + scales;
    fp4_quantize  -- per-tensor FP4 (amax pass, scale, nibble encode) of
                     16384x16384 bf16 (the FP4 decode output's shape)."""
    unit, bound = "GB/s", "hbm"
    profile = None

    def __init__(self, rank, args, kind):
        from fp4_fp8_for_torch_mps import _lib as L
        from fp4_fp8_for_torch_mps.workloads import fp8_roundtrip_input
        self.L, self.kind = L, kind
        self.name, self.metric = kind, f"{kind}_GBps"
        g = torch.Generator().manual_seed(rank)
        if kind == "fp8_quantize":
            self.x_host = fp8_roundtrip_input(seed=rank)
            self.dtype, sets = "f32->e4m3 (per tensor)", 4
        elif kind == "quantize_rows":
            self.x_host = torch.randn(16384, 4096, generator=g).to(torch.bfloat16)
            self.dtype, sets = "bf16->e4m3 (per row)", 2
        else:
            self.x_host = (torch.randn(16384, 16384, generator=g) * 3).to(torch.bfloat16)
            self.dtype, sets = "bf16->fp4 e2m1 (per tensor)", 1
        x = self.x_host
        n, eb = x.numel(), x.element_size()
        self.n, self.sets = n, sets
        self.xs = [x.cuda() for _ in range(sets)]
        out_n = n // 2 if kind == "fp4_quantize" else n
        self.outs = [torch.empty(out_n, dtype=torch.uint8, device="cuda") for _ in range(sets)]
        rows = x.shape[0]
        self.scales = torch.empty(rows if kind == "quantize_rows" else 2, dtype=torch.float32, device="cuda")
        self.scratch = torch.zeros(1, dtype=torch.int32, device="cuda")
        self.work = n * eb + out_n + (4 * rows if kind == "quantize_rows" else 0)
        self.h2d, self.d2h = n * eb, out_n + 4 * (rows if kind == "quantize_rows" else 1)
        per_set = n * eb + out_n
        self.config = {"workload": kind, "shape": list(x.shape), "src": str(x.dtype).replace("torch.", ""),
                       "l2": (f"{sets} rotating buffer sets ({sets * per_set / 2**20:.0f} MiB) > L2" if sets > 1
                              else f"{per_set / 2**20:.0f} MiB per step > L2")}
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
        through the buffer sets), replayed once for the timed region: a step
        is up to three kernels of a few to 25 us (clear, amax, encode for
        the per-tensor rows), which host launches one by one cannot keep
        fed; the host-launched path is what `e2e` measures."""
        side = torch.cuda.Stream()
        self.graph = torch.cuda.CUDAGraph()
        n0 = self.L.launch_count()
        with torch.cuda.stream(side):
            with torch.cuda.graph(self.graph, stream=side):
                for j in range(steps):
                    self._launch((self.i + j) % self.sets, side.cuda_stream)
        self.graph_launches = self.L.launch_count() - n0
        torch.cuda.synchronize()
        self.config["launch"] = f"one CUDA graph of {steps} steps"

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
        if self.kind == "fp8_quantize":
            scale = 448.0 / amax if amax > 0 else 1.0
            ok = np.array_equal(got[:m], O.encode_fp8_scaled(xf, scale, 0))
        else:
            scale = 6.0 / amax if amax > 0 else 1.0
            ok = np.array_equal(got[:m // 2], O.fp4_encode_ref(xf, scale))
        return bool(ok and self.h_scales[0].item() == np.float32(1.0 / scale))

    def cpu_run(self):
        return Quantize.cpu_run_for(self.kind)

    @staticmethod
    def cpu_run_for(kind, reps=1):
        """The oracle (C, one thread) on a 1024-row sample: amax, scale, encode."""
        import numpy as np
        from oracle import oracle as O
        from fp4_fp8_for_torch_mps.workloads import fp8_roundtrip_input
        g = torch.Generator().manual_seed(0)
        if kind == "fp8_quantize":
            x = fp8_roundtrip_input(0)[:1024].numpy()
            eb, outb = 4, 1.0
        elif kind == "quantize_rows":
            x = torch.randn(1024, 4096, generator=g).to(torch.bfloat16).float().numpy()
            eb, outb = 2, 1.0
        else:
            x = (torch.randn(1024, 16384, generator=g) * 3).to(torch.bfloat16).float().numpy()
            eb, outb = 2, 0.5
        t0 = time.perf_counter()
        for _ in range(reps):
            if kind == "quantize_rows":
                for r in range(x.shape[0]):
                    a = float(np.max(np.abs(x[r])))
                    O.encode_fp8_scaled(x[r], np.float32(448.0 / a if a > 0 else 1.0), 0)
            elif kind == "fp8_quantize":
                O.encode_fp8_scaled(x, 448.0 / float(np.max(np.abs(x))), 0)
            else:
                O.fp4_encode_ref(x, 6.0 / float(np.max(np.abs(x))))
        dt = (time.perf_counter() - t0) / reps
        return x.size * (eb + outb) / dt / 1e9, 1, f"{x.shape[0]}x{x.shape[1]} {kind} per pass (oracle, C, 1 thread)"


class ScaledMM:
    name = "scaled_mm"
    unit, bound, kernels_per_step = "TFLOP/s", "tensor", 1
    dtype = "e4m3xe4m3->bf16 (f32 acc)"

    def __init__(self, rank, args, rowwise=False):
        from fp4_fp8_for_torch_mps import _lib as L
        from fp4_fp8_for_torch_mps.workloads import ROWWISE_SHAPES, rowwise_operands, scaled_mm_operands
        self.L = L
        if rowwise:
            M, N, K = ROWWISE_SHAPES[args.shape]
            aq, bq, sa, sb = rowwise_operands(M, N, K, seed=rank)
            self.name, self.metric = "scaled_mm_rowwise", "scaled_mm_rowwise_TFLOPS"
        else:
            M = N = K = args.size
            aq, bq, sa, sb = scaled_mm_operands(M, N, K, seed=rank)
            self.name, self.metric = "scaled_mm", "scaled_mm_TFLOPS"
        self.M, self.N, self.K = M, N, K
        self.profile = f"{self.name}_{M}x{N}x{K}"
        self.a_host, self.b_host, self.sa_host, self.sb_host = aq, bq, sa, sb
        self.a, self.b = aq.cuda(), bq.cuda()
        self.sa, self.sb = sa.cuda(), sb.cuda()
        self.out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        self.work = 2.0 * M * N * K
        self.h2d = M * K + N * K
        self.d2h = M * N * 2
        l2 = "A+B+D {:.0f} MiB".format((M * K + N * K + 2 * M * N) / 2**20)
        self.config = {"workload": self.name, "M": M, "N": N, "K": K,
                       "scales": "rowwise" if rowwise else "tensorwise", "out": "bf16",
                       "l2": l2 + (" > L2, no flush" if (M * K + N * K + 2 * M * N) > 126e6 else
                                   " (one GEMM reads each operand tile from L2 repeatedly by design)")}
        self.stream = torch.cuda.current_stream()
        self.lib = L.lib()
        self.la = L.SCALE_ROWWISE if rowwise else L.SCALE_TENSOR
        self.h_a, self.h_b = aq.view(torch.uint8).pin_memory(), bq.view(torch.uint8).pin_memory()
        self.h_out = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()
        self.d_a = torch.empty_like(self.a.view(torch.uint8))
        self.d_b = torch.empty_like(self.b.view(torch.uint8))

    def step(self):
        L = self.L
        rc = self.lib.fp8b200_scaled_mm(self.a.data_ptr(), L.E4M3, self.K, self.b.data_ptr(), L.E4M3, self.K,
                                        self.M, self.N, self.K, self.sa.data_ptr(), self.la, self.sb.data_ptr(),
                                        self.la, None, 0, None, self.out.data_ptr(), L.BF16, self.N,
                                        self.stream.cuda_stream)
        if rc:
            L.check(rc, "scaled_mm")

    def e2e_step(self):
        # public API: torch._scaled_mm on operands copied from pinned host memory
        self.d_a.copy_(self.h_a, non_blocking=True)
        self.d_b.copy_(self.h_b, non_blocking=True)
        r = torch._scaled_mm(self.d_a.view(torch.float8_e4m3fn), self.d_b.view(torch.float8_e4m3fn).t(),
                             self.sa, self.sb, out_dtype=torch.bfloat16)
        self.h_out.copy_(r, non_blocking=True)

    def check(self):
        import numpy as np
        from oracle import oracle as O
        rows = np.arange(0, self.M, max(1, self.M // 16))[:16]
        ref, S = O.scaled_mm_ref(self.a_host.view(torch.uint8).numpy(), self.b_host.view(torch.uint8).numpy(),
                                 self.sa_host.numpy().reshape(-1), self.sb_host.numpy().reshape(-1), rows=rows)
        got = self.h_out[torch.from_numpy(rows)].float().double().numpy()
        return bool(np.all(np.abs(got - ref) <= O.bf16_ulp(ref) + 2.0 ** -20 * S))

    def cpu_run(self, reps=1):
        """float32 dequantise-and-matmul on the host (the CPU path for this
        GEMM; CPU torch._scaled_mm is per-tensor only and ~0.1 GFLOP/s), on a
        256-row slice of A."""
        threads = torch.get_num_threads()
        rows = 256
        A = self.a_host[:rows].float() * self.sa_host.reshape(-1, 1)[:rows] if self.sa_host.numel() > 1 \
            else self.a_host[:rows].float() * self.sa_host
        B = self.b_host.float() * (self.sb_host.reshape(-1, 1) if self.sb_host.numel() > 1 else self.sb_host)
        t0 = time.perf_counter()
        for _ in range(reps):
            (A @ B.t()).to(torch.bfloat16)
        dt = (time.perf_counter() - t0) / reps
        return 2.0 * rows * self.N * self.K / dt / 1e12, threads, \
            f"{rows}x{self.N}x{self.K} f32 dequantised matmul (CPU torch, {threads} threads)"


class ScaledMMSmallM:
    """Decode-sized rowwise GEMM: M (--m, default 16) activation rows against
    Llama-shaped e4m3 weights (N, K from --shape). The weights dominate the
    bytes, so the bound is HBM: work = N*K + M*K bytes read + 2*M*N written.
    Weight sets rotate (>= 300 MB in total) so that every step reads its
    weights from HBM, not L2."""
    name = "scaled_mm_small_m"
    metric = "scaled_mm_small_m_GBps"
    unit, bound, kernels_per_step = "GB/s", "hbm", 1
    dtype = "e4m3xe4m3->bf16 (f32 acc)"

    def __init__(self, rank, args):
        from fp4_fp8_for_torch_mps import _lib as L
        from fp4_fp8_for_torch_mps.workloads import ROWWISE_SHAPES, rowwise_operands
        self.L = L
        _, N, K = ROWWISE_SHAPES[args.shape]
        M = args.m or 16
        aq, bq, sa, sb = rowwise_operands(M, N, K, seed=rank)
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
        self.config = {"workload": self.name, "M": M, "N": N, "K": K, "scales": "rowwise", "out": "bf16",
                       "l2": f"{self.nsets} rotating weight sets, {self.nsets * N * K / 2**20:.0f} MiB > L2"}
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

    def cpu_run(self, reps=3):
        """float32 dequantise-and-matmul of the same M rows on the host."""
        threads = torch.get_num_threads()
        A = self.a_host.float() * self.sa_host.reshape(-1, 1)
        B = self.b_host.float() * self.sb_host.reshape(-1, 1)
        t0 = time.perf_counter()
        for _ in range(reps):
            (A @ B.t()).to(torch.bfloat16)
        dt = (time.perf_counter() - t0) / reps
        return self.work / dt / 1e9, threads, \
            f"{self.M}x{self.N}x{self.K} f32 dequantised matmul (CPU torch, {threads} threads; weights pre-dequantised)"


class LinearFp8W:
    """FP8-weight linear with dequant-on-load: y = x @ (w * s)^T, x bf16
    (M, K) N(0,1), w e4m3 quantised per output channel from N(0, 0.02),
    Llama shapes (N, K from --shape, M from --m, default 16384). Compute in
    bf16 on the tensor cores: the roofline peak is the measured bf16 rate;
    for M <= 256 the weight bytes bound it and the line reports GB/s (weights
    + x + y) against HBM."""
    name = "linear_fp8w"
    metric = "linear_fp8w_TFLOPS"
    unit, bound, kernels_per_step = "TFLOP/s", "tensor_bf16", 1
    dtype = "bf16 x e4m3 (dequantised on load) -> bf16, f32 acc"

    def __init__(self, rank, args):
        from fp4_fp8_for_torch_mps import _lib as L
        from fp4_fp8_for_torch_mps import fp8_mps_native as nat
        from fp4_fp8_for_torch_mps.workloads import ROWWISE_SHAPES, rowwise_operands
        self.L, self.nat = L, nat
        _, N, K = ROWWISE_SHAPES[args.shape]
        M = args.m or 16384
        g = torch.Generator().manual_seed(rank)
        self.x_host = torch.randn(M, K, generator=g).to(torch.bfloat16)
        _, wq, _, sw = rowwise_operands(1, N, K, seed=rank)
        self.w_host, self.s_host = wq, sw.reshape(-1)
        self.M, self.N, self.K = M, N, K
        self.profile = f"{self.name}_{M}x{N}x{K}"
        self.x, self.w, self.s = self.x_host.cuda(), wq.cuda(), self.s_host.cuda()
        foot = M * K * 2 + N * K + M * N * 2
        # weight sets rotate when one step's operands would fit in L2 (decode-sized M)
        self.nsets = 1 if foot > 300_000_000 else max(2, min(32, -(-300_000_000 // (N * K))))
        self.ws = [self.w] + [self.w.clone() for _ in range(self.nsets - 1)]
        self.i = 0
        self.out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        self.work = 2.0 * M * N * K
        if M <= 256:  # decode-sized M: the weight bytes bound it, so report bytes against HBM
            self.metric, self.unit, self.bound = "linear_fp8w_GBps", "GB/s", "hbm"
            self.work = float(N * K + M * K * 2 + M * N * 2)
        self.h2d, self.d2h = M * K * 2, M * N * 2
        self.config = {"workload": self.name, "M": M, "N": N, "K": K, "weights": "e4m3, per-channel scale",
                       "activations": "bf16", "out": "bf16",
                       "l2": ("x+w+y {:.0f} MiB > L2".format(foot / 2**20) if self.nsets == 1 else
                              f"{self.nsets} rotating weight sets, {self.nsets * N * K / 2**20:.0f} MiB > L2")}
        self.stream = torch.cuda.current_stream()
        self.lib = L.lib()
        self.h_x = self.x_host.pin_memory()
        self.h_out = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()
        self.d_x = torch.empty_like(self.x)

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

    def cpu_run(self, reps=1):
        """float32 matmul of a (at most) 256-row slice against the dequantised
        weights (CPU torch); in GB/s of the step's bytes for M <= 256."""
        threads = torch.get_num_threads()
        W = self.w_host.float() * self.s_host.reshape(-1, 1)
        rows = min(256, self.M)
        A = self.x_host[:rows].float()
        t0 = time.perf_counter()
        for _ in range(reps):
            (A @ W.t()).to(torch.bfloat16)
        dt = (time.perf_counter() - t0) / reps
        sample = f"{rows}x{self.N}x{self.K} f32 matmul, weights dequantised beforehand (CPU torch, {threads} threads)"
        if self.M <= 256:
            return (self.N * self.K + rows * self.K * 2 + rows * self.N * 2) / dt / 1e9, threads, sample
        return 2.0 * rows * self.N * self.K / dt / 1e12, threads, sample


class LlamaFp8:
    """32 Llama-3-8B-shaped layers, e4m3 weights, per-token e4m3 activations,
    every linear through torch._scaled_mm; batch 8 x 2048 tokens split across
    the ranks (strong scaling). Metric: tokens/s."""
    name = "llama_fp8"
    metric = "llama_fp8_tokens_per_s"
    unit, bound, kernels_per_step = "tokens/s", "tensor", 1
    profile = "scaled_mm_llama_fp8"
    dtype = "e4m3 linears (f32 acc), bf16 attention/norms"
    scaling = "strong"
    sustained = True  # a step is ~0.1 s of GEMMs at the power cap

    def __init__(self, rank, args):
        from fp4_fp8_for_torch_mps.workloads import LLAMA, Fp8LlamaStack, llama_input
        ws = int(os.environ.get("WORLD_SIZE", "1"))
        total_batch, self.seq = 8, 2048
        if total_batch % ws:
            raise SystemExit(f"llama_fp8: batch {total_batch} does not split over {ws} ranks")
        self.batch = total_batch // ws
        self.layers = args.layers or LLAMA["layers"]
        self.model = Fp8LlamaStack(torch.device("cuda"), layers=self.layers, seed=0)
        x = llama_input(total_batch, self.seq, seed=0)
        t = self.batch * self.seq
        self.x_host = x[rank * t:(rank + 1) * t].contiguous()
        self.x = self.x_host.cuda()
        self.work = float(t)                       # tokens per step on this rank
        self.h2d = self.d2h = self.x_host.numel() * 2
        self.config = {"workload": "llama_fp8", "layers": self.layers, "hidden": 4096, "intermediate": 14336,
                       "heads": 32, "kv_heads": 8, "global_batch": total_batch, "seq_len": self.seq,
                       "tokens_per_rank": t, "l2": "activations and weights per step >> L2"}
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
        if getattr(self, "eager", False):
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
        self.config["launch"] = "forward pass captured once as a CUDA graph, replayed per step"

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

    def cpu_run(self, reps=1):
        return llama_cpu_tokens_per_s(self.layers, reps)


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
        f"one layer, 1x{seq} tokens, float32 e4m3-dequantised weights (CPU torch, {threads} threads), x{layers} layers"


WORKLOADS = {"fp4_decode": Fp4Decode, "fp8_roundtrip": Fp8RoundTrip, "llama_fp8": LlamaFp8,
             "scaled_mm": lambda r, a: ScaledMM(r, a, False),
             "scaled_mm_rowwise": lambda r, a: ScaledMM(r, a, True), "scaled_mm_small_m": ScaledMMSmallM,
             "linear_fp8w": LinearFp8W,
             "fp8_quantize": lambda r, a: Quantize(r, a, "fp8_quantize"),
             "quantize_rows": lambda r, a: Quantize(r, a, "quantize_rows"),
             "fp4_quantize": lambda r, a: Quantize(r, a, "fp4_quantize")}


# ---------------------------------------------------------------- reference arm
def reference_line(args):
    if args.workload == "llama_fp8":
        layers = args.layers or 32
        vals = [llama_cpu_tokens_per_s(layers) for _ in range(max(min(args.steps, 3), 1))]
        unit, metric = "tokens/s", "llama_fp8_tokens_per_s"
        config = {"workload": "llama_fp8", "layers": layers, "global_batch": 8, "seq_len": 2048}
    elif args.workload == "fp4_decode":
        vals = [Fp4Decode.cpu_run(rows=16384, reps=1) for _ in range(max(args.steps, 1))]
        unit, metric = "GB/s", "fp4_decode_GBps"
        config = {"workload": "fp4_decode", "shape": [16384, 8192], "out": "bf16", "scale": 0.37}
    elif args.workload == "fp8_roundtrip":
        vals = [Fp8RoundTrip.cpu_run_for(rows=4096, reps=1, src=args.src, fmt=args.fmt) for _ in range(max(args.steps, 1))]
        unit, metric = "GB/s", "fp8_roundtrip_GBps"
        config = {"workload": "fp8_roundtrip", "shape": [args.elems] if args.elems else [4096, 4096],
                  "src": args.src, "fp8": Fp8RoundTrip.FMT[args.fmt][0],
                  "sample": "4096x4096 elements per step" if args.elems else "full size"}
    elif args.workload in ("fp8_quantize", "quantize_rows", "fp4_quantize"):
        vals = [Quantize.cpu_run_for(args.workload) for _ in range(max(args.steps, 1))]
        unit, metric = "GB/s", f"{args.workload}_GBps"
        shape = {"fp8_quantize": [4096, 4096], "quantize_rows": [16384, 4096], "fp4_quantize": [16384, 16384]}
        config = {"workload": args.workload, "shape": shape[args.workload], "sample": "1024 rows per step"}
    elif args.workload == "linear_fp8w":
        w = LinearFp8W.__new__(LinearFp8W)
        from fp4_fp8_for_torch_mps.workloads import ROWWISE_SHAPES, rowwise_operands
        _, N, K = ROWWISE_SHAPES[args.shape]
        M = args.m or 16384
        w.x_host = torch.randn(min(256, M), K, generator=torch.Generator().manual_seed(0)).to(torch.bfloat16)
        _, w.w_host, _, sw = rowwise_operands(1, N, K)
        w.s_host = sw.reshape(-1)
        w.M, w.N, w.K = M, N, K
        vals = [w.cpu_run() for _ in range(max(args.steps, 1))]
        unit, metric = ("GB/s", "linear_fp8w_GBps") if M <= 256 else ("TFLOP/s", "linear_fp8w_TFLOPS")
        config = {"workload": args.workload, "M": M, "N": N, "K": K, "out": "bf16"}
    elif args.workload == "scaled_mm_small_m":
        w = ScaledMMSmallM.__new__(ScaledMMSmallM)
        from fp4_fp8_for_torch_mps.workloads import ROWWISE_SHAPES, rowwise_operands
        _, N, K = ROWWISE_SHAPES[args.shape]
        m = args.m or 16
        w.a_host, w.b_host, w.sa_host, w.sb_host = rowwise_operands(m, N, K)
        w.M, w.N, w.K = m, N, K
        w.work = float(N * K + m * K + 2 * m * N)
        vals = [w.cpu_run() for _ in range(max(args.steps, 1))]
        unit, metric = "GB/s", "scaled_mm_small_m_GBps"
        config = {"workload": args.workload, "M": m, "N": N, "K": K, "out": "bf16"}
    else:
        w = ScaledMM.__new__(ScaledMM)
        from fp4_fp8_for_torch_mps.workloads import ROWWISE_SHAPES, rowwise_operands, scaled_mm_operands
        rowwise = args.workload == "scaled_mm_rowwise"
        M, N, K = ROWWISE_SHAPES[args.shape] if rowwise else (args.size,) * 3
        # a 256-row slice of A is all the CPU path runs
        ops = (rowwise_operands if rowwise else scaled_mm_operands)(256, N, K)
        w.a_host, w.b_host, w.sa_host, w.sb_host = ops
        w.M, w.N, w.K = 256, N, K
        vals = [w.cpu_run() for _ in range(max(args.steps, 1))]
        unit, metric = "TFLOP/s", ("scaled_mm_rowwise_TFLOPS" if rowwise else "scaled_mm_TFLOPS")
        config = {"workload": args.workload, "M": M, "N": N, "K": K, "out": "bf16"}
    v = statistics.median(x[0] for x in vals)
    return {"metric": metric, "value": round(v, 4), "unit": unit, "config": config,
            "cpu_baseline": {"value": round(v, 4), "unit": unit, "cores": vals[0][1], "kind": "port",
                             "sample": vals[0][2]},
            "dtype": "cpu"}


# ---------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="fp4_decode", choices=sorted(WORKLOADS))
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
                    help="scaled_mm at N > 1: also time the replicated-output all-gather of the M-sharded result")
    ap.add_argument("--m", type=int, default=0,
                    help="rows of A / x: scaled_mm_small_m (default 16), linear_fp8w (default 16384)")
    args = ap.parse_args()
    rank, local, ws = rank_info()

    if args.impl == "reference":
        if rank != 0:
            return 0
        line = reference_line(args)
        line.update({"impl": "reference", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                     "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "data": "synthetic",
                     "e2e": {"value": line["value"], "unit": line["unit"],
                             "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
        print(json.dumps(line))
        return 0

    dist_on = ws > 1
    torch.cuda.set_device(local)
    if dist_on:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    import fp4_fp8_for_torch_mps  # noqa: F401  (registers the overrides used by e2e)
    from fp4_fp8_for_torch_mps import _lib as L

    w = WORKLOADS[args.workload](rank, args)
    warm = max(args.warmup, 3)
    for _ in range(warm):
        w.step()
    torch.cuda.synchronize()
    graphed = hasattr(w, "capture")
    if graphed:  # launch-bound workloads: the K timed steps replay as one CUDA graph
        w.capture(args.steps)
        w.replay()  # warm replay of the captured steps
        torch.cuda.synchronize()

    sampler = ClockSampler(local)
    sampler.start()
    n0 = L.launch_count()
    if graphed:
        ms = timed_region(w.replay, 1, w.stream, dist_on)
    else:
        ms = timed_region(w.step, args.steps, w.stream, dist_on)
    launches = L.launch_count() - n0 + getattr(w, "graph_launches", 0)
    clocks = sampler.stop()

    for _ in range(2):
        w.e2e_step()
    torch.cuda.synchronize()
    e2e_steps = max(3, min(args.steps, 10))
    e2e_ms = timed_region(w.e2e_step, e2e_steps, torch.cuda.current_stream(), dist_on)
    ok = w.check()
    gather = gather_line(w, ws, rank) if (args.gather and dist_on and hasattr(w, "out")) else None

    pk, pk_kind = peaks()
    per_step_s = ms / args.steps * 1e-3
    scale = {"GB/s": 1e9, "TFLOP/s": 1e12}.get(w.unit, 1.0)
    value = w.work * ws / per_step_s / scale
    e2e_value = w.work * ws / (e2e_ms / e2e_steps * 1e-3) / scale
    achieved = w.work / per_step_s / scale  # per GPU, per launch-averaged step
    extra = {}
    if hasattr(w, "gemm_roofline"):
        achieved, gemm_ms, n_gemm = w.gemm_roofline()
        extra = {"gemm_ms_per_step": round(gemm_ms, 3), "gemm_launches_per_step": n_gemm,
                 "gemm_share": round(gemm_ms / (ms / args.steps), 4)}
    # GEMMs timed inside a long step (seconds under the power cap) against the
    # sustained GEMM peak, GEMMs timed on their own against the burst peak
    bf16_key = "bf16_tflops_sustained" if getattr(w, "sustained", False) and "bf16_tflops_sustained" in pk \
        else "bf16_tflops"
    if w.bound == "hbm":
        peak, punit, psrc = pk["hbm_gbs"], "GB/s", f"{pk_kind} hbm_gbs"
    elif w.bound == "tensor_bf16":
        peak, punit, psrc = pk[bf16_key], "TFLOP/s", f"{pk_kind} {bf16_key}"
    else:
        peak, punit = 2.0 * pk[bf16_key], "TFLOP/s"
        psrc = f"2 x {pk_kind} {bf16_key} (dense fp8 issue rate is twice bf16 on tcgen05)"
    cpu = None
    if rank == 0:
        v, cores, sample = w.cpu_run() if hasattr(w, "cpu_run") else (None, None, None)
        cpu = {"value": round(v, 4), "unit": w.unit, "cores": cores, "kind": "port", "sample": sample}
    if dist_on:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": w.metric, "value": round(value, 3), "unit": w.unit, "n_gpus": ws, "steps": args.steps,
        "warmup": warm, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
        "vs_baseline": None, "dtype": w.dtype, "data": "synthetic",
        "scaling": getattr(w, "scaling", "weak"),
        "config": dict(w.config, parallelism=f"replicas{ws}" if ws > 1 else "single"),
        "e2e": {"value": round(e2e_value, 3), "unit": w.unit, "h2d_bytes_per_step": int(w.h2d),
                "d2h_bytes_per_step": int(w.d2h)},
        "roofline": {"bound": "tensor" if w.bound == "tensor_bf16" else w.bound, "achieved": round(achieved, 2), "peak": peak, "unit": punit,
                     "frac": round(achieved / peak, 4), "peak_source": psrc,
                     "traffic": profile_traffic(w.profile), **extra},
        "cpu_baseline": cpu,
        "gpu_launches": int(launches),
        "clocks": clocks,
        "result_check": ok,
    }
    if gather is not None:
        line["gather"] = gather
    print(json.dumps(line))
    return 0


if __name__ == "__main__":
    sys.exit(main())
