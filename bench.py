#!/usr/bin/env python
"""Benchmark of the NVFP4 FFN path on B200: the 30-layer FFN stack of the Wan-1.3B DiT
(d_model 1536, d_ff 8960, GELU-tanh, bias; 30 distinct layers) over 15360 tokens, the
token rows split across the GPUs, one process per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference]
                    [--workload c4|c5]
    torchrun --nproc-per-node N bench.py --gpus N ...     (N > 1)

A step is one pass of the stack over one batch: 15360 synthetic tokens (four 48x80
latent frames, N(0,1), seed 3), split into N contiguous row blocks of 15360/N rows
(strong scaling: the total work is fixed as N grows).  Each rank runs the 30 layers on
its rows with replicated weights (layer l: W ~ N(0, 0.02), bias ~ N(0, 0.01), seeded,
``workloads.stack_layer_params(l)``), then one NCCL all-gather over NVLink assembles the
[15360, 1536] output on every rank; the all-gather is inside the step.  The 30 layers' 120
kernel launches are captured once into a CUDA graph and each step replays it.  `--workload c5`
runs the 4K-stream batch instead: 64800 tokens (two 135x240 frames, Student-t(4) x 0.5,
seed 4).  The weights alone (464 MB) and each layer's intermediate are far larger than
the 126 MB L2, so no step finds its operands in L2.

Prints one JSON line (rank 0).  `value` is whole-job tokens/s (tokens through all 30
layers, gathered) with inputs resident in HBM, timed on the device as the max over
ranks; `e2e` is the same metric through the public module API (NVFP4FFN modules and
sharding.gather_rows) with host buffers: every step uploads each rank's rows from pinned
host memory and rank 0 reads the gathered output back, inside the timed region;
`roofline` describes the layer's two GEMM launches (per-launch CUDA-event times from a
second pass over the same steps); `cpu_baseline` times the reference arithmetic (the
CPU oracle) on this host.  Extras after the timed steps (skip with --no-extras):
`single_layer` (one layer over 7680 tokens per GPU), `c5_stack` (the 64800-token batch),
`stack_check` (N > 1: shards with whole-tensor global scales gathered equal the
unsharded stack bit for bit), `quantize_sweep`, `fp8_mode`, `pil_resize`, `dit_block`
(rank 0), and at N = 1 `flashinfer` (the reference's own sm_100 kernels on the same
box and shapes).  The all-gather's time and bus bandwidth come last.

`--impl reference` times the reference's NVFP4 FFN arithmetic on the host CPU (the
oracle restatement; the reference itself needs FlashInfer on a GPU) with all host
threads, on bounded samples of the same workload.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

D_MODEL, D_FF = 1536, 8960
LAYERS = 30
TOKENS = 7680                       # the single-layer extra: tokens per GPU
FLOP_PER_TOKEN = 2 * D_MODEL * D_FF * 2
ROTATE = 8
METRIC = "nvfp4_ffn_tokens_per_s"
# launches per layer of fvq_nvfp4_ffn: amax+quantize(x), GEMM1 (+bias, GELU, amax), quantize(h), GEMM2
LAUNCHES_PER_LAYER = 4
STACK_WORKLOADS = {
    "c4": {"total": 15360, "dist": "gaussian", "seed": 3,
           "name": "ffn_stack30_d1536_ff8960_15360tok_rows_sharded_allgather",
           "input": "N(0,1) bf16, seed 3 (four 48x80 latent frames)"},
    "c5": {"total": 64800, "dist": "student_t", "seed": 4,
           "name": "ffn_stack30_d1536_ff8960_64800tok_rows_sharded_allgather",
           "input": "Student-t(4) x 0.5 bf16, seed 4 (two 135x240 latent frames, 4K output)"},
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("native", "reference"), default="native")
    ap.add_argument("--workload", choices=tuple(STACK_WORKLOADS), default="c4")
    ap.add_argument("--tokens", type=int, default=TOKENS,
                    help="tokens per GPU of the single-layer extra and of --case layer")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the separate measurements that follow the timed steps")
    ap.add_argument("--cpu-seconds", type=float, default=20.0,
                    help="wall-time budget of the CPU baseline sample")
    ap.add_argument("--case", choices=("stack", "shard", "layer", "layer_fused", "fp8_ffn",
                                       "pil_resize", "dit_block", "sustained"),
                    default="stack",
                    help="stack: the benchmark (default); shard: the stack on rank 0's row block "
                         "of a --shard-of N split, on this GPU alone (no collective); layer / "
                         "layer_fused: one fvq_nvfp4_ffn / fvq_nvfp4_ffn_fused layer over --tokens "
                         "rows, --steps calls (e.g. under a profiler); sustained: each of the "
                         "layer's launches, cuBLASLt on the same operands and the stack step over "
                         "--tokens rows, each back to back for seconds under the power cap, with "
                         "clock, power and energy per launch; fp8_ffn / "
                         "pil_resize / dit_block: only that separate measurement, one JSON line")
    ap.add_argument("--shard-of", type=int, default=8,
                    help="--case shard: the number of ranks whose first row block is run")
    return ap.parse_args()


def env_rank():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0")),
            int(os.environ.get("WORLD_SIZE", "1")))


# ---------------------------------------------------------------- clocks
class NvmlClockSampler:
    """SM clock, power and clock-event reasons read through NVML every 2 ms from a
    thread of this process, so that even a timed region of a few tens of
    milliseconds is sampled (nvidia-smi takes longer than that to start)."""

    def __init__(self, gpu_id: str):
        import pynvml
        self.nv = pynvml
        pynvml.nvmlInit()
        self.h = pynvml.nvmlDeviceGetHandleByUUID(gpu_id.encode())
        self.smax = float(pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM))
        self.samples: list[tuple[float, float, int]] = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                sm = float(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                pw = nv.nvmlDeviceGetPowerUsage(self.h) / 1000.0
                rs = int(nv.nvmlDeviceGetCurrentClocksEventReasons(self.h))
                self.samples.append((sm, pw, rs))
            except nv.NVMLError:
                pass
            self._stop.wait(0.002)

    def start(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()

    def stop(self) -> dict:
        self._stop.set()
        if self._t:
            self._t.join(timeout=2)
        nv = self.nv
        names = {nv.nvmlClocksEventReasonHwSlowdown: "hw_slowdown",
                 nv.nvmlClocksEventReasonHwThermalSlowdown: "hw_thermal_slowdown",
                 nv.nvmlClocksEventReasonSwThermalSlowdown: "sw_thermal_slowdown",
                 nv.nvmlClocksEventReasonSwPowerCap: "sw_power_cap"}
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.smax, "reasons": ["no samples"], "samples": 0}
        reasons = sorted({nm for _, _, rs in self.samples for bit, nm in names.items() if rs & bit})
        return {"sm_mhz": statistics.median(sm for sm, _, _ in self.samples), "sm_max_mhz": self.smax,
                "reasons": reasons, "samples": len(self.samples),
                "power_w_max": max(pw for _, pw, _ in self.samples), "source": "nvml"}


def clock_sampler(gpu_id: str):
    try:
        return NvmlClockSampler(gpu_id)
    except Exception:  # noqa: BLE001 - NVML missing or refused: fall back to nvidia-smi
        return ClockSampler(gpu_id)


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons while the GPU is busy."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", self.gpu_id], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
            return
        self._t = threading.Thread(target=self._read, daemon=True)
        self._t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self._t:
            self._t.join(timeout=2)
        sm, smax, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power)}


# ---------------------------------------------------------------- the stack workload
def to_dev(torch, bits: np.ndarray, dev):
    return torch.from_numpy(np.ascontiguousarray(bits).astype(np.int16)).view(torch.bfloat16).to(dev)


def stack_input_rows(wl: dict, r0: int, r1: int) -> np.ndarray:
    """bf16 bits of rows [r0, r1) of the workload's input.  The whole input is generated
    from its seed, so every rank cuts its block out of the same tensor."""
    from flashvsr_optimizations_b200 import workloads as W
    gen = W.gaussian if wl["dist"] == "gaussian" else W.student_t
    return np.ascontiguousarray(gen(wl["total"], D_MODEL, seed=wl["seed"])[r0:r1])


class StackWeights:
    """The 30 layers' NVFP4 weights on one GPU, quantized by the library exactly as
    QuantLinear(linear, 'nvfp4') quantizes them (global scale, then the 128x4-swizzled
    codes and scales), with their C-ABI descriptors.  keep_bf16 also keeps the bf16
    weights (for building the reference's own modules on the same weights)."""

    def __init__(self, torch, ops, dev, layers=LAYERS, keep_bf16=False):
        from flashvsr_optimizations_b200 import _lib, workloads as W
        self.tensors, self.structs, self.bf16 = [], [], []
        for layer in range(layers):
            w1, b1, w2, b2 = W.stack_layer_params(layer)
            pair = []
            for wb, bb, in_f, out_f in ((w1, b1, D_MODEL, D_FF), (w2, b2, D_FF, D_MODEL)):
                w, b = to_dev(torch, wb, dev), to_dev(torch, bb, dev)
                g = ops.global_scale(w)
                q, s = ops.nvfp4_quantize(w, g)
                self.tensors.append((q, s, g, b))
                pair.append(_lib.FvqLinear(q.data_ptr(), s.data_ptr(), g.data_ptr(), b.data_ptr(),
                                           in_f, out_f))
                if keep_bf16:
                    self.bf16.append((w, b))
                del w
            self.structs.append(tuple(pair))

    def modules(self, torch):
        """The public modules: one NVFP4FFN (QuantLinear, GELU(tanh), QuantLinear) per layer."""
        from flashvsr_optimizations_b200.ffn_quantization import NVFP4FFN, QuantLinear
        mods = []
        for i in range(0, len(self.tensors), 2):
            (q1, s1, g1, b1), (q2, s2, g2, b2) = self.tensors[i], self.tensors[i + 1]
            mods.append(NVFP4FFN(QuantLinear.from_quantized(q1, s1, g1, b1, D_MODEL),
                                 torch.nn.GELU(approximate="tanh"),
                                 QuantLinear.from_quantized(q2, s2, g2, b2, D_FF)))
        return mods


class StackRun:
    """The stack on this rank's row block: one fvq_nvfp4_ffn_chain call per layer (four
    launches, ping-pong activation buffers, one workspace; each layer hands the next the
    max |y| of its output, so only layer 0 runs the amax pass over its input), then (N > 1)
    the NCCL all-gather of the last layer's rows into the full output."""

    def __init__(self, torch, lib, dev, stream, weights, wl, world, rank):
        from flashvsr_optimizations_b200.sharding import row_range
        self.total = wl["total"]
        r0, r1 = row_range(self.total, world, rank)
        self.rows = r1 - r0
        self.x = to_dev(torch, stack_input_rows(wl, r0, r1), dev)
        self.ws_bytes = lib.fvq_nvfp4_ffn_workspace_bytes(self.rows, D_MODEL, D_FF)
        self.ws = torch.zeros(self.ws_bytes, dtype=torch.uint8, device=dev)
        self.bufs = [torch.empty(self.rows, D_MODEL, dtype=torch.bfloat16, device=dev)
                     for _ in range(2)]
        self.amax = torch.zeros(2, dtype=torch.float32, device=dev)   # max |y|, ping-pong
        self.out = (torch.empty(self.total, D_MODEL, dtype=torch.bfloat16, device=dev)
                    if world > 1 else None)
        self.lib, self.sptr, self.structs, self.world = lib, stream.cuda_stream, weights.structs, world
        self.dev, self.graph, self.graph_out = dev, None, None

    def layers(self, profile: list | None = None):
        """The 30 layers on this rank's rows; with `profile`, each layer runs through
        fvq_nvfp4_ffn_chain_profile (events around its four launches, one host wait per
        layer) and appends the four device times (ms)."""
        cur = self.x
        last = len(self.structs) - 1
        a0, a1 = self.amax.data_ptr(), self.amax.data_ptr() + 4
        for i, (l1, l2) in enumerate(self.structs):
            out = self.bufs[i % 2]
            x_amax = None if i == 0 else (a0, a1)[(i - 1) % 2]
            y_amax = None if i == last else (a0, a1)[i % 2]
            args = (cur.data_ptr(), self.rows, ctypes.byref(l1), ctypes.byref(l2), out.data_ptr(),
                    x_amax, y_amax, self.ws.data_ptr(), self.ws_bytes, self.sptr)
            if profile is None:
                rc = self.lib.fvq_nvfp4_ffn_chain(*args)
            else:
                ms = (ctypes.c_float * 4)()
                rc = self.lib.fvq_nvfp4_ffn_chain_profile(*args, ms)
                profile.append(list(ms))
            if rc != 0:
                raise RuntimeError(self.lib.fvq_last_error().decode())
            cur = out
        return cur

    def capture(self, torch):
        """The 30 layers' 120 launches captured once into a CUDA graph, which step() then
        replays on the current stream (the same kernels on the same buffers, no host work per
        layer).  Warm-up passes run on the capture stream first."""
        side = torch.cuda.Stream(self.dev)
        side.wait_stream(torch.cuda.current_stream(self.dev))
        sptr, self.sptr = self.sptr, side.cuda_stream
        try:
            with torch.cuda.stream(side):
                for _ in range(2):
                    self.layers()
            torch.cuda.current_stream(self.dev).wait_stream(side)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=side):
                self.graph_out = self.layers()
        finally:
            self.sptr = sptr

    def step(self):
        if self.graph is not None:
            self.graph.replay()
            y = self.graph_out
        else:
            y = self.layers()
        if self.world > 1:
            from flashvsr_optimizations_b200.sharding import gather_rows
            return gather_rows(y, self.total, out=self.out)
        return y


def barrier_sync(torch, dist, dev, world):
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)


def max_over_ranks(torch, dist, dev, world, values: list[float]) -> list[float]:
    if world == 1:
        return values
    t = torch.tensor(values, device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t.tolist()]


def timed_steps(torch, dist, dev, stream, world, fn, steps, warmup, sampler=None) -> float:
    """max over ranks of the device time (ms) of `steps` calls of fn, after `warmup` calls,
    bracketed by a barrier and a device synchronisation on both sides."""
    for i in range(max(3, warmup)):
        fn(i)
    barrier_sync(torch, dist, dev, world)
    if sampler is not None:
        sampler.start()
        if isinstance(sampler, ClockSampler):
            time.sleep(0.15)  # nvidia-smi's start-up
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier_sync(torch, dist, dev, world)
    start.record(stream)
    for i in range(steps):
        fn(i)
    end.record(stream)
    barrier_sync(torch, dist, dev, world)
    return max_over_ranks(torch, dist, dev, world, [start.elapsed_time(end)])[0]


def stack_kernel_timing(torch, dist, dev, world, run, passes) -> dict:
    """Per-launch device times of the layer's four launches over `passes` passes of the
    stack (fvq_nvfp4_ffn_profile: the library's CUDA events around its launches on the
    launching stream), max over ranks of the per-launch means."""
    prof: list = []
    run.layers(prof)                      # one untimed pass
    prof.clear()
    for _ in range(passes):
        run.layers(prof)
    qx, g1, qh, g2 = (statistics.fmean(p[j] for p in prof) for j in range(4))
    qx, g1, qh, g2 = max_over_ranks(torch, dist, dev, world, [qx, g1, qh, g2])
    rows = run.rows
    qh_bytes = rows * D_FF * 2 + rows * D_FF // 2 + (rows + 127) // 128 * 128 * D_FF // 16
    gemm_flop = rows * D_MODEL * D_FF * 2
    return {"rows_per_launch": rows, "launches_timed_per_kernel": len(prof),
            "quant_x_ms": qx, "gemm1_ms": g1, "quant_h_ms": qh, "gemm2_ms": g2, "gemm_ms": g1 + g2,
            "gemm1_tflops": gemm_flop / (g1 * 1e-3) / 1e12, "gemm2_tflops": gemm_flop / (g2 * 1e-3) / 1e12,
            "quant_h_GBps": qh_bytes / (qh * 1e-3) / 1e9, "quant_h_bytes": qh_bytes,
            "note": "each layer's four launches queued back to back; one host wait per layer"}


def stack_e2e(torch, dist, weights, run, dev, world, rank, steps, warmup) -> dict:
    """The stack through the public API with host buffers: per step every rank uploads its
    rows from pinned host memory, runs the 30 NVFP4FFN modules as an NVFP4FFNStack (torch
    custom op fvq::nvfp4_ffn_chain) replayed from a CUDA graph (GraphedFFNStack, one per
    input buffer), all-gathers with sharding.gather_rows, and rank 0 copies the gathered
    [total, 1536] output to pinned host memory.  Uploads, compute and the
    download run on three streams, double-buffered, so one step's copies overlap its
    neighbours' compute."""
    from flashvsr_optimizations_b200.ffn_quantization import NVFP4FFNStack
    from flashvsr_optimizations_b200.sharding import gather_rows
    stack = NVFP4FFNStack(weights.modules(torch))
    xh = run.x.cpu().pin_memory()
    xd = [run.x.clone() for _ in range(2)]
    graphs = [stack.graphed(b) for b in xd]   # the stack over each input buffer, one CUDA graph
    out_rows = run.total if world > 1 else run.rows
    outs = ([torch.empty(run.total, D_MODEL, dtype=torch.bfloat16, device=dev) for _ in range(2)]
            if world > 1 else None)
    yh = ([torch.empty(out_rows, D_MODEL, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
          if rank == 0 else None)
    s_up, s_cmp, s_down = (torch.cuda.Stream(dev) for _ in range(3))
    done_cmp = [torch.cuda.Event() for _ in range(2)]    # compute that read xd[b] finished
    done_down = [torch.cuda.Event() for _ in range(2)]   # download that read outs[b] finished
    for ev in done_cmp:
        ev.record(s_cmp)
    for ev in done_down:
        ev.record(s_down)

    def step(i):
        b = i % 2
        up = torch.cuda.Event()
        with torch.cuda.stream(s_up):
            s_up.wait_event(done_cmp[b])
            xd[b].copy_(xh, non_blocking=True)
            up.record(s_up)
        with torch.cuda.stream(s_cmp):
            s_cmp.wait_event(up)
            s_cmp.wait_event(done_down[b])   # graph b's output (or outs[b]) has been read out
            y = graphs[b]()
            if world > 1:
                y = gather_rows(y, run.total, out=outs[b])
            done_cmp[b].record(s_cmp)
        with torch.cuda.stream(s_down):
            s_down.wait_event(done_cmp[b])
            if rank == 0:
                yh[b].copy_(y, non_blocking=True)
            done_down[b].record(s_down)

    with torch.no_grad():
        for i in range(max(3, warmup)):
            step(i)
        barrier_sync(torch, dist, dev, world)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(s_up)
        for st in (s_cmp, s_down):
            st.wait_event(s)
        for i in range(steps):
            step(i)
        for st in (s_up, s_cmp):
            ev = torch.cuda.Event()
            ev.record(st)
            s_down.wait_event(ev)
        e.record(s_down)
        torch.cuda.synchronize(dev)
    ms = max_over_ranks(torch, dist, dev, world, [s.elapsed_time(e)])[0]
    nbytes = run.total * D_MODEL * 2
    return {"value": run.total * steps / (ms * 1e-3), "unit": "tokens/s",
            "h2d_bytes_per_step": nbytes, "d2h_bytes_per_step": nbytes,
            "steps": steps, "ms_per_step": ms / steps,
            "api": "NVFP4FFNStack of 30 NVFP4FFN modules (torch custom op fvq::nvfp4_ffn_chain), "
                   "replayed as GraphedFFNStack (one CUDA graph per input buffer) + "
                   "sharding.gather_rows; "
                   "each rank uploads its rows, rank 0 downloads the gathered output; "
                   "three streams, double-buffered"}


def stack_check(torch, dist, dev, weights, run, wl, world, rank) -> dict:
    """N > 1: the stack run on the shards with whole-tensor global scales
    (sharding.nvfp4_ffn_global_scales: an all-reduce MAX of amax(x) and of amax(h) per
    layer), gathered, against the unsharded stack on rank 0 (fvq_nvfp4_ffn per layer over
    all rows): the two must agree bit for bit."""
    from flashvsr_optimizations_b200.sharding import gather_rows, nvfp4_ffn_global_scales
    mods = weights.modules(torch)
    with torch.no_grad():
        y = run.x
        for m in mods:
            y = nvfp4_ffn_global_scales(y, m)
        full = gather_rows(y, run.total)
        res = {"check": "30-layer stack, shards with whole-tensor global scales, gathered, vs "
                        "the unsharded stack on rank 0"}
        if rank == 0:
            ref = to_dev(torch, stack_input_rows(wl, 0, run.total), dev)
            for m in mods:
                ref = m(ref)
            res["bit_identical"] = bool(torch.equal(full, ref))
            res["differing_values"] = int((full != ref).sum().item())
            del ref
        del full, y
    barrier_sync(torch, dist, dev, world)
    return res


def fused_requant_timing(torch, dist, dev, stream, world, weights, run, wl, rank) -> dict:
    """The stack with the intermediate quantized inside GEMM1's epilogue (NVFP4FFN with
    delayed h scaling: three launches per layer, no bf16 intermediate), through the public
    modules, on this rank's rows.  Two batches of the stack workload alternate (this
    rank's rows of the workload input and of a second batch with the next seed), so every
    call's estimate of max |h| comes from the other batch, as in a video stream; the
    output is compared with the exact stack on the same batch."""
    from flashvsr_optimizations_b200.sharding import row_range
    mods = weights.modules(torch)
    for m in mods:
        m.set_h_scaling("delayed")
    r0, r1 = row_range(wl["total"], world, rank)
    other = to_dev(torch, stack_input_rows(dict(wl, seed=wl["seed"] + 100), r0, r1), dev)
    batches = [run.x, other]

    def fused(i):
        y = batches[i % 2]
        for m in mods:
            y = m(y)
        return y

    with torch.no_grad():
        fused(1)                                       # exact; seeds the estimates
        ms = timed_steps(torch, dist, dev, stream, world, fused, 4, 2) / 4
        fused(1)
        y_f = fused(0).float()                        # estimates from the other batch
        y_e = run.layers().float()
        rel = float(((y_f - y_e).norm() / y_e.norm()).item())
        flags = max(m.h_flags() for m in mods)
        prof = (ctypes.c_float * 3)()
        hint = torch.full((1,), 4.0, dtype=torch.float32, device=dev)
        seen = torch.zeros(1, dtype=torch.float32, device=dev)
        fl = torch.zeros(1, dtype=torch.int32, device=dev)
        fws_bytes = run.lib.fvq_nvfp4_ffn_fused_workspace_bytes(run.rows, D_MODEL, D_FF)
        fws = torch.zeros(fws_bytes, dtype=torch.uint8, device=dev)
        acc = [[] for _ in range(3)]
        cur = run.x
        for i, (l1, l2) in enumerate(run.structs):
            out = run.bufs[i % 2]
            rc = run.lib.fvq_nvfp4_ffn_fused_profile(
                cur.data_ptr(), run.rows, ctypes.byref(l1), ctypes.byref(l2), out.data_ptr(),
                hint.data_ptr(), 1, seen.data_ptr(), fl.data_ptr(), fws.data_ptr(), fws_bytes,
                run.sptr, prof)
            if rc != 0:
                raise RuntimeError(run.lib.fvq_last_error().decode())
            for j in range(3):
                acc[j].append(prof[j])
            cur = out
    ms, = max_over_ranks(torch, dist, dev, world, [ms])
    kq = [statistics.fmean(a) for a in acc]
    return {"mode": "NVFP4FFN.set_h_scaling('delayed'): GELU + NVFP4 quantization of h in GEMM1's "
                    "epilogue with the previous call's max |h| x 2 (fvq_nvfp4_ffn_fused)",
            "ms_per_stack": ms, "tokens_per_s": wl["total"] / (ms * 1e-3),
            "rel_vs_exact_stack": rel, "flags": flags,
            "kernels_ms": {"quant_x": kq[0], "gemm1_bias_gelu_quantize": kq[1], "gemm2_bias": kq[2]},
            "gemm1_tflops": run.rows * D_MODEL * D_FF * 2 / (kq[1] * 1e-3) / 1e12}


def gather_timing(torch, dist, dev, stream, world, run, reps=20) -> dict:
    """The output all-gather alone (sharding.gather_rows, NCCL all_gather_into_tensor into
    the preallocated output): device time, max over ranks, and NCCL's bus bandwidth."""
    from flashvsr_optimizations_b200.sharding import gather_rows
    local = run.bufs[1]
    ms = timed_steps(torch, dist, dev, stream, world,
                     lambda i: gather_rows(local, run.total, out=run.out), reps, 3) / reps
    nbytes = run.total * D_MODEL * 2
    busbw = (world - 1) / world * nbytes / (ms * 1e-3) / 1e9
    return {"ms": ms, "bytes": nbytes, "busbw_GBps": busbw,
            "frac_of_nvlink_peer_copy": busbw / 770.0,
            "api": "sharding.gather_rows (NCCL all_gather_into_tensor, no padding or concatenation)"}


# ---------------------------------------------------------------- CPU legs
def cpu_stack_tokens_per_s(steps: int, warmup: int, seconds: float, wl: dict) -> dict:
    """The reference NVFP4 FFN arithmetic (the oracle, fp32 BLAS matmul) on host threads, on a
    bounded sample of the stack workload: `rows` tokens of its input through layer 0 of the
    stack per step (every layer has the same shapes and cost), scaled to tokens through all
    30 layers."""
    from oracle import nvfp4_oracle as O
    from flashvsr_optimizations_b200 import workloads as W
    threads = os.cpu_count() or 1
    w1, b1, w2, b2 = W.stack_layer_params(0)
    l1, l2 = O.OracleQuantLinear(w1, b1), O.OracleQuantLinear(w2, b2)
    x_all = stack_input_rows(wl, 0, 4096)
    probe = x_all[:64]
    O.ffn_forward(probe, l1, l2, fp32_matmul=True)
    t0 = time.perf_counter()
    O.ffn_forward(probe, l1, l2, fp32_matmul=True)
    per_tok = (time.perf_counter() - t0) / 64
    rows = int(seconds / max(1, steps + warmup) / max(per_tok, 1e-6))
    rows = max(16, min(1024, rows // 16 * 16))
    for i in range(warmup):
        O.ffn_forward(x_all[(i * rows) % (4096 - rows):][:rows], l1, l2, fp32_matmul=True)
    times = []
    for i in range(steps):
        xs = x_all[(i * rows) % (4096 - rows):][:rows]
        t = time.perf_counter()
        O.ffn_forward(xs, l1, l2, fp32_matmul=True)
        times.append(time.perf_counter() - t)
    per_layer = sum(times)
    return {"value": rows * steps / (per_layer * LAYERS), "unit": "tokens/s", "cores": threads,
            "kind": "port", "rows_per_step": rows, "seconds": per_layer,
            "sample": (f"{steps} steps of {rows} tokens of the {wl['total']}-token stack input through "
                       f"layer 0 (numpy oracle: quantize, dequantize, fp32 BLAS matmul, bias, "
                       f"GELU-tanh, requantize, second GEMM), the per-layer time x {LAYERS} layers; "
                       f"weights quantized once outside the timing; {threads} host threads")}


# ---------------------------------------------------------------- the single-layer extra
def make_sets(torch, ops, dev, tokens, rank):
    """ROTATE distinct (x, layer-1, layer-2) sets on the device, seeded per rank / set."""
    sets = []
    for i in range(ROTATE):
        gen = torch.Generator(device=dev)
        gen.manual_seed(1000 * rank + i + 1)
        z = torch.randn(tokens, D_MODEL, device=dev, generator=gen)
        chi = (torch.randn(4, tokens, D_MODEL, device=dev, generator=gen) ** 2).sum(0) / 4.0
        x = (0.5 * z / chi.sqrt()).to(torch.bfloat16)          # Student-t(4) x 0.5
        layers = []
        for (n, k) in ((D_FF, D_MODEL), (D_MODEL, D_FF)):
            w = (torch.randn(n, k, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
            b = (torch.randn(n, device=dev, generator=gen) * 0.01).to(torch.bfloat16)
            g = ops.global_scale(w)
            q, s = ops.nvfp4_quantize(w, g)
            layers.append((q, s, g, b))
        sets.append((x, layers))
    return sets


def single_layer_timing(torch, dist, ops, lib, dev, stream, world, rank, tokens, steps) -> dict:
    """One FFN layer over `tokens` tokens per GPU (two 48x80 latent frames, Student-t(4) x 0.5)
    with no collective (weak scaling), rotating over ROTATE distinct activation/weight sets
    (312 MB > L2): whole-job tokens/s and the four launches' device times."""
    from flashvsr_optimizations_b200 import _lib
    sets = make_sets(torch, ops, dev, tokens, rank)
    ws_bytes = lib.fvq_nvfp4_ffn_workspace_bytes(tokens, D_MODEL, D_FF)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
    ys = [torch.empty(tokens, D_MODEL, dtype=torch.bfloat16, device=dev) for _ in range(ROTATE)]
    sptr = stream.cuda_stream
    structs = []
    for x, ((q1, s1, g1, b1), (q2, s2, g2, b2)) in sets:
        l1 = _lib.FvqLinear(q1.data_ptr(), s1.data_ptr(), g1.data_ptr(), b1.data_ptr(), D_MODEL, D_FF)
        l2 = _lib.FvqLinear(q2.data_ptr(), s2.data_ptr(), g2.data_ptr(), b2.data_ptr(), D_FF, D_MODEL)
        structs.append((x, l1, l2))

    def step(i):
        x, l1, l2 = structs[i % ROTATE]
        rc = lib.fvq_nvfp4_ffn(x.data_ptr(), tokens, ctypes.byref(l1), ctypes.byref(l2),
                               ys[i % ROTATE].data_ptr(), ws.data_ptr(), ws_bytes, sptr)
        if rc != 0:
            raise RuntimeError(lib.fvq_last_error().decode())

    ms = timed_steps(torch, dist, dev, stream, world, step, steps, 5)
    kms = (ctypes.c_float * 4)()
    acc = [[] for _ in range(4)]
    for i in range(min(steps, 200) + 5):
        x, l1, l2 = structs[i % ROTATE]
        rc = lib.fvq_nvfp4_ffn_profile(x.data_ptr(), tokens, ctypes.byref(l1), ctypes.byref(l2),
                                       ys[i % ROTATE].data_ptr(), ws.data_ptr(), ws_bytes, sptr, kms)
        if rc != 0:
            raise RuntimeError(lib.fvq_last_error().decode())
        if i >= 5:
            for j in range(4):
                acc[j].append(kms[j])
    qx, g1, qh, g2 = max_over_ranks(torch, dist, dev, world, [statistics.fmean(a) for a in acc])
    value = tokens * world * steps / (ms * 1e-3)
    gemm_flop = tokens * FLOP_PER_TOKEN
    return {"workload": "ffn_layer_d1536_ff8960_gelu_tanh_bias_7680tok_per_gpu (weak scaling)",
            "tokens_per_s": value, "ms_per_layer": ms / steps, "steps": steps,
            "tflops": value * FLOP_PER_TOKEN / 1e12,
            "kernels_ms": {"quant_x": qx, "gemm1_bias_gelu_amax": g1, "quant_h": qh, "gemm2_bias": g2},
            "gemm_tflops": gemm_flop / ((g1 + g2) * 1e-3) / 1e12,
            "l2": f"inputs rotate over {ROTATE} distinct activation/weight sets (312 MB > 126 MB L2)"}


# ---------------------------------------------------------------- other separate measurements
def quantize_sweep(torch, lib, dev, stream, hbm_peak) -> list:
    """The standalone activation-quantize sweep: K in {1536, 8960} x M in {1024, 4096, 16384,
    65536}, N(0,1) with 0.1% of elements x50 (seed 2).  Per shape: the quantizer with a
    given scale (one read of x: 2MK + MK/2 + pad128(M)K/16 bytes) and the dynamic path
    (amax + scale + quantize in one launch; x is read twice when it does not fit in L2)."""
    st = stream.cuda_stream
    ws = torch.zeros(lib.fvq_amax_workspace_bytes(), dtype=torch.uint8, device=dev)
    out = []
    for k in (1536, 8960):
        for m in (1024, 4096, 16384, 65536):
            gen = torch.Generator(device=dev)
            gen.manual_seed(2)
            x = torch.randn(m, k, device=dev, generator=gen)
            idx = torch.randint(0, m * k, (max(1, m * k // 1000),), device=dev, generator=gen)
            x.view(-1)[idx] *= 50.0
            x = x.to(torch.bfloat16)
            del idx
            codes = torch.empty(m, k // 2, dtype=torch.uint8, device=dev)
            sf = torch.empty((m + 127) // 128 * 128, k // 16, dtype=torch.uint8, device=dev)
            g = torch.empty(1, dtype=torch.float32, device=dev)

            def dyn():
                lib.fvq_nvfp4_quantize_dynamic(x.data_ptr(), m, k, None, g.data_ptr(), codes.data_ptr(),
                                               sf.data_ptr(), ws.data_ptr(), ws.numel(), st)

            def fixed():
                lib.fvq_nvfp4_quantize(x.data_ptr(), m, k, g.data_ptr(), codes.data_ptr(),
                                       sf.data_ptr(), st)
            one_read = 2 * m * k + m * k // 2 + (m + 127) // 128 * 128 * k // 16
            row = {"m": m, "k": k}
            for name, f, nbytes in (("quantize", fixed, one_read), ("dynamic", dyn, one_read + 2 * m * k)):
                reps = max(5, min(200, int(2e9 // (2 * m * k))))
                for _ in range(3):
                    f()
                torch.cuda.synchronize(dev)
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record(stream)
                for _ in range(reps):
                    f()
                e.record(stream)
                e.synchronize()
                us = s.elapsed_time(e) / reps * 1e3
                gbs = nbytes / (us * 1e-6) / 1e9
                row[name] = {"us": round(us, 2), "GBps": round(gbs, 1),
                             "frac_of_hbm": round(gbs / hbm_peak, 3) if hbm_peak else None}
            out.append(row)
            del x, codes, sf
    torch.cuda.empty_cache()
    return out


def fp4_library_sustained(torch, dev, seconds=2.0, rows=TOKENS) -> dict | None:
    """cuBLASLt NVFP4 (torch._scaled_mm) on the layer's two GEMM shapes at `rows` rows, each
    run back to back for `seconds` so that it sits under the same power cap as the layer: the
    library's sustained TFLOP/s next to which the layer's GEMMs can be read."""
    try:
        out = {}
        for name, (m, n, k) in ((f"gemm1_{rows}x8960x1536", (rows, D_FF, D_MODEL)),
                                (f"gemm2_{rows}x1536x8960", (rows, D_MODEL, D_FF))):
            a = torch.randint(0, 256, (m, k // 2), dtype=torch.uint8, device=dev).view(torch.float4_e2m1fn_x2)
            b = torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, device=dev).view(torch.float4_e2m1fn_x2)
            sa = torch.full((m * k // 16,), 0x38, dtype=torch.uint8, device=dev).view(torch.float8_e4m3fn)
            sb = torch.full((n * k // 16,), 0x38, dtype=torch.uint8, device=dev).view(torch.float8_e4m3fn)
            f = lambda: torch._scaled_mm(a, b.t(), sa, sb, out_dtype=torch.bfloat16)  # noqa: E731
            for _ in range(10):
                f()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            reps = 0
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            while time.perf_counter() - t0 < seconds:
                for _ in range(50):
                    f()
                reps += 50
                torch.cuda.synchronize()
            e.record()
            e.synchronize()
            us = s.elapsed_time(e) / reps * 1e3
            out[name] = {"us": round(us, 2), "tflops": round(2 * m * n * k / (us * 1e-6) / 1e12, 1)}
        return out
    except Exception:
        return None


FP8_ROTATE = 4


def fp8_mode_timing(torch, ops, lib, dev, stream, tokens, fp8_peak, steps=200) -> dict:
    """The reference's other FFN mode, QuantLinear('fp8') (E4M3 W8A8 with per-row scales),
    through fvq_fp8_ffn on the same layer: device-timed tokens/s over `steps` layers
    rotating over FP8_ROTATE distinct (activation, weight) sets (204 MB > L2), the
    four launches' device times, and torch._scaled_mm (the reference's own GEMM call,
    cuBLASLt) on the two GEMM shapes back to back for comparison."""
    from flashvsr_optimizations_b200 import _lib, workloads as W
    g = torch.Generator(device=dev).manual_seed(7)
    sets = []
    for i in range(FP8_ROTATE):
        x = (0.5 * torch.randn(tokens, D_MODEL, device=dev, generator=g)).to(torch.bfloat16)
        w1 = (0.02 * torch.randn(D_FF, D_MODEL, device=dev, generator=g)).to(torch.bfloat16)
        w2 = (0.02 * torch.randn(D_MODEL, D_FF, device=dev, generator=g)).to(torch.bfloat16)
        b1 = (0.01 * torch.randn(D_FF, device=dev, generator=g)).to(torch.bfloat16)
        b2 = (0.01 * torch.randn(D_MODEL, device=dev, generator=g)).to(torch.bfloat16)
        q1, s1 = ops.fp8_row_quant(w1)
        q2, s2 = ops.fp8_row_quant(w2)
        s1, s2 = s1.reshape(-1).contiguous(), s2.reshape(-1).contiguous()
        l1 = _lib.FvqLinearFp8(q1.data_ptr(), s1.data_ptr(), b1.data_ptr(), D_MODEL, D_FF)
        l2 = _lib.FvqLinearFp8(q2.data_ptr(), s2.data_ptr(), b2.data_ptr(), D_FF, D_MODEL)
        sets.append((x, l1, l2, (q1, s1, b1, q2, s2, b2)))
    ws_bytes = lib.fvq_fp8_ffn_workspace_bytes(tokens, D_MODEL, D_FF)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    y = torch.empty(tokens, D_MODEL, dtype=torch.bfloat16, device=dev)
    sptr = stream.cuda_stream

    def step(i):
        x, l1, l2, _ = sets[i % FP8_ROTATE]
        rc = lib.fvq_fp8_ffn(x.data_ptr(), tokens, ctypes.byref(l1), ctypes.byref(l2), y.data_ptr(),
                             ws.data_ptr(), ws_bytes, sptr)
        if rc != 0:
            raise RuntimeError(lib.fvq_last_error().decode())

    for i in range(5):
        step(i)
    torch.cuda.synchronize(dev)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for i in range(steps):
        step(i)
    e.record(stream)
    e.synchronize()
    ms = s.elapsed_time(e) / steps
    kms = (ctypes.c_float * 4)()
    acc = [[] for _ in range(4)]
    for i in range(60):
        x, l1, l2, _ = sets[i % FP8_ROTATE]
        rc = lib.fvq_fp8_ffn_profile(x.data_ptr(), tokens, ctypes.byref(l1), ctypes.byref(l2),
                                     y.data_ptr(), ws.data_ptr(), ws_bytes, sptr, kms)
        if rc != 0:
            raise RuntimeError(lib.fvq_last_error().decode())
        if i >= 10:
            for j in range(4):
                acc[j].append(kms[j])
    med = [statistics.median(a) for a in acc]
    gemm_ms = med[1] + med[3]
    gemm_tflops = tokens * FLOP_PER_TOKEN / (gemm_ms * 1e-3) / 1e12
    out = {"mode": "fp8 (QuantLinear(mode='fp8'): E4M3, per-row scales, fvq_fp8_ffn)",
           "tokens_per_s": tokens / (ms * 1e-3), "ms_per_layer": ms,
           "tflops": tokens * FLOP_PER_TOKEN / (ms * 1e-3) / 1e12,
           "kernels_ms": {"quant_x": med[0], "gemm1_bias_gelu_rowmax": med[1],
                          "quant_h": med[2], "gemm2_bias": med[3]},
           "quant_h_GBps": tokens * D_FF * 3 / (med[2] * 1e-3) / 1e9,
           "roofline": {"bound": "tensor", "kernel": "fp8_gemm_kernel (GEMM1 + GEMM2)",
                        "achieved": gemm_tflops, "peak": fp8_peak, "unit": "TFLOP/s",
                        "frac": gemm_tflops / fp8_peak,
                        "peak_source": "2 x measured cuBLAS bf16 sustained (dense FP8 = 2x bf16)"},
           "l2": f"{FP8_ROTATE} distinct activation/weight sets (204 MB > 126 MB L2)"}
    try:  # torch._scaled_mm with row-wise scales on the same GEMM shapes
        lib_us = {}
        x, _, _, (q1, s1, b1, q2, s2, b2) = sets[0]
        qx, sx = ops.fp8_row_quant(x)
        h = (0.1 * torch.randn(tokens, D_FF, device=dev, generator=g)).to(torch.bfloat16)
        qh, sh = ops.fp8_row_quant(h)
        for name, (a, sa, w, sw) in (("gemm1_7680x8960x1536", (qx, sx, q1, s1)),
                                     ("gemm2_7680x1536x8960", (qh, sh, q2, s2))):
            f = lambda: torch._scaled_mm(a, w.t(), scale_a=sa, scale_b=sw.reshape(1, -1),  # noqa: E731
                                         out_dtype=torch.bfloat16, use_fast_accum=False)
            for _ in range(10):
                f()
            s.record(stream)
            for _ in range(100):
                f()
            e.record(stream)
            e.synchronize()
            lib_us[name] = round(s.elapsed_time(e) / 100 * 1e3, 2)
        out["torch_scaled_mm_us"] = lib_us
    except Exception as exc:  # noqa: BLE001
        out["torch_scaled_mm_us"] = f"unavailable: {type(exc).__name__}"
    return out


def dit_block_timing(torch, lib, dev, stream, sets, tokens, hbm_peak, steps=200) -> dict:
    """The DiT block's FFN step around the layer, x + gate * FFN(LN(x) * (1 + scale) + shift)
    (LN without affine, eps 1e-6): fvq_nvfp4_ffn_block (the LayerNorm + modulation kernel,
    the layer's four launches, the gated residual in GEMM2's epilogue) against the same
    step composed of torch's layer_norm and elementwise ops around fvq_nvfp4_ffn, both
    device-timed over `steps` calls rotating over the benchmark's sets; and the
    LayerNorm + modulation kernel alone (one read of x, one write of u: 4 bytes a value)."""
    from flashvsr_optimizations_b200 import _lib
    import torch.nn.functional as F
    g = torch.Generator(device=dev).manual_seed(13)
    shift, scale, gate = ((s * torch.randn(D_MODEL, device=dev, generator=g)).to(torch.bfloat16)
                          for s in (0.2, 0.2, 0.5))
    eps = 1e-6
    bound = []
    for x, ((q1, s1, g1, b1), (q2, s2, g2, b2)) in sets:
        l1 = _lib.FvqLinear(q1.data_ptr(), s1.data_ptr(), g1.data_ptr(), b1.data_ptr(), D_MODEL, D_FF)
        l2 = _lib.FvqLinear(q2.data_ptr(), s2.data_ptr(), g2.data_ptr(), b2.data_ptr(), D_FF, D_MODEL)
        bound.append((x, l1, l2))
    n = len(bound)
    bws = lib.fvq_nvfp4_ffn_block_workspace_bytes(tokens, D_MODEL, D_FF)
    fws = lib.fvq_nvfp4_ffn_workspace_bytes(tokens, D_MODEL, D_FF)
    ws = torch.zeros(bws, dtype=torch.uint8, device=dev)
    out = torch.empty(tokens, D_MODEL, dtype=torch.bfloat16, device=dev)
    y = torch.empty_like(out)
    u = torch.empty_like(out)
    sptr = stream.cuda_stream
    ptrs = (shift.data_ptr(), scale.data_ptr(), gate.data_ptr())

    def check(rc):
        if rc != 0:
            raise RuntimeError(lib.fvq_last_error().decode())

    def fused(i):
        x, l1, l2 = bound[i % n]
        check(lib.fvq_nvfp4_ffn_block(x.data_ptr(), tokens, *ptrs, ctypes.c_float(eps),
                                      ctypes.byref(l1), ctypes.byref(l2), out.data_ptr(),
                                      ws.data_ptr(), bws, sptr))

    def composed(i):
        x, l1, l2 = bound[i % n]
        v = F.layer_norm(x, (D_MODEL,), eps=eps) * (1 + scale) + shift
        check(lib.fvq_nvfp4_ffn(v.data_ptr(), tokens, ctypes.byref(l1), ctypes.byref(l2),
                                y.data_ptr(), ws.data_ptr(), fws, sptr))
        torch.add(x, gate * y, out=out)

    def ln_only(i):
        x = bound[i % n][0]
        check(lib.fvq_ln_modulate(x.data_ptr(), tokens, D_MODEL, ptrs[0], ptrs[1],
                                  ctypes.c_float(eps), u.data_ptr(), sptr))

    res = {"step": "x + gate * FFN(LN(x) * (1 + scale) + shift), LN without affine, eps 1e-6",
           "tokens": tokens}
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for name, fn, k in (("fused_fvq_nvfp4_ffn_block", fused, steps),
                        ("torch_ln_modulate_gate_around_fvq_nvfp4_ffn", composed, steps),
                        ("ln_modulate_kernel", ln_only, 4 * steps)):
        for i in range(5):
            fn(i)
        torch.cuda.synchronize(dev)
        s.record(stream)
        for i in range(k):
            fn(i)
        e.record(stream)
        e.synchronize()
        ms = s.elapsed_time(e) / k
        res[name] = {"ms": ms, "tokens_per_s": tokens / (ms * 1e-3)}
    gbs = 4 * tokens * D_MODEL / (res["ln_modulate_kernel"]["ms"] * 1e-3) / 1e9
    res["ln_modulate_kernel"].update({"GBps": gbs, "peak_GBps": hbm_peak, "frac": gbs / hbm_peak})
    res["l2"] = f"{n} rotating activation/weight sets"
    return res


def pil_resize_timing(torch, dev, stream, hbm_peak, frames=32, iters=50) -> dict:
    """The input pipeline's Pillow-exact resize (reference pil_exact_gpu.py): 32-frame
    chunks of 426x240 RGB -> 1704x960 bicubic -> crop 1664x896, as bf16 [T,3,896,1664]
    (fused with the normalisation) and as uint8 [T,896,1664,3]; device-timed, against
    Pillow itself on this host (resize + crop, per frame, one thread)."""
    from flashvsr_optimizations_b200 import _lib
    lib = _lib.load()
    g = torch.Generator(device=dev).manual_seed(11)
    src = torch.randint(0, 256, (frames, 240, 426, 3), dtype=torch.uint8, device=dev, generator=g)
    outb = torch.empty((frames, 3, 896, 1664), dtype=torch.bfloat16, device=dev)
    out8 = torch.empty((frames, 896, 1664, 3), dtype=torch.uint8, device=dev)
    sptr = stream.cuda_stream
    res = {"frames_per_call": frames, "geometry": "426x240 -> 1704x960 bicubic, crop (20,32)-(1684,928)"}
    for name, (u8, bf) in (("fused_bf16", (None, outb)), ("u8", (out8, None))):
        def call():
            rc = lib.fvq_pil_resize(src.data_ptr(), frames, 240, 426, 960, 1704, 32, 20, 896, 1664,
                                    None if u8 is None else u8.data_ptr(),
                                    None if bf is None else bf.data_ptr(), sptr)
            if rc != 0:
                raise RuntimeError(lib.fvq_last_error().decode())
        for _ in range(5):
            call()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        for _ in range(iters):
            call()
        e.record(stream)
        e.synchronize()
        ms = s.elapsed_time(e) / iters
        out_bytes = frames * 896 * 1664 * 3 * (2 if bf is not None else 1)
        nbytes = out_bytes + src.numel()
        res[name] = {"ms_per_call": ms, "frames_per_s": frames / (ms * 1e-3),
                     "GBps": nbytes / (ms * 1e-3) / 1e9, "frac_of_hbm": nbytes / (ms * 1e-3) / 1e9 / hbm_peak}
    try:
        from PIL import Image
        host = src[:4].cpu().numpy()
        t0 = time.perf_counter()
        for f in host:
            np.asarray(Image.fromarray(f).resize((1704, 960), Image.BICUBIC).crop((20, 32, 1684, 928)))
        dt = (time.perf_counter() - t0) / len(host)
        res["cpu_pillow_frames_per_s"] = 1.0 / dt
    except Exception as exc:  # noqa: BLE001
        res["cpu_pillow_frames_per_s"] = f"unavailable: {type(exc).__name__}"
    return res


def fp4_library_peak(torch, dev) -> float | None:
    """Dense NVFP4 throughput of cuBLASLt (torch._scaled_mm) at 8192^3, TFLOP/s, or None."""
    try:
        n = 8192
        a = torch.randint(0, 256, (n, n // 2), dtype=torch.uint8, device=dev).view(torch.float4_e2m1fn_x2)
        b = torch.randint(0, 256, (n, n // 2), dtype=torch.uint8, device=dev).view(torch.float4_e2m1fn_x2)
        sa = torch.full((n * n // 16,), 0x38, dtype=torch.uint8, device=dev).view(torch.float8_e4m3fn)
        sb = torch.full((n * n // 16,), 0x38, dtype=torch.uint8, device=dev).view(torch.float8_e4m3fn)
        f = lambda: torch._scaled_mm(a, b.t(), sa, sb, out_dtype=torch.bfloat16)  # noqa: E731
        for _ in range(3):
            f()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(20):
            f()
        e.record()
        e.synchronize()
        return 2 * n ** 3 * 20 / (s.elapsed_time(e) * 1e-3) / 1e12
    except Exception:
        return None


# ---------------------------------------------------------------- the reference's sm_100 kernels
def _event_ms(torch, stream, fn, reps: int, warmup: int = 3) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for _ in range(reps):
        fn()
    e.record(stream)
    e.synchronize()
    return s.elapsed_time(e) / reps


def flashinfer_comparison(torch, ops, lib, dev, stream, weights, run) -> dict:
    """The reference's own path on this GPU and shapes: FlashInfer's sm_100a
    nvfp4_quantize, its CUTLASS mm_fp4 (ffn_quantization.py:64-67) and the reference's
    QuantLinear modules (its global_scale Triton kernel, FlashInfer, torch bias and GELU),
    from the reference module installed unmodified in baseline/_ref and FlashInfer's JIT
    modules prebuilt in baseline/fi_jit, against this library on the same inputs.
    speedup = reference time / this library's time."""
    ref_dir, jit_dir = ROOT / "baseline" / "_ref", ROOT / "baseline" / "fi_jit"
    if not (ref_dir / "ffn_quantization.py").exists():
        return {"unavailable": "the reference module is not installed in baseline/_ref "
                               "(__graft_entry__.build() installs it where the reference tree exists)"}
    os.environ.setdefault("FLASHINFER_WORKSPACE_BASE", str(jit_dir))
    os.environ.setdefault("FLASHINFER_CUDA_ARCH_LIST", "10.0a")
    try:
        import flashinfer
        if str(ref_dir) not in sys.path:
            sys.path.insert(0, str(ref_dir))
        import ffn_quantization as ref
    except Exception as exc:  # noqa: BLE001
        return {"unavailable": f"FlashInfer or the reference module did not load: {type(exc).__name__}: {exc}"}
    from flashvsr_optimizations_b200 import workloads as W
    st = stream.cuda_stream
    res = {"flashinfer": flashinfer.__version__}
    try:
        with torch.no_grad():
            # --- the activation quantizer on the sweep's shapes (N(0,1), 0.1% x50, seed 2)
            quant = {}
            for k in W.QUANT_SWEEP_K:
                for m in W.QUANT_SWEEP_M:
                    gen = torch.Generator(device=dev)
                    gen.manual_seed(2)
                    x = torch.randn(m, k, device=dev, generator=gen)
                    idx = torch.randint(0, m * k, (max(1, m * k // 1000),), device=dev, generator=gen)
                    x.view(-1)[idx] *= 50.0
                    x = x.to(torch.bfloat16)
                    del idx
                    g = ref.global_scale(x)
                    codes = torch.empty(m, k // 2, dtype=torch.uint8, device=dev)
                    sf = torch.empty((m + 127) // 128 * 128, k // 16, dtype=torch.uint8, device=dev)
                    ws = torch.zeros(lib.fvq_amax_workspace_bytes(), dtype=torch.uint8, device=dev)
                    gout = torch.empty(1, dtype=torch.float32, device=dev)
                    reps = max(5, min(200, int(2e9 // (2 * m * k))))
                    t_ref = _event_ms(torch, stream, lambda: flashinfer.nvfp4_quantize(x, g), reps)
                    t_our = _event_ms(torch, stream, lambda: lib.fvq_nvfp4_quantize(
                        x.data_ptr(), m, k, g.data_ptr(), codes.data_ptr(), sf.data_ptr(), st), reps)
                    t_ref_d = _event_ms(torch, stream,
                                        lambda: flashinfer.nvfp4_quantize(x, ref.global_scale(x)), reps)
                    t_our_d = _event_ms(torch, stream, lambda: lib.fvq_nvfp4_quantize_dynamic(
                        x.data_ptr(), m, k, None, gout.data_ptr(), codes.data_ptr(), sf.data_ptr(),
                        ws.data_ptr(), ws.numel(), st), reps)
                    q_ref, s_ref = flashinfer.nvfp4_quantize(x, g)
                    lib.fvq_nvfp4_quantize(x.data_ptr(), m, k, g.data_ptr(), codes.data_ptr(),
                                           sf.data_ptr(), st)
                    same = bool(torch.equal(q_ref.view(torch.uint8), codes) and
                                torch.equal(s_ref.view(torch.uint8).reshape(-1), sf.reshape(-1)))
                    quant[f"{m}x{k}"] = {"ref_us": round(t_ref * 1e3, 2), "ours_us": round(t_our * 1e3, 2),
                                         "speedup": t_ref / t_our,
                                         "with_global_scale_ref_us": round(t_ref_d * 1e3, 2),
                                         "with_global_scale_ours_us": round(t_our_d * 1e3, 2),
                                         "with_global_scale_speedup": t_ref_d / t_our_d,
                                         "same_bits": same}
                    del x, codes, sf, q_ref, s_ref
            res["quantize"] = quant
            torch.cuda.empty_cache()

            # --- the reference's modules on the stack's weights
            def ref_linear(w, b):
                lin = torch.nn.Linear(w.shape[1], w.shape[0], bias=True, device=dev, dtype=torch.bfloat16)
                lin.weight.copy_(w)
                lin.bias.copy_(b)
                return ref.QuantLinear(lin, "nvfp4")

            ref_layers = []
            for i in range(0, len(weights.bf16), 2):
                (w1, b1), (w2, b2) = weights.bf16[i], weights.bf16[i + 1]
                ref_layers.append(torch.nn.Sequential(ref_linear(w1, b1), torch.nn.GELU(approximate="tanh"),
                                                      ref_linear(w2, b2)))
            rows = run.rows
            x = run.x
            # --- the two GEMM shapes of a layer at this batch (mm_fp4 with the bias add as the
            # reference runs it; this library's GEMM1 also applies GELU and takes the amax)
            l1, l2 = ref_layers[0][0], ref_layers[0][2]
            g_x = ref.global_scale(x)
            qx, sx = flashinfer.nvfp4_quantize(x, g_x)
            (mq1, ms1, mg1, mb1), (mq2, ms2, mg2, mb2) = weights.tensors[0], weights.tensors[1]
            h = torch.nn.functional.gelu(l1(x), approximate="tanh")
            g_h = ref.global_scale(h)
            qh, sh = flashinfer.nvfp4_quantize(h, g_h)
            gemms = {}
            for name, (qa, sa, ga, lin, mq, ms, mg, mb, n, k, epi) in (
                    (f"gemm1_{rows}x{D_FF}x{D_MODEL}", (qx, sx, g_x, l1, mq1, ms1, mg1, mb1, D_FF, D_MODEL, 1)),
                    (f"gemm2_{rows}x{D_MODEL}x{D_FF}", (qh, sh, g_h, l2, mq2, ms2, mg2, mb2, D_MODEL, D_FF, 0))):
                alpha = 1. / (ga * lin.global_sf)
                out = torch.empty(rows, n, dtype=torch.bfloat16, device=dev)
                amax = torch.zeros(1, dtype=torch.float32, device=dev)
                t_ref = _event_ms(torch, stream, lambda: flashinfer.mm_fp4(
                    qa, lin.qweight.t(), sa, lin.scale.t(), alpha=alpha, out_dtype=torch.bfloat16,
                    backend="cutlass") + lin.bias, 20)
                t_our = _event_ms(torch, stream, lambda: lib.fvq_nvfp4_gemm(
                    qa.view(torch.uint8).data_ptr(), sa.view(torch.uint8).data_ptr(), ga.data_ptr(),
                    mq.data_ptr(), ms.data_ptr(), mg.data_ptr(), mb.data_ptr(), out.data_ptr(),
                    rows, n, k, epi, amax.data_ptr() if epi == 1 else None, st), 20)
                flop = 2 * rows * n * k
                gemms[name] = {"ref_mm_fp4_plus_bias_us": round(t_ref * 1e3, 2),
                               "ours_us": round(t_our * 1e3, 2), "speedup": t_ref / t_our,
                               "ours_tflops": flop / (t_our * 1e-3) / 1e12,
                               "ours_epilogue": "bias + GELU + amax" if epi == 1 else "bias"}
            res["gemm"] = gemms
            del h, qh, sh
            torch.cuda.empty_cache()
            # --- one layer and the whole stack, reference modules against fvq_nvfp4_ffn
            l0 = run.structs[0]
            y0 = run.bufs[0]
            def ours_layer():
                rc = lib.fvq_nvfp4_ffn(x.data_ptr(), rows, ctypes.byref(l0[0]), ctypes.byref(l0[1]),
                                       y0.data_ptr(), run.ws.data_ptr(), run.ws_bytes, st)
                if rc != 0:
                    raise RuntimeError(lib.fvq_last_error().decode())

            t_ref = _event_ms(torch, stream, lambda: ref_layers[0](x), 10)
            t_our = _event_ms(torch, stream, ours_layer, 10)
            y_ref0 = ref_layers[0](x)
            ours_layer()
            same_layer = bool(torch.equal(y_ref0, y0))
            del y_ref0
            res["layer"] = {"rows": rows, "ref_ms": t_ref, "ours_ms": t_our, "speedup": t_ref / t_our,
                            "same_bits": same_layer}

            def ref_stack():
                y = x
                for m in ref_layers:
                    y = m(y)
                return y

            t_ref = _event_ms(torch, stream, ref_stack, 3, warmup=1)
            t_our = _event_ms(torch, stream, run.layers, 3, warmup=1)
            same_stack = bool(torch.equal(ref_stack(), run.layers()))
            res["stack30"] = {"rows": rows, "ref_ms": t_ref, "ours_ms": t_our, "speedup": t_ref / t_our,
                              "ref_tokens_per_s": rows / (t_ref * 1e-3), "same_bits": same_stack}
    except Exception as exc:  # noqa: BLE001
        res["error"] = f"{type(exc).__name__}: {exc}"
    return res


def layer_case(torch, ops, lib, dev, stream, tokens, steps, fused=False) -> dict:
    """One FFN call (layer 0 of the stack) over the first `tokens` rows of the stack input,
    `steps` times: the launch sequence a profiler capture looks at.  fused: the call is
    fvq_nvfp4_ffn_fused (GEMM1 quantizes h; estimate of max |h| 4.0, one bit of headroom)
    instead of fvq_nvfp4_ffn."""
    weights = StackWeights(torch, ops, dev, layers=1)
    wl = STACK_WORKLOADS["c4" if tokens <= STACK_WORKLOADS["c4"]["total"] else "c5"]
    run = StackRun(torch, lib, dev, stream, weights, dict(wl, total=tokens), 1, 0)
    if not fused:
        for _ in range(steps):
            run.layers()
    else:
        l1, l2 = run.structs[0]
        hint = torch.full((1,), 4.0, dtype=torch.float32, device=dev)
        seen = torch.zeros(1, dtype=torch.float32, device=dev)
        flags = torch.zeros(1, dtype=torch.int32, device=dev)
        nbytes = lib.fvq_nvfp4_ffn_fused_workspace_bytes(tokens, D_MODEL, D_FF)
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        for _ in range(steps):
            rc = lib.fvq_nvfp4_ffn_fused(run.x.data_ptr(), tokens, ctypes.byref(l1), ctypes.byref(l2),
                                         run.bufs[0].data_ptr(), hint.data_ptr(), 1, seen.data_ptr(),
                                         flags.data_ptr(), ws.data_ptr(), nbytes, run.sptr)
            if rc != 0:
                raise RuntimeError(lib.fvq_last_error().decode())
    torch.cuda.synchronize(dev)
    return {"tokens": tokens, "calls": steps, "fused": fused}


def shard_case(torch, dist, ops, lib, dev, stream, wl, shard_of, steps, warmup) -> dict:
    """The 30-layer stack on rank 0's row block of a `shard_of`-way split, on this GPU alone
    and without the all-gather: the per-rank compute of the N-GPU benchmark, measured on one
    GPU (device time of `steps` stacks, and the per-launch times of one more pass)."""
    from flashvsr_optimizations_b200.sharding import row_range
    weights = StackWeights(torch, ops, dev)
    run = StackRun(torch, lib, dev, stream, weights, wl, 1, 0)
    r0, r1 = row_range(wl["total"], shard_of, 0)
    run.rows = r1 - r0
    run.x = run.x[:run.rows].contiguous()
    run.bufs = [b[:run.rows] for b in run.bufs]
    run.capture(torch)   # as the N-GPU benchmark's ranks run it: one CUDA graph replay per stack
    ms = timed_steps(torch, dist, dev, stream, 1, lambda i: run.step(), steps, warmup) / steps
    # host time to issue one stack's 120 launches (the device is idle when each issue starts)
    host = []
    for _ in range(5):
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        run.layers()
        host.append((time.perf_counter() - t0) * 1e3)
    torch.cuda.synchronize(dev)
    kt = stack_kernel_timing(torch, dist, dev, 1, run, passes=2)
    return {"workload": wl["name"], "shard_of": shard_of, "rows": run.rows, "ms_per_stack": ms,
            "host_issue_ms_per_stack": statistics.median(host),
            "tokens_per_s": run.rows / (ms * 1e-3),
            "tflops": run.rows * LAYERS * FLOP_PER_TOKEN / (ms * 1e-3) / 1e12, "kernels_ms": kt}


def sustained_case(torch, ops, lib, dev, stream, rows, seconds=2.0) -> dict:
    """Each of the layer's launches, and the whole stack step, run back to back for
    `seconds` after 1.5 s at load (so the power cap has settled), with NVML sampling the SM
    clock and power draw: the sustained time per launch, its median clock and power, and
    the energy per launch.  cuBLASLt NVFP4 (torch._scaled_mm, no epilogue) runs on the same
    codes and scales for comparison.  Under the cap, time per launch follows energy."""
    from flashvsr_optimizations_b200 import workloads as W
    d, f, m = D_MODEL, D_FF, rows
    x = to_dev(torch, stack_input_rows(STACK_WORKLOADS["c4"], 0, m), dev) if m <= 15360 else \
        torch.randn(m, d, device=dev, generator=torch.Generator(device=dev).manual_seed(0)).to(torch.bfloat16)
    w1, b1, w2, b2 = (to_dev(torch, a, dev) for a in W.stack_layer_params(0))
    gx, g1, g2 = ops.global_scale(x), ops.global_scale(w1), ops.global_scale(w2)
    qx, sx = ops.nvfp4_quantize(x, gx)
    q1, s1 = ops.nvfp4_quantize(w1, g1)
    q2, s2 = ops.nvfp4_quantize(w2, g2)
    h = torch.empty(m, f, dtype=torch.bfloat16, device=dev)
    amax = torch.zeros(1, dtype=torch.float32, device=dev)
    sp = stream.cuda_stream

    def gemm1():
        lib.fvq_nvfp4_gemm(qx.data_ptr(), sx.data_ptr(), gx.data_ptr(), q1.data_ptr(), s1.data_ptr(),
                           g1.data_ptr(), b1.data_ptr(), h.data_ptr(), m, f, d, 1, amax.data_ptr(), sp)
    gemm1()
    torch.cuda.synchronize(dev)
    gh = ops.global_scale(h)
    qh, sh = ops.nvfp4_quantize(h, gh)
    y = torch.empty(m, d, dtype=torch.bfloat16, device=dev)

    def gemm2():
        lib.fvq_nvfp4_gemm(qh.data_ptr(), sh.data_ptr(), gh.data_ptr(), q2.data_ptr(), s2.data_ptr(),
                           g2.data_ptr(), b2.data_ptr(), y.data_ptr(), m, d, f, 0, None, sp)

    def quant_h():
        ops.nvfp4_quantize(h, gh)

    def lt(a, sa, b, sb):
        av, bv = a.view(torch.float4_e2m1fn_x2), b.view(torch.float4_e2m1fn_x2)
        sav, sbv = sa.view(torch.float8_e4m3fn).reshape(-1), sb.view(torch.float8_e4m3fn).reshape(-1)
        return lambda: torch._scaled_mm(av, bv.t(), sav, sbv, out_dtype=torch.bfloat16)
    cases = {"gemm1_bias_gelu_amax": gemm1, "quantize_h": quant_h, "gemm2_bias": gemm2}
    try:
        cases["cublaslt_gemm1_no_epilogue"] = lt(qx, sx, q1, s1)
        cases["cublaslt_gemm2_no_epilogue"] = lt(qh, sh, q2, s2)
    except (AttributeError, RuntimeError):
        pass
    weights = StackWeights(torch, ops, dev)
    run = StackRun(torch, lib, dev, stream, weights, STACK_WORKLOADS["c4"], 1, 0)
    run.rows = m
    run.x = run.x[:m].contiguous()
    run.bufs = [b[:m] for b in run.bufs]
    cases["stack_step_30_layers"] = run.layers
    gpu_uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    out = {}
    for name, fn in cases.items():
        reps_per_check = 2 if name.startswith("stack") else 20
        try:
            for _ in range(reps_per_check):
                fn()
            torch.cuda.synchronize(dev)
        except RuntimeError as e:   # e.g. a torch without NVFP4 _scaled_mm
            out[name] = {"unavailable": str(e).splitlines()[0][:120]}
            continue
        t0 = time.perf_counter()
        while time.perf_counter() - t0 < 1.5:
            for _ in range(reps_per_check):
                fn()
            torch.cuda.synchronize(dev)
        sampler = clock_sampler(gpu_uuid)
        sampler.start()
        s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 0
        t1 = time.perf_counter()
        s_ev.record(stream)
        while time.perf_counter() - t1 < seconds:
            for _ in range(reps_per_check):
                fn()
            reps += reps_per_check
            torch.cuda.synchronize(dev)
        e_ev.record(stream)
        e_ev.synchronize()
        clk = sampler.stop()
        samples = getattr(sampler, "samples", [])
        power = statistics.median(pw for _, pw, _ in samples) if samples else None
        us = s_ev.elapsed_time(e_ev) / reps * 1e3
        out[name] = {"us_per_launch": round(us, 2), "launches": reps, "sm_mhz_median": clk.get("sm_mhz"),
                     "power_w_median": power, "reasons": clk.get("reasons"),
                     "energy_mj_per_launch": round(us * 1e-3 * power, 2) if power else None}
        time.sleep(1.0)
    return {"rows": m, "seconds_timed": seconds, "note": "1.5 s at load before each timed loop; "
            "stack_step_30_layers is one fvq_nvfp4_ffn_chain pass over the 30 layers", "cases": out}


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except ValueError:
            pass
    return {}


def main():
    args = parse()
    rank, local_rank, world = env_rank()
    if args.impl == "reference":
        return run_reference(args, rank, world)
    import torch
    import torch.distributed as dist
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
    from flashvsr_optimizations_b200 import _lib, ops
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev)
    peaks = measured_peaks()
    hbm = peaks.get("hbm_gbs") or 6650.0
    if args.case != "stack":
        if args.case == "shard":
            out = shard_case(torch, dist, ops, lib, dev, stream, STACK_WORKLOADS[args.workload],
                             args.shard_of, args.steps, args.warmup)
        elif args.case in ("layer", "layer_fused"):
            out = layer_case(torch, ops, lib, dev, stream, args.tokens, args.steps,
                             fused=args.case == "layer_fused")
        elif args.case == "fp8_ffn":
            peak8 = 2.0 * (peaks.get("bf16_tflops_sustained") or 1400.0)
            out = fp8_mode_timing(torch, ops, lib, dev, stream, args.tokens, peak8, steps=args.steps)
        elif args.case == "sustained":
            out = sustained_case(torch, ops, lib, dev, stream, args.tokens)
        elif args.case == "dit_block":
            out = dit_block_timing(torch, lib, dev, stream, make_sets(torch, ops, dev, args.tokens, rank)[:4],
                                   args.tokens, hbm, steps=args.steps)
        else:
            out = pil_resize_timing(torch, dev, stream, hbm, iters=args.steps)
        if rank == 0:
            print(json.dumps({"case": args.case, **out}), flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return

    wl = STACK_WORKLOADS[args.workload]
    extras_here = not args.no_extras
    weights = StackWeights(torch, ops, dev, keep_bf16=extras_here and world == 1)
    run = StackRun(torch, lib, dev, stream, weights, wl, world, rank)

    # ---- the timed steps: 30 layers on this rank's rows (one CUDA graph replay) + the all-gather
    run.capture(torch)
    gpu_uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    sampler = clock_sampler(gpu_uuid)
    ms = timed_steps(torch, dist, dev, stream, world, lambda i: run.step(), args.steps, args.warmup,
                     sampler=sampler)
    clocks = sampler.stop()
    total = wl["total"]
    value = total * args.steps / (ms * 1e-3)
    flop_per_step = total * LAYERS * FLOP_PER_TOKEN
    tflops = flop_per_step * args.steps / (ms * 1e-3) / 1e12

    # ---- per-launch device times (a second pass over the same steps' layers)
    kt = stack_kernel_timing(torch, dist, dev, world, run, passes=max(1, min(args.steps, 5)))
    burst = peaks.get("bf16_tflops")
    sustained = peaks.get("bf16_tflops_sustained")
    if burst:
        peak, peak_src = 4.0 * burst, ("4 x measured cuBLAS bf16 burst (MEASURED_PEAKS.json); dense "
                                       "FP4 runs at 4x bf16 on B200; the GEMMs are timed per launch")
    else:
        peak, peak_src = 4.0 * 1590.0, "4 x fallback bf16 burst 1.59 PFLOP/s"
    peak_sus = 4.0 * (sustained or 1400.0)
    gemm_flop = run.rows * FLOP_PER_TOKEN
    achieved = gemm_flop / (kt["gemm_ms"] * 1e-3) / 1e12
    traffic = None
    tp = ROOT / "profiles" / f"nvfp4_gemm_pair_{run.rows}tok_traffic.json"
    if tp.exists():
        try:
            traffic = json.loads(tp.read_text()).get("dram_bytes_per_gemm_pair")
        except ValueError:
            traffic = None

    # ---- the vendor library (cuBLASLt NVFP4, no epilogue) on this rank's two GEMM shapes
    lib_shapes = fp4_library_sustained(torch, dev, seconds=1.0, rows=run.rows)

    # ---- end to end through the public module API with host buffers
    e2e = stack_e2e(torch, dist, weights, run, dev, world, rank, args.steps, args.warmup)

    result = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": "nvfp4 (e2m1 codes, e4m3 1x16 scales, fp32 global scales), fp32 accumulate, bf16 io",
        "data": f"synthetic: {wl['input']}; layer weights N(0,0.02), biases N(0,0.01), seeded",
        "config": {"workload": wl["name"], "tokens": total, "layers": LAYERS, "d_model": D_MODEL,
                   "d_ff": D_FF, "rows_per_gpu": run.rows,
                   "parallelism": f"token-row shards x{world}, replicated weights, NCCL all-gather "
                                  f"of the output inside the step",
                   "l2": "inputs larger than L2: 464 MB of weights per step, each layer's "
                         f"{run.rows * D_FF * 2 / 1e6:.0f} MB intermediate"},
        "tflops": tflops, "tflops_frac_of_fp4_peak": tflops / (peak * world),
        "gpu_launches": LAUNCHES_PER_LAYER * LAYERS * args.steps,
        "roofline": {"bound": "tensor",
                     "kernel": "the layer's two NVFP4 GEMM launches (tcgen05 mxf4nvf4)",
                     "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                     "traffic": traffic, "peak_source": peak_src,
                     "frac_of_sustained": achieved / peak_sus,
                     "algorithmic_flop_per_launch_pair": gemm_flop,
                     **({"cublaslt_same_shapes_us": {k: v["us"] for k, v in lib_shapes.items()},
                         "frac_of_cublaslt_same_shapes":
                             (sum(v["us"] for v in lib_shapes.values()) * 1e-3) / kt["gemm_ms"]}
                        if lib_shapes else {})},
        "quantize": {"kernel": f"quantize_kernel on the {run.rows}x{D_FF} intermediate",
                     "GBps": kt["quant_h_GBps"], "peak_GBps": hbm, "frac": kt["quant_h_GBps"] / hbm,
                     "ms": kt["quant_h_ms"]},
        "kernels_ms": kt,
        "e2e": e2e,
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_stack_tokens_per_s(3, 1, args.cpu_seconds, wl)

    tail = {}
    if extras_here:
        result["single_layer"] = single_layer_timing(torch, dist, ops, lib, dev, stream, world, rank,
                                                     args.tokens, 200)
        if args.workload == "c4":
            wl5 = STACK_WORKLOADS["c5"]
            run5 = StackRun(torch, lib, dev, stream, weights, wl5, world, rank)
            ms5 = timed_steps(torch, dist, dev, stream, world, lambda i: run5.step(), 3, 1)
            v5 = wl5["total"] * 3 / (ms5 * 1e-3)
            tail["c5_stack"] = {"workload": wl5["name"], "tokens": wl5["total"], "rows_per_gpu": run5.rows,
                                "ms_per_stack": ms5 / 3, "tokens_per_s": v5,
                                "tflops": v5 * LAYERS * FLOP_PER_TOKEN / 1e12,
                                "tflops_frac_of_fp4_peak": v5 * LAYERS * FLOP_PER_TOKEN / 1e12 / (peak * world)}
            del run5
            torch.cuda.empty_cache()
        fr = fused_requant_timing(torch, dist, dev, stream, world, weights, run, wl, rank)
        fr["speedup_vs_exact"] = (ms / args.steps) / fr["ms_per_stack"]
        tail["fused_requant"] = fr
        if world > 1 and args.workload == "c4":
            tail["stack_check"] = stack_check(torch, dist, dev, weights, run, wl, world, rank)
        if world == 1:
            result["quantize_sweep"] = quantize_sweep(torch, lib, dev, stream, hbm)
            fp8_peak = 2.0 * (sustained or 1400.0)
            result["fp8_mode"] = fp8_mode_timing(torch, ops, lib, dev, stream, args.tokens, fp8_peak)
            result["pil_resize"] = pil_resize_timing(torch, dev, stream, hbm)
            result["dit_block"] = dit_block_timing(torch, lib, dev, stream,
                                                   make_sets(torch, ops, dev, args.tokens, rank)[:4],
                                                   args.tokens, hbm)
            lib_sus = fp4_library_sustained(torch, dev)
            if lib_sus:
                result["fp4_cublas_sustained_layer_shapes"] = lib_sus
            fp4_cublas = fp4_library_peak(torch, dev)
            if fp4_cublas:
                result["fp4_cublas_8192_tflops"] = fp4_cublas
            tail["flashinfer"] = flashinfer_comparison(torch, ops, lib, dev, stream, weights, run)
    if world > 1:
        tail["gather"] = gather_timing(torch, dist, dev, stream, world, run)
    result.update(tail)
    # the figures that matter most for scaling last, where a truncated log keeps them
    result["summary"] = {"n_gpus": world, "ms_per_step": ms / args.steps, "tokens_per_s": value,
                         "e2e_tokens_per_s": e2e["value"], "gemm_frac_of_burst": achieved / peak,
                         **({"gather_ms": tail["gather"]["ms"],
                             "gather_busbw_GBps": tail["gather"]["busbw_GBps"]} if "gather" in tail else {})}
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_reference(args, rank, world):
    """The reference arm: the reference's NVFP4 FFN arithmetic restated on the host CPU (the
    reference's own path runs only on a GPU), rank 0 only, on bounded samples."""
    if rank != 0:
        return
    wl = STACK_WORKLOADS[args.workload]
    res = cpu_stack_tokens_per_s(args.steps, args.warmup, seconds=60.0, wl=wl)
    ms_per_step = res["seconds"] / args.steps * LAYERS * 1e3
    line = {"metric": METRIC, "value": res["value"], "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "nvfp4 emulated (fp32 dequantized matmul)", "data": "synthetic (seeded)",
            "config": {"workload": wl["name"], "tokens_per_step": res["rows_per_step"],
                       "layers": LAYERS, "d_model": D_MODEL, "d_ff": D_FF, "parallelism": "host CPU"},
            "impl": "reference",
            "cpu_baseline": {"value": res["value"], "unit": "tokens/s", "cores": res["cores"],
                             "kind": res["kind"], "sample": res["sample"]},
            "e2e": {"value": res["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
