#!/usr/bin/env python
"""Benchmark of the NVFP4 FFN path on B200: one FFN layer (d_model 1536, d_ff 8960,
GELU-tanh, bias) over 7680 tokens per GPU, one process per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...     (N > 1)

A step is one pass of the FFN layer over a batch of 7680 synthetic tokens
(two 48x80 latent frames, Student-t(4) x 0.5 activations, N(0, 0.02) weights,
N(0, 0.01) biases; seeded).  Token rows are independent, so each rank runs
its own batch with replicated weights and no collective in the step (weak
scaling); the output all-gather the path uses after a stack is timed
separately (`gather`).  Inputs rotate over 8 distinct (activation, weight)
sets, 312 MB in all, so no step finds its operands in the 126 MB L2.

Prints one JSON line (rank 0).  `value` is whole-job tokens/s with inputs
resident in HBM; `e2e` is the same metric through the public module API with
host buffers (pinned H2D of the input and D2H of the output inside the timed
region); `roofline` describes the GEMM kernel; `cpu_baseline` times the
reference arithmetic (the CPU oracle) on this host.  Two separate measurements
follow the timed steps (skip them with --no-extras): `stack_30_layers`, the
30-layer stack of distinct layers over 15360 tokens with rows sharded across the
ranks and the outputs all-gathered, `quantize_sweep` (rank 0), the
activation quantizer on K in {1536, 8960} x M in {1024, 4096, 16384, 65536}, and
`fp8_mode` (rank 0), the same layer in the reference's other mode,
QuantLinear('fp8') (E4M3 W8A8, per-row scales), `pil_resize` (rank 0), the
input pipeline's Pillow-exact 4x bicubic resize of 32-frame chunks, and
`dit_block` (rank 0), the DiT block's step around the layer (LayerNorm +
modulation in, gated residual out) fused against torch's composition.

`--impl reference` times the reference's NVFP4 FFN arithmetic on the host CPU
(the oracle restatement; the reference itself needs FlashInfer on a GPU) with
all host threads, on bounded samples of the same workload.
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
TOKENS = 7680
FLOP_PER_TOKEN = 2 * D_MODEL * D_FF * 2
ROTATE = 8
METRIC = "nvfp4_ffn_tokens_per_s"
WORKLOAD = "ffn_layer_d1536_ff8960_gelu_tanh_bias_7680tok_per_gpu"
# fvq_nvfp4_ffn launches per layer: amax+quantize(x), GEMM1 (+bias, GELU, amax), quantize(h), GEMM2
LAUNCHES_PER_LAYER = 4


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=("native", "reference"), default="native")
    ap.add_argument("--tokens", type=int, default=TOKENS)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the quantize sweep and the 30-layer stack (separate measurements)")
    ap.add_argument("--cpu-seconds", type=float, default=20.0,
                    help="wall-time budget of the CPU baseline sample")
    ap.add_argument("--case", choices=("ffn", "fp8_ffn", "pil_resize", "dit_block"), default="ffn",
                    help="ffn: the benchmark (default); fp8_ffn / pil_resize / dit_block: only that "
                         "separate measurement, --steps calls, one JSON line (e.g. under a profiler)")
    return ap.parse_args()


def env_rank():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0")),
            int(os.environ.get("WORLD_SIZE", "1")))


# ---------------------------------------------------------------- clocks
class NvmlClockSampler:
    """SM clock, power and clock-event reasons read through NVML every 5 ms from a
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
            self._stop.wait(0.005)

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


# ---------------------------------------------------------------- CPU legs
def cpu_ffn_tokens_per_s(steps: int, warmup: int, seconds: float, log=print) -> dict:
    """Reference NVFP4 FFN arithmetic (the oracle, fp32 matmul) on host threads."""
    from oracle import nvfp4_oracle as O
    from flashvsr_optimizations_b200 import workloads as W
    threads = os.cpu_count() or 1
    w1, b1 = W.linear_params(D_FF, D_MODEL, seed=20, b_std=0.01)
    w2, b2 = W.linear_params(D_MODEL, D_FF, seed=21, b_std=0.01)
    l1, l2 = O.OracleQuantLinear(w1, b1), O.OracleQuantLinear(w2, b2)
    # calibrate the per-step sample so the whole run fits the time budget
    probe = W.student_t(64, D_MODEL, seed=1)
    t0 = time.perf_counter()
    O.ffn_forward(probe, l1, l2, fp32_matmul=True)
    t0 = time.perf_counter()
    O.ffn_forward(probe, l1, l2, fp32_matmul=True)
    per_tok = (time.perf_counter() - t0) / 64
    rows = int(seconds / max(1, steps + warmup) / max(per_tok, 1e-6))
    rows = max(16, min(1024, rows // 16 * 16))
    x_all = W.student_t(TOKENS, D_MODEL, seed=1)
    for i in range(warmup):
        O.ffn_forward(x_all[(i * rows) % (TOKENS - rows):][:rows], l1, l2, fp32_matmul=True)
    times = []
    for i in range(steps):
        xs = x_all[(i * rows) % (TOKENS - rows):][:rows]
        t = time.perf_counter()
        O.ffn_forward(xs, l1, l2, fp32_matmul=True)
        times.append(time.perf_counter() - t)
    total = sum(times)
    return {"value": rows * steps / total, "unit": "tokens/s", "cores": threads,
            "kind": "port", "rows_per_step": rows, "seconds": total,
            "sample": (f"{steps} steps of {rows} tokens from the 7680-token layer workload; numpy oracle "
                       f"(quantize, dequantize, fp32 BLAS matmul, bias, GELU-tanh, requantize); "
                       f"weights quantized once outside the timing; {threads} host threads")}


# ---------------------------------------------------------------- GPU setup
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


def stack_timing(torch, dist, ops, lib, dev, stream, world, rank, steps=10) -> dict:
    """The 30-layer FFN stack: M = 15360 N(0,1) tokens (seed 3), 30 layers with distinct
    N(0,0.02) weights (and N(0,0.01) biases), token rows sharded over the ranks, outputs
    all-gathered.  Time = max over ranks of (30 layers + gather)."""
    from flashvsr_optimizations_b200.sharding import gather_rows, row_range
    total, layers = 15360, 30
    r0, r1 = row_range(total, world, rank)
    rows = r1 - r0
    gen = torch.Generator(device=dev)
    gen.manual_seed(3)
    x_all = torch.randn(total, D_MODEL, device=dev, generator=gen).to(torch.bfloat16)
    x = x_all[r0:r1].contiguous()
    del x_all
    structs, keep = [], []
    for layer in range(layers):
        gl = torch.Generator(device=dev)
        gl.manual_seed(100 + layer)
        pair = []
        for (n, k) in ((D_FF, D_MODEL), (D_MODEL, D_FF)):
            w = (torch.randn(n, k, device=dev, generator=gl) * 0.02).to(torch.bfloat16)
            b = (torch.randn(n, device=dev, generator=gl) * 0.01).to(torch.bfloat16)
            gsc = ops.global_scale(w)
            q, sc = ops.nvfp4_quantize(w, gsc)
            keep.append((q, sc, gsc, b))
            pair.append(_lib_linear(q, sc, gsc, b, k, n))
        structs.append(pair)
    ws_bytes = lib.fvq_nvfp4_ffn_workspace_bytes(rows, D_MODEL, D_FF)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
    bufs = [torch.empty(rows, D_MODEL, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    st = stream.cuda_stream

    def run_stack():
        cur = x
        for i, (l1, l2) in enumerate(structs):
            out = bufs[i % 2]
            rc = lib.fvq_nvfp4_ffn(cur.data_ptr(), rows, ctypes.byref(l1), ctypes.byref(l2),
                                   out.data_ptr(), ws.data_ptr(), ws_bytes, st)
            if rc != 0:
                raise RuntimeError(lib.fvq_last_error().decode())
            cur = out
        return gather_rows(cur, total) if world > 1 else cur

    for _ in range(2):
        run_stack()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for _ in range(steps):
        y = run_stack()
    e.record(stream)
    torch.cuda.synchronize(dev)
    ms = s.elapsed_time(e) / steps
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    tflops = total * layers * FLOP_PER_TOKEN / (ms * 1e-3) / 1e12
    finite = bool(torch.isfinite(y.float()).all().item())
    return {"tokens": total, "layers": layers, "ms_per_stack": ms,
            "tokens_per_s": total / (ms * 1e-3), "tflops": tflops, "finite_output": finite,
            "rows_per_rank": rows, "includes": "30 fvq_nvfp4_ffn calls per rank + all-gather of the outputs"}


def _lib_linear(q, s, g, b, in_f, out_f):
    from flashvsr_optimizations_b200 import _lib
    return _lib.FvqLinear(q.data_ptr(), s.data_ptr(), g.data_ptr(), b.data_ptr(), in_f, out_f)


def fp4_library_sustained(torch, dev, seconds=2.0) -> dict | None:
    """cuBLASLt NVFP4 (torch._scaled_mm) on the layer's two GEMM shapes, each run back to
    back for `seconds` so that it sits under the same power cap as the layer: the library's
    sustained TFLOP/s next to which the layer's GEMMs can be read."""
    try:
        out = {}
        for name, (m, n, k) in (("gemm1_7680x8960x1536", (TOKENS, D_FF, D_MODEL)),
                                ("gemm2_7680x1536x8960", (TOKENS, D_MODEL, D_FF))):
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
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    import flashvsr_optimizations_b200 as fvq
    from flashvsr_optimizations_b200 import _lib, ops
    from flashvsr_optimizations_b200.ffn_quantization import NVFP4FFN
    lib = _lib.load()
    tokens = args.tokens
    if args.case != "ffn":
        stream = torch.cuda.current_stream(dev)
        hbm = measured_peaks().get("hbm_gbs") or 6650.0
        if args.case == "fp8_ffn":
            peak8 = 2.0 * (measured_peaks().get("bf16_tflops_sustained") or 1400.0)
            out = fp8_mode_timing(torch, ops, lib, dev, stream, tokens, peak8, steps=args.steps)
        elif args.case == "dit_block":
            out = dit_block_timing(torch, lib, dev, stream, make_sets(torch, ops, dev, tokens, rank)[:4],
                                   tokens, hbm, steps=args.steps)
        else:
            out = pil_resize_timing(torch, dev, stream, hbm, iters=args.steps)
        if rank == 0:
            print(json.dumps({"case": args.case, **out}), flush=True)
        return
    sets = make_sets(torch, ops, dev, tokens, rank)
    ws_bytes = lib.fvq_nvfp4_ffn_workspace_bytes(tokens, D_MODEL, D_FF)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
    ys = [torch.empty(tokens, D_MODEL, dtype=torch.bfloat16, device=dev) for _ in range(ROTATE)]
    stream = torch.cuda.current_stream(dev)
    sptr = stream.cuda_stream
    # pre-bound C-ABI calls (fvq_nvfp4_ffn), one per rotating set
    structs = []
    for x, ((q1, s1, g1, b1), (q2, s2, g2, b2)) in sets:
        l1 = _lib.FvqLinear(q1.data_ptr(), s1.data_ptr(), g1.data_ptr(), b1.data_ptr(), D_MODEL, D_FF)
        l2 = _lib.FvqLinear(q2.data_ptr(), s2.data_ptr(), g2.data_ptr(), b2.data_ptr(), D_FF, D_MODEL)
        structs.append((x, l1, l2))
    ffn_call = lib.fvq_nvfp4_ffn

    def step(i):
        x, l1, l2 = structs[i % ROTATE]
        rc = ffn_call(x.data_ptr(), tokens, ctypes.byref(l1), ctypes.byref(l2), ys[i % ROTATE].data_ptr(),
                      ws.data_ptr(), ws_bytes, sptr)
        if rc != 0:
            raise RuntimeError(lib.fvq_last_error().decode())

    def barrier_sync():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for i in range(max(3, args.warmup)):
        step(i)
    barrier_sync()
    gpu_uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    sampler = clock_sampler(gpu_uuid)
    sampler.start()
    if isinstance(sampler, ClockSampler):
        time.sleep(0.15)  # nvidia-smi's start-up
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier_sync()
    start.record(stream)
    for i in range(args.steps):
        step(i)
    end.record(stream)
    barrier_sync()
    clocks = sampler.stop()
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    total_tokens = tokens * args.steps * world
    value = total_tokens / (ms * 1e-3)
    tflops = value * FLOP_PER_TOKEN / 1e12

    # ---- per-kernel timing (the library's events around fvq_nvfp4_ffn's launches)
    kt = kernel_timing(lib, structs, ys, ws, ws_bytes, tokens, sptr, min(args.steps, 400))
    if world > 1:
        t = torch.tensor([kt["gemm_ms"], kt["quant_h_ms"]], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        kt["gemm_ms"], kt["quant_h_ms"] = (float(v) for v in t.tolist())

    # ---- end to end through the public module API with host buffers
    e2e = e2e_timing(torch, dist, fvq, NVFP4FFN, sets, tokens, dev, stream, world,
                     min(args.steps, 500), args.warmup)

    # ---- output gather (NCCL all-gather over NVLink) of one layer's output
    gather = None
    if world > 1:
        from flashvsr_optimizations_b200.sharding import gather_rows
        total = tokens * world
        for _ in range(3):
            gather_rows(ys[0], total)
        barrier_sync()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        for _ in range(20):
            gather_rows(ys[0], total)
        e.record(stream)
        barrier_sync()
        gms = s.elapsed_time(e) / 20
        t = torch.tensor([gms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        gms = float(t.item())
        gather = {"ms": gms, "bytes": total * D_MODEL * 2,
                  "busbw_GBps": (world - 1) * tokens * D_MODEL * 2 / (gms * 1e-3) / 1e9,
                  "api": "sharding.gather_rows (NCCL all_gather_into_tensor)"}

    peaks = measured_peaks()
    fp4_cublas = fp4_library_peak(torch, dev) if rank == 0 else None
    # the GEMMs are timed inside long runs of layers, where the 1000 W cap holds the SM
    # clock well below its maximum: the sustained bf16 figure is the matching denominator
    bf16_sustained = peaks.get("bf16_tflops_sustained")
    if bf16_sustained:
        peak = 4.0 * bf16_sustained
        peak_src = ("4 x measured cuBLAS bf16 sustained (MEASURED_PEAKS.json, power-capped); "
                    "dense FP4 runs at 4x bf16 on B200")
    else:
        peak, peak_src = 4.0 * 1400.0, "4 x fallback sustained bf16 1.4 PFLOP/s"
    hbm = peaks.get("hbm_gbs") or 6650.0
    gemm_flop = tokens * FLOP_PER_TOKEN
    achieved = gemm_flop / (kt["gemm_ms"] * 1e-3) / 1e12
    traffic = None
    tp = ROOT / "profiles" / "nvfp4_gemm_ffn_layer_7680tok_traffic.json"
    if tp.exists():
        try:
            traffic = json.loads(tp.read_text()).get("dram_bytes_per_gemm_pair")
        except ValueError:
            traffic = None
    extras = {}
    if not args.no_extras:
        stack = stack_timing(torch, dist, ops, lib, dev, stream, world, rank)
        stack["tflops_frac_of_fp4_peak"] = stack["tflops"] / (peak * world)  # whole job / N GPUs
        extras["stack_30_layers"] = stack
        if rank == 0:
            extras["quantize_sweep"] = quantize_sweep(torch, lib, dev, stream, hbm)
            fp8_peak = 2.0 * (bf16_sustained or 1400.0)
            extras["fp8_mode"] = fp8_mode_timing(torch, ops, lib, dev, stream, tokens, fp8_peak)
            extras["pil_resize"] = pil_resize_timing(torch, dev, stream, hbm)
            extras["dit_block"] = dit_block_timing(torch, lib, dev, stream, sets, tokens, hbm)
    result = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "nvfp4(e2m1+e4m3 scales), fp32 accumulate, bf16 io",
        "data": "synthetic (seeded Student-t(4)x0.5 activations, N(0,0.02) weights, N(0,0.01) bias)",
        "config": {"workload": WORKLOAD, "tokens_per_gpu": tokens, "d_model": D_MODEL, "d_ff": D_FF,
                   "layers": 1, "parallelism": f"token-row shards x{world}, replicated weights",
                   "l2": f"inputs rotate over {ROTATE} distinct activation/weight sets (312 MB > 126 MB L2)"},
        "tflops": tflops, "tflops_frac_of_fp4_peak": tflops / (peak * world),
        "gpu_launches": LAUNCHES_PER_LAYER * args.steps,
        "roofline": {"bound": "tensor", "kernel": "nvfp4_gemm_kernel (GEMM1 + GEMM2 of the layer)",
                     "achieved": achieved, "peak": peak, "peak_source": peak_src, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "algorithmic_flop_per_launch_pair": gemm_flop},
        "quantize": {"kernel": "quantize_kernel on the 7680x8960 intermediate",
                     "GBps": kt["quant_h_gbs"], "peak_GBps": hbm, "frac": kt["quant_h_gbs"] / hbm,
                     "ms": kt["quant_h_ms"]},
        "kernels_ms": kt,
        "e2e": e2e,
        "clocks": clocks,
    }
    if gather:
        result["gather"] = gather
    result.update(extras)
    if fp4_cublas:
        result["fp4_cublas_8192_tflops"] = fp4_cublas
    if rank == 0 and not args.no_extras:
        lib_sustained = fp4_library_sustained(torch, dev)
        if lib_sustained:
            result["fp4_cublas_sustained_layer_shapes"] = lib_sustained
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_ffn_tokens_per_s(5, 1, args.cpu_seconds)
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def kernel_timing(lib, structs, ys, ws, ws_bytes, tokens, sptr, steps) -> dict:
    """Device time of each of fvq_nvfp4_ffn's four launches, from the library's own
    CUDA events (fvq_nvfp4_ffn_profile runs the same launch sequence and synchronises
    after each layer, so every launch here starts on an idle GPU)."""
    ms = (ctypes.c_float * 4)()
    acc = [[] for _ in range(4)]

    def one(i):
        x, l1, l2 = structs[i % ROTATE]
        rc = lib.fvq_nvfp4_ffn_profile(x.data_ptr(), tokens, ctypes.byref(l1), ctypes.byref(l2),
                                       ys[i % ROTATE].data_ptr(), ws.data_ptr(), ws_bytes, sptr, ms)
        if rc != 0:
            raise RuntimeError(lib.fvq_last_error().decode())

    for i in range(5):
        one(i)
    for i in range(steps):
        one(i)
        for j in range(4):
            acc[j].append(ms[j])
    qx, g1t, qh, g2t = (sum(v) / len(v) for v in acc)
    d, f = D_MODEL, D_FF
    qh_bytes = tokens * f * 2 + tokens * f // 2 + (tokens + 127) // 128 * 128 * f // 16
    return {"quant_x_ms": qx, "gemm1_ms": g1t, "quant_h_ms": qh, "gemm2_ms": g2t,
            "gemm_ms": g1t + g2t, "quant_h_gbs": qh_bytes / (qh * 1e-3) / 1e9,
            "gemm1_tflops": tokens * 2 * d * f / (g1t * 1e-3) / 1e12,
            "gemm2_tflops": tokens * 2 * d * f / (g2t * 1e-3) / 1e12, "steps": steps,
            "note": "quant_x also writes the replicated W2 scales when GEMM2 runs on one SM per tile (not with the default SM pairs); launches timed one layer at a time"}


def e2e_timing(torch, dist, fvq, NVFP4FFN, sets, tokens, dev, stream, world, steps, warmup) -> dict:
    """Same metric through the public module (NVFP4FFN) with pinned host input/output.

    Every step copies its input host->device, runs the module and copies the result
    device->host, all inside the timed region.  The copies run on their own streams,
    so step i+1's upload and step i-1's download overlap step i's compute (PCIe is
    full duplex); device inputs are double-buffered and ordered with events.
    """
    from flashvsr_optimizations_b200.ffn_quantization import QuantLinear
    mods = []
    for x, ((q1, s1, g1, b1), (q2, s2, g2, b2)) in sets:
        l1 = QuantLinear.from_quantized(q1, s1, g1, b1, D_MODEL)
        l2 = QuantLinear.from_quantized(q2, s2, g2, b2, D_FF)
        mods.append(NVFP4FFN(l1, torch.nn.GELU(approximate="tanh"), l2))
    xh = [x.cpu().pin_memory() for x, _ in sets]
    yh = [torch.empty(tokens, D_MODEL, dtype=torch.bfloat16).pin_memory() for _ in range(ROTATE)]
    xd = [torch.empty(tokens, D_MODEL, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    s_up, s_cmp, s_down = (torch.cuda.Stream(dev) for _ in range(3))
    done_cmp = [torch.cuda.Event() for _ in range(2)]   # compute that read xd[b] finished
    for ev in done_cmp:
        ev.record(s_cmp)

    def step(i):
        j, b = i % ROTATE, i % 2
        up = torch.cuda.Event()
        with torch.cuda.stream(s_up):
            s_up.wait_event(done_cmp[b])
            xd[b].copy_(xh[j], non_blocking=True)
            up.record(s_up)
        with torch.cuda.stream(s_cmp):
            s_cmp.wait_event(up)
            y = mods[j](xd[b])
            done_cmp[b].record(s_cmp)
        with torch.cuda.stream(s_down):
            s_down.wait_event(done_cmp[b])
            yh[j].copy_(y, non_blocking=True)
            y.record_stream(s_down)

    with torch.no_grad():
        for i in range(max(3, warmup)):
            step(i)
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
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
    ms = s.elapsed_time(e)
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return {"value": tokens * steps * world / (ms * 1e-3), "unit": "tokens/s",
            "h2d_bytes_per_step": tokens * D_MODEL * 2, "d2h_bytes_per_step": tokens * D_MODEL * 2,
            "steps": steps, "ms_per_step": ms / steps,
            "api": "NVFP4FFN.forward (install_ffn's fused module) via torch custom op fvq::nvfp4_ffn; "
                   "uploads, layers and downloads on three streams, overlapped across steps"}


def run_reference(args, rank, world):
    if rank != 0:
        return
    res = cpu_ffn_tokens_per_s(args.steps, args.warmup, seconds=60.0)
    ms_per_step = res["seconds"] / args.steps * 1e3
    line = {"metric": METRIC, "value": res["value"], "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "nvfp4 emulated (fp32 dequantized matmul)", "data": "synthetic (seeded)",
            "config": {"workload": WORKLOAD, "tokens_per_step": res["rows_per_step"],
                       "d_model": D_MODEL, "d_ff": D_FF, "layers": 1, "parallelism": "host CPU"},
            "impl": "reference",
            "cpu_baseline": {"value": res["value"], "unit": "tokens/s", "cores": res["cores"],
                             "kind": res["kind"], "sample": res["sample"]},
            "e2e": {"value": res["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
