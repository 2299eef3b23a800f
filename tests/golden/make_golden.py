"""Generate the golden fixtures of tests/golden/ from the reference path on a B200.

    FLASHINFER_WORKSPACE_BASE=baseline/fi_jit FLASHINFER_CUDA_ARCH_LIST=10.0a \
        python tests/golden/make_golden.py [--out tests/golden] [--time out.json] [--stack-only]

The reference computes its NVFP4 FFN with ``global_scale`` (ffn_quantization.py
:29-32), ``flashinfer.nvfp4_quantize`` (:47, :64), ``flashinfer.mm_fp4(...,
backend='cutlass')`` (:65-67), a bf16 bias add (:68-69) and the upstream
``GELU(approximate='tanh')`` between the two linears.  This script runs that
sequence with FlashInfer's own kernels on seeded inputs from ``workloads.py``.
The stack-workload cases come from the reference's own module
(``ffn_quantization.QuantLinear``, installed unmodified into baseline/_ref by
``__graft_entry__.build()``); the earlier cases restate its scalar glue inline,
and the script records in golden_meta.json whether that restatement and the
reference module give the same bits (``restated_glue_equals_reference_module``).
It stores:

* quantizer cases: codes, swizzled scale factors and global scale, plus the
  GPU's ``rcp.approx.ftz.f32`` results for every reciprocal argument the case
  needs (measured with libfvq's probe), so the CPU oracle can be bit-exact;
* large quantizer cases: SHA-256 digests of codes and scale factors;
* a QuantLinear case and a small FFN case: full bf16 outputs;
* the one-layer FFN at 7680 tokens: 64 seeded rows of the output and its norm;
* one layer of the 30-layer stack workloads (15360 and 64800 tokens) on the whole
  input and on rank 0's row block at 2, 4 and 8 GPUs: 64 seeded rows, the norm and
  the global scale of x, computed by the reference's own ``ffn_quantization``
  module when it is installed in baseline/_ref (``--stack-only`` adds just these).

Inputs are not stored: tests regenerate them from the same seeds.
With ``--time`` it also times the reference kernels on the benchmark shapes.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import flashvsr_optimizations_b200 as fvq  # noqa: E402
from flashvsr_optimizations_b200 import workloads as W  # noqa: E402
from oracle import nvfp4_oracle as O  # noqa: E402

import flashinfer  # noqa: E402


def to_dev(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(bits.astype(np.int16)).view(torch.bfloat16).cuda()


def ref_global_scale(x: torch.Tensor) -> torch.Tensor:
    # _partial_amax + p.amax() is an exact max; 2688./t is t.reciprocal()*2688
    amax = x.float().abs().amax()
    return (2688. / amax.clamp_min(1.e-12)).reshape(1)


class RefQuantLinear:
    def __init__(self, w: torch.Tensor, b: torch.Tensor | None):
        self.bias = b
        self.global_sf = ref_global_scale(w)
        self.qweight, self.scale = flashinfer.nvfp4_quantize(w, self.global_sf)
        self.out_features = w.shape[0]

    def forward(self, x: torch.Tensor, keep: dict | None = None) -> torch.Tensor:
        g = ref_global_scale(x)
        q, s = flashinfer.nvfp4_quantize(x, g)
        out = flashinfer.mm_fp4(q, self.qweight.t(), s, self.scale.t(), alpha=1. / (g * self.global_sf),
                                out_dtype=torch.bfloat16, backend="cutlass")
        if keep is not None:
            keep.update(g=g, q=q, s=s)
        if self.bias is not None:
            out = out + self.bias
        return out


def ref_ffn(x, l1, l2, keep=None):
    k1, k2 = ({}, {}) if keep is not None else (None, None)
    h = l1.forward(x, k1)
    h = torch.nn.functional.gelu(h, approximate="tanh")
    y = l2.forward(h, k2)
    if keep is not None:
        keep.update(h=h, g1=k1["g"], g2=k2["g"], qh=k2["q"], sh=k2["s"])
    return y


def u32(t: torch.Tensor | np.ndarray) -> np.ndarray:
    a = t.detach().cpu().numpy() if isinstance(t, torch.Tensor) else t
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def raw(t: torch.Tensor) -> np.ndarray:
    """The bytes of any tensor (fp4 / bf16 dtypes included) as a uint8 array."""
    return t.detach().contiguous().view(torch.uint8).cpu().numpy()


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(raw(t).tobytes()).hexdigest()


def rcp_table(x_bits: np.ndarray, g: float) -> tuple[np.ndarray, np.ndarray]:
    args = np.array(O.rcp_arguments(x_bits, g), dtype=np.uint32)
    res = fvq.ops.rcp_approx_probe(torch.from_numpy(args.view(np.float32)).cuda())
    return args, u32(res)


QUANT_CASES = {
    # name: (generator, kwargs)
    "q_gauss_128x1536": (W.gaussian, dict(m=128, k=1536, seed=10)),
    "q_gauss_200x192": (W.gaussian, dict(m=200, k=192, seed=11)),
    "q_outlier_16x8960": (W.with_outliers, dict(m=16, k=8960, seed=2)),
    "q_studentt_64x1536": (W.student_t, dict(m=64, k=1536, seed=12)),
    "q_edge_130x256": (W.edge_case_tensor, dict(m=130, k=256, seed=5)),
}
FIXED_G_CASES = {  # explicit encode scales: saturating (x > 448 scales) and underflowing
    "q_edge_130x256_g1e6": ("q_edge_130x256", 1.0e6),
    "q_edge_130x256_g1e-3": ("q_edge_130x256", 1.0e-3),
}
HASH_CASES = {
    "h_outlier_1024x1536": (W.with_outliers, dict(m=1024, k=1536, seed=2)),
    "h_outlier_1024x8960": (W.with_outliers, dict(m=1024, k=8960, seed=2)),
    "h_gauss_4096x1536": (W.gaussian, dict(m=4096, k=1536, seed=13)),
}


def quant_fixture(x_bits: np.ndarray, g: torch.Tensor | None):
    x = to_dev(x_bits)
    if g is None:
        g = ref_global_scale(x)
    q, s = flashinfer.nvfp4_quantize(x, g)
    args, res = rcp_table(x_bits, float(g.item()))
    return dict(codes=raw(q), sf=raw(s).reshape(-1),
                g_bits=u32(g), rcp_args=args, rcp_res=res), q, s


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(ROOT / "tests" / "golden"))
    ap.add_argument("--time", default=None, help="also time the reference kernels; JSON path")
    ap.add_argument("--stack-only", action="store_true",
                    help="only (re)make the stack-workload cases and add them to golden_meta.json")
    a = ap.parse_args()
    out = Path(a.out)
    out.mkdir(parents=True, exist_ok=True)
    torch.manual_seed(0)
    if a.stack_only:
        meta = json.loads((out / "golden_meta.json").read_text())
        stack_cases(out, meta)
        (out / "golden_meta.json").write_text(json.dumps(meta, indent=1, sort_keys=True))
        print("added stack cases to", out)
        return
    meta = {"flashinfer": flashinfer.__version__, "torch": torch.__version__,
            "device": torch.cuda.get_device_name(), "cases": {}}

    # ---- quantizer, full outputs
    for name, (gen, kw) in QUANT_CASES.items():
        xb = gen(**kw)
        fix, _, _ = quant_fixture(xb, None)
        np.savez_compressed(out / f"{name}.npz", **fix)
        meta["cases"][name] = {"generator": gen.__name__, **kw}
    for name, (base, gval) in FIXED_G_CASES.items():
        gen, kw = QUANT_CASES[base]
        xb = gen(**kw)
        fix, _, _ = quant_fixture(xb, torch.tensor([gval], dtype=torch.float32, device="cuda"))
        np.savez_compressed(out / f"{name}.npz", **fix)
        meta["cases"][name] = {"generator": gen.__name__, **kw, "g": gval}

    # ---- quantizer, digests
    for name, (gen, kw) in HASH_CASES.items():
        xb = gen(**kw)
        x = to_dev(xb)
        g = ref_global_scale(x)
        q, s = flashinfer.nvfp4_quantize(x, g)
        args, res = rcp_table(xb, float(g.item()))
        np.savez_compressed(out / f"{name}.npz", g_bits=u32(g), rcp_args=args, rcp_res=res)
        meta["cases"][name] = {"generator": gen.__name__, **kw, "codes_sha256": sha(q),
                               "sf_sha256": sha(s)}

    # ---- QuantLinear (mm_fp4 + bias)
    wb, bb = W.linear_params(256, 1536, seed=30, b_std=0.01)
    xb = W.gaussian(200, 1536, seed=31)
    lin = RefQuantLinear(to_dev(wb), to_dev(bb))
    keep = {}
    y = lin.forward(to_dev(xb), keep)
    np.savez_compressed(out / "lin_200x1536x256.npz", y=raw(y).view(np.uint16),
                        g_bits=u32(keep["g"]), gw_bits=u32(lin.global_sf))
    meta["cases"]["lin_200x1536x256"] = {"x": "gaussian(200,1536,seed=31)",
                                         "w": "linear_params(256,1536,seed=30,b_std=0.01)",
                                         "qweight_sha256": sha(lin.qweight), "scale_sha256": sha(lin.scale)}

    # ---- FFN, small (full output) and one layer at 7680 tokens (sampled rows)
    w1, b1 = W.linear_params(W.D_FF, W.D_MODEL, seed=20, b_std=0.01)
    w2, b2 = W.linear_params(W.D_MODEL, W.D_FF, seed=21, b_std=0.01)
    l1 = RefQuantLinear(to_dev(w1), to_dev(b1))
    l2 = RefQuantLinear(to_dev(w2), to_dev(b2))
    weights_meta = {"w1": "linear_params(8960,1536,seed=20,b_std=0.01)",
                    "w2": "linear_params(1536,8960,seed=21,b_std=0.01)",
                    "qweight1_sha256": sha(l1.qweight), "scale1_sha256": sha(l1.scale),
                    "qweight2_sha256": sha(l2.qweight), "scale2_sha256": sha(l2.scale),
                    "global_sf1_bits": int(u32(l1.global_sf)[0]),
                    "global_sf2_bits": int(u32(l2.global_sf)[0])}
    xb = W.student_t(64, W.D_MODEL, seed=1)
    keep = {}
    y = ref_ffn(to_dev(xb), l1, l2, keep)
    np.savez_compressed(out / "ffn_64.npz", y=raw(y).view(np.uint16),
                        g1_bits=u32(keep["g1"]), g2_bits=u32(keep["g2"]),
                        h=raw(keep["h"]).view(np.uint16))
    meta["cases"]["ffn_64"] = {"x": "student_t(64,1536,seed=1)", **weights_meta,
                               "h_codes_sha256": sha(keep["qh"]), "h_sf_sha256": sha(keep["sh"])}
    xb = W.student_t(W.M_ONE_LAYER, W.D_MODEL, seed=1)
    keep = {}
    y = ref_ffn(to_dev(xb), l1, l2, keep)
    rows = np.sort(np.random.default_rng(99).choice(W.M_ONE_LAYER, 64, replace=False))
    np.savez_compressed(out / "ffn_7680_rows.npz", rows=rows,
                        y_rows=raw(y[torch.from_numpy(rows).cuda()]).view(np.uint16),
                        g1_bits=u32(keep["g1"]), g2_bits=u32(keep["g2"]))
    meta["cases"]["ffn_7680_rows"] = {"x": "student_t(7680,1536,seed=1)", **weights_meta,
                                      "y_fro": float(y.float().norm().item()),
                                      "y_sha256": sha(y)}
    stack_cases(out, meta)
    (out / "golden_meta.json").write_text(json.dumps(meta, indent=1, sort_keys=True))
    print("wrote", len(meta["cases"]), "cases to", out)

    if a.time:
        timings = time_reference(l1, l2)
        Path(a.time).write_text(json.dumps(timings, indent=1))
        print(json.dumps(timings, indent=1))


def reference_module():
    """The reference's own ffn_quantization module, installed unmodified into baseline/_ref
    (``__graft_entry__.build()`` puts it there), or None when it is not installed."""
    ref_dir = ROOT / "baseline" / "_ref"
    if not (ref_dir / "ffn_quantization.py").exists():
        return None
    if str(ref_dir) not in sys.path:
        sys.path.insert(0, str(ref_dir))
    import ffn_quantization
    return ffn_quantization


def reference_ffn_modules(w1, b1, w2, b2):
    """nn.Sequential(QuantLinear, GELU(tanh), QuantLinear) built by the reference's own
    QuantLinear(linear, 'nvfp4') (ffn_quantization.py:35-52) from bf16 weights."""
    ref = reference_module()

    def linear(wb, bb):
        out_f, in_f = wb.shape
        lin = torch.nn.Linear(in_f, out_f, bias=True, device="cuda", dtype=torch.bfloat16)
        with torch.no_grad():
            lin.weight.copy_(to_dev(wb))
            lin.bias.copy_(to_dev(bb))
        return ref.QuantLinear(lin, "nvfp4")

    return torch.nn.Sequential(linear(w1, b1), torch.nn.GELU(approximate="tanh"), linear(w2, b2))


# Stack workloads: one layer (layer 0 of the stack's weights) on the stack inputs, on the
# whole tensor and on rank 0's row block at each GPU count (the reference run on that
# shard: per-shard global scales).  (name, input generator, kwargs, rows of the shard)
STACK_CASES = [
    ("ffn_c4_15360", W.gaussian, dict(m=W.M_STACK, k=W.D_MODEL, seed=3), (15360, 7680, 3840, 1920)),
    ("ffn_c5_64800", W.student_t, dict(m=W.M_4K, k=W.D_MODEL, seed=4), (64800, 32400, 16200, 8100)),
]


def stack_cases(out: Path, meta: dict) -> None:
    """64 seeded output rows, the Frobenius norm and the global scales of one FFN layer at
    the stack workloads' sizes, from the reference's own module when it is installed (else
    from the restated glue above, which gives the same bits: checked on ffn_64 here)."""
    w1, b1, w2, b2 = W.stack_layer_params(0)
    ref = reference_module()
    with torch.no_grad():
        if ref is not None:
            seq = reference_ffn_modules(w1, b1, w2, b2)
            run = lambda x: seq(x)  # noqa: E731
            # the restated glue and the reference module agree on the small golden case
            sw1, sb1 = W.linear_params(W.D_FF, W.D_MODEL, seed=20, b_std=0.01)
            sw2, sb2 = W.linear_params(W.D_MODEL, W.D_FF, seed=21, b_std=0.01)
            l1 = RefQuantLinear(to_dev(sw1), to_dev(sb1))
            l2 = RefQuantLinear(to_dev(sw2), to_dev(sb2))
            small = reference_ffn_modules(sw1, sb1, sw2, sb2)
            xs = to_dev(W.student_t(64, W.D_MODEL, seed=1))
            meta["restated_glue_equals_reference_module"] = bool(
                torch.equal(ref_ffn(xs, l1, l2), small(xs)))
            source = "baseline/_ref/ffn_quantization.py (the reference module, unmodified)"
        else:
            l1 = RefQuantLinear(to_dev(w1), to_dev(b1))
            l2 = RefQuantLinear(to_dev(w2), to_dev(b2))
            run = lambda x: ref_ffn(x, l1, l2)  # noqa: E731
            source = "restated glue (reference module not installed)"
        for name, gen, kw, shard_rows in STACK_CASES:
            x_all = to_dev(gen(**kw))
            for rows in shard_rows:
                x = x_all[:rows].contiguous()
                y = run(x)
                pick = np.sort(np.random.default_rng(rows).choice(rows, 64, replace=False))
                g1 = ref_global_scale(x)
                case = f"{name}_rows{rows}"
                np.savez_compressed(out / f"{case}.npz", rows=pick,
                                    y_rows=raw(y[torch.from_numpy(pick).cuda()]).view(np.uint16),
                                    g1_bits=u32(g1))
                meta["cases"][case] = {"x": f"{gen.__name__}({kw['m']},{kw['k']},seed={kw['seed']})[:{rows}]",
                                       "weights": "workloads.stack_layer_params(0)",
                                       "y_fro": float(y.float().norm().item()), "y_sha256": sha(y),
                                       "source": source}
                del y, x
            del x_all
            torch.cuda.empty_cache()


def _time(fn, iters=20, warmup=5):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    ts = []
    for _ in range(iters):
        flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        ts.append(s.elapsed_time(e))
    return float(np.median(ts))


def time_reference(l1, l2) -> dict:
    res = {"flashinfer": flashinfer.__version__, "device": torch.cuda.get_device_name()}
    for m in W.QUANT_SWEEP_M:
        for k in W.QUANT_SWEEP_K:
            x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
            g = ref_global_scale(x)
            ms = _time(lambda: flashinfer.nvfp4_quantize(x, g))
            ms_gs = _time(lambda: flashinfer.nvfp4_quantize(x, ref_global_scale(x)))
            nbytes = m * k * 2 + m * k // 2 + ((m + 127) // 128 * 128) * k // 16
            res[f"nvfp4_quantize_{m}x{k}"] = {"ms": ms, "GBps": nbytes / ms / 1e6,
                                              "with_global_scale_ms": ms_gs}
    m = W.M_ONE_LAYER
    x = torch.randn(m, W.D_MODEL, device="cuda", dtype=torch.bfloat16)
    g = ref_global_scale(x)
    q, s = flashinfer.nvfp4_quantize(x, g)
    alpha = 1. / (g * l1.global_sf)
    ms = _time(lambda: flashinfer.mm_fp4(q, l1.qweight.t(), s, l1.scale.t(), alpha=alpha,
                                         out_dtype=torch.bfloat16, backend="cutlass"))
    res["mm_fp4_gemm1_7680x8960x1536"] = {"ms": ms, "TFLOPs": 2 * m * W.D_FF * W.D_MODEL / ms / 1e9}
    h = torch.randn(m, W.D_FF, device="cuda", dtype=torch.bfloat16)
    g = ref_global_scale(h)
    q, s = flashinfer.nvfp4_quantize(h, g)
    alpha = 1. / (g * l2.global_sf)
    ms = _time(lambda: flashinfer.mm_fp4(q, l2.qweight.t(), s, l2.scale.t(), alpha=alpha,
                                         out_dtype=torch.bfloat16, backend="cutlass"))
    res["mm_fp4_gemm2_7680x1536x8960"] = {"ms": ms, "TFLOPs": 2 * m * W.D_FF * W.D_MODEL / ms / 1e9}
    xb = torch.randn(m, W.D_MODEL, device="cuda", dtype=torch.bfloat16)
    ms = _time(lambda: ref_ffn(xb, l1, l2))
    res["ref_ffn_layer_7680"] = {"ms": ms, "tokens_per_s": m / ms * 1e3,
                                 "TFLOPs": m * W.FLOP_PER_TOKEN / ms / 1e9}
    return res


if __name__ == "__main__":
    t0 = time.time()
    main()
    print(f"done in {time.time() - t0:.1f}s")
