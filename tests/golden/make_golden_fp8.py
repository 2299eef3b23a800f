"""Generate the FP8-mode golden fixtures of tests/golden/ from the reference's steps on a B200.

    python tests/golden/make_golden_fp8.py [--out tests/golden] [--time out.json]

The reference's FP8 mode quantizes rows with a Triton kernel (``_row_quant``,
ffn_quantization.py:6-13, called by ``row_quant`` :22-26 on weights :44-45
and activations :58) and multiplies with ``torch._scaled_mm(q, qweight.t(),
scale_a=s, scale_b=scale.t(), out_dtype=bf16, use_fast_accum=False)``
(:59-60) before the bias add (:68-69).  Its per-tensor activation quantizer
(decoder_fp8.py:9-24, reused by lq_fp8.py:24-31) is a second Triton kernel
after a ``_partial_amax`` pass and a torch ``amax / 448``.

The reference file is not available where this runs, so the two Triton
kernels are restated below step for step -- the same loads, the same fp32
operations (``tl.max`` of ``|x|``, ``/ 448.``, ``tl.maximum(.., 1e-12)``,
``x / scale``, the clamp to +-448) and the same fp8 stores -- so Triton emits
the same instructions.  They also store their fp32 quotients: for each
division whose GPU result (``div.full.f32``) differs from the IEEE quotient
in a way that changes an E4M3 code or a scale, the fixture keeps (dividend,
divisor, quotient) bits, which make the CPU oracle bit-exact.

Stored per case (inputs are regenerated from seeds by ``workloads.py``):
row and tensor quantizer codes and scales (or their SHA-256 for large cases),
a QuantLinear('fp8') output, a small FFN's output and intermediate, and 64
seeded rows of the one-layer FFN at 7680 tokens.  It also records how many
Triton quotients differ from libfvq's ``div.full.f32`` probe on the same
operands (``quotients_differing_from_div_full``; the tests require 0).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import sys
import time
from pathlib import Path

import numpy as np
import torch
import triton
import triton.language as tl

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import flashvsr_optimizations_b200 as fvq  # noqa: E402
from flashvsr_optimizations_b200 import workloads as W  # noqa: E402
from oracle import nvfp4_oracle as O  # noqa: E402


@triton.jit
def _rows_to_e4m3(X, Q, S, D, K: tl.constexpr, BLOCK: tl.constexpr, KEEP_D: tl.constexpr):
    row = tl.program_id(0)
    col = tl.arange(0, BLOCK)
    inside = col < K
    v = tl.load(X + row * K + col, inside, other=0).to(tl.float32)
    s = tl.maximum(tl.max(tl.abs(v), 0) / 448., 1.e-12)
    d = v / s
    tl.store(Q + row * K + col, d, inside)
    if KEEP_D:
        tl.store(D + row * K + col, d, inside)
    tl.store(S + row, s)


@triton.jit
def _tensor_to_e4m3(X, Q, S, D, N: tl.constexpr, B: tl.constexpr):
    i = tl.program_id(0) * B + tl.arange(0, B)
    inside = i < N
    v = tl.load(X + i, inside, other=0).to(tl.float32)
    s = tl.load(S)
    d = v / s
    tl.store(Q + i, tl.minimum(tl.maximum(d, -448.), 448.), inside)
    tl.store(D + i, d, inside)


def to_dev(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).astype(np.int16)).view(torch.bfloat16).cuda()


def raw(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.uint8).cpu().numpy()


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(raw(t).tobytes()).hexdigest()


def u32(t) -> np.ndarray:
    a = t.detach().cpu().numpy() if isinstance(t, torch.Tensor) else t
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def ref_row_quant(x: torch.Tensor, keep_quotients: bool = True):
    """(q e4m3 [M, K], s fp32 [M, 1], fp32 quotients [M, K] or None) -- the reference's
    row_quant; without keep_quotients it does exactly the reference kernel's work."""
    m, k = x.shape
    q = torch.empty_like(x, dtype=torch.float8_e4m3fn)
    s = torch.empty((m, 1), device=x.device, dtype=torch.float32)
    d = torch.empty((m, k) if keep_quotients else (1,), device=x.device, dtype=torch.float32)
    _rows_to_e4m3[(m,)](x, q, s, d, k, triton.next_power_of_2(k), keep_quotients)
    return q, s, (d if keep_quotients else None)


def ref_quantize_activation(x: torch.Tensor):
    """(q e4m3 like x, scale fp32 [1], fp32 quotients) -- decoder_fp8.quantize_activation."""
    n = x.numel()
    scale = (x.float().abs().amax() / 448.).clamp_min(1e-12).reshape(1)
    q = torch.empty_like(x, dtype=torch.float8_e4m3fn)
    d = torch.empty_like(x, dtype=torch.float32)
    _tensor_to_e4m3[(triton.cdiv(n, 4096),)](x, q, scale, d, n, 4096)
    return q, scale, d


class RefFp8Linear:
    def __init__(self, w: torch.Tensor, b: torch.Tensor | None, tables: list | None = None):
        self.qweight, self.scale, d = ref_row_quant(w, keep_quotients=tables is not None)
        if tables is not None:
            tables.append(row_table(w, self.scale, d))
        self.bias = b
        self.out_features = w.shape[0]

    def forward(self, x: torch.Tensor, keep: dict | None = None,
                tables: list | None = None) -> torch.Tensor:
        q, s, d = ref_row_quant(x, keep_quotients=tables is not None)
        if tables is not None:
            tables.append(row_table(x, s, d))
        out = torch._scaled_mm(q, self.qweight.t(), scale_a=s, scale_b=self.scale.t(),
                               out_dtype=torch.bfloat16, use_fast_accum=False)
        if keep is not None:
            keep.update(q=q, s=s)
        if self.bias is not None:
            out = out + self.bias
        return out


def ref_ffn(x, l1, l2, keep=None, tables=None):
    k1, k2 = ({}, {}) if keep is not None else (None, None)
    h = l1.forward(x, k1, tables)
    h = torch.nn.functional.gelu(h, approximate="tanh")
    y = l2.forward(h, k2, tables)
    if keep is not None:
        keep.update(h=h, qh=k2["q"], sh=k2["s"])
    return y


def code_changing_divisions(a: np.ndarray, b: np.ndarray, d_gpu: np.ndarray, clamp: bool):
    """(a, b, q) bits of the divisions whose GPU quotient differs from the IEEE one
    by enough to change the E4M3 code, and the count of all differing quotients."""
    shape = np.shape(a)
    a = np.ascontiguousarray(a, dtype=np.float32).ravel()
    b = np.ascontiguousarray(np.broadcast_to(np.asarray(b, np.float32), shape)).ravel()
    g = np.ascontiguousarray(d_gpu, dtype=np.float32).ravel()
    with np.errstate(all="ignore"):
        ieee = (a / b).astype(np.float32)
    diff = ieee.view(np.uint32) != g.view(np.uint32)
    if clamp:
        ci, cg = np.clip(ieee, -448, 448), np.clip(g, -448, 448)
    else:
        ci, cg = ieee, g
    changes = diff & (O.f32_to_e4m3(ci) != O.f32_to_e4m3(cg))
    return (a[changes].view(np.uint32), b[changes].view(np.uint32), g[changes].view(np.uint32),
            int(diff.sum()))


def row_table(x: torch.Tensor, s: torch.Tensor, d: torch.Tensor):
    """Division table of one row quantization: (a, b, q) bits of the code-changing
    element divisions and of every row scale that differs from the IEEE one, plus
    the count of element quotients that differ from IEEE and of such rows."""
    xf = x.detach().float().cpu().numpy()
    s_np = s.detach().cpu().numpy().reshape(-1).astype(np.float32)
    a, b, qd, n_diff = code_changing_divisions(xf, s_np[:, None], d.cpu().numpy(), clamp=False)
    amax = np.abs(xf).max(axis=1).astype(np.float32)
    with np.errstate(all="ignore"):
        ieee_s = np.maximum((amax / np.float32(448)).astype(np.float32), np.float32(1e-12))
    bad = ieee_s.view(np.uint32) != s_np.view(np.uint32)
    a = np.concatenate([a, amax[bad].view(np.uint32)])
    b = np.concatenate([b, np.full(int(bad.sum()), np.float32(448)).view(np.uint32)])
    qd = np.concatenate([qd, s_np[bad].view(np.uint32)])
    return a, b, qd, n_diff, int(bad.sum())


def merged(tables: list) -> dict:
    return dict(div_a=np.concatenate([t[0] for t in tables]).astype(np.uint32),
                div_b=np.concatenate([t[1] for t in tables]).astype(np.uint32),
                div_q=np.concatenate([t[2] for t in tables]).astype(np.uint32))


def row_fixture(xb: np.ndarray, store_codes: bool = True):
    x = to_dev(xb)
    q, s, d = ref_row_quant(x)
    xf = O.bf16_bits_to_f32(xb)
    a, b, qd, n_diff, n_bad = row_table(x, s, d)
    # the instruction the reference's `/` becomes is the one libfvq issues
    probe = fvq.ops.div_full_probe(torch.from_numpy(xf).cuda(),
                                   s.expand(-1, xf.shape[1]).contiguous())
    fix = dict(s_bits=u32(s.reshape(-1)), div_a=a, div_b=b, div_q=qd)
    if store_codes:
        fix["q"] = raw(q)
    info = {"quotients_differing_from_ieee": n_diff, "code_changing": int(len(a) - n_bad),
            "scale_rows_differing": n_bad,
            "quotients_differing_from_div_full": int((probe.view(torch.int32)
                                                      != d.view(torch.int32)).sum().item())}
    return fix, info, q, s


ROW_CASES = {
    "f8_row_gauss_128x1536": (W.gaussian, dict(m=128, k=1536, seed=10)),
    "f8_row_studentt_64x8960": (W.student_t, dict(m=64, k=8960, seed=12)),
    "f8_row_outlier_16x8960": (W.with_outliers, dict(m=16, k=8960, seed=2)),
    "f8_row_edge_130x256": (W.edge_case_tensor, dict(m=130, k=256, seed=5)),
    "f8_row_weight_256x1536": (lambda m, k, seed: W.linear_params(m, k, seed=seed)[0],
                               dict(m=256, k=1536, seed=30)),
}
ROW_HASH_CASES = {
    "f8_hrow_outlier_1024x8960": (W.with_outliers, dict(m=1024, k=8960, seed=2)),
    "f8_hrow_gauss_4096x1536": (W.gaussian, dict(m=4096, k=1536, seed=13)),
}
TENSOR_CASES = {  # shapes of decoder / LQ activations (channels_last), small
    "f8_tensor_gauss_2x64x24x40": (W.gaussian, dict(m=2 * 24 * 40, k=64, seed=40)),
    "f8_tensor_outlier_3x48x20x36": (W.with_outliers, dict(m=3 * 20 * 36, k=48, seed=41)),
    "f8_tensor_edge_130x256": (W.edge_case_tensor, dict(m=130, k=256, seed=5)),
}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(ROOT / "tests" / "golden"))
    ap.add_argument("--time", default=None, help="also time the reference FP8 path; JSON path")
    args = ap.parse_args()
    out = Path(args.out)
    out.mkdir(parents=True, exist_ok=True)
    meta = {"torch": torch.__version__, "triton": triton.__version__,
            "device": torch.cuda.get_device_name(), "cases": {}}

    for name, (gen, kw) in ROW_CASES.items():
        xb = gen(**kw)
        fix, info, _, _ = row_fixture(xb)
        np.savez_compressed(out / f"{name}.npz", **fix)
        meta["cases"][name] = {"generator": getattr(gen, "__name__", "linear_params_weight"), **kw,
                               **info}
    for name, (gen, kw) in ROW_HASH_CASES.items():
        xb = gen(**kw)
        fix, info, q, s = row_fixture(xb, store_codes=False)
        np.savez_compressed(out / f"{name}.npz", **fix)
        meta["cases"][name] = {"generator": gen.__name__, **kw, **info, "q_sha256": sha(q),
                               "s_sha256": sha(s)}
    for name, (gen, kw) in TENSOR_CASES.items():
        xb = gen(**kw)                        # [pixels, channels]: channels_last memory order
        x = to_dev(xb)
        q, scale, d = ref_quantize_activation(x)
        xf = O.bf16_bits_to_f32(xb)
        a, b, qd, n_diff = code_changing_divisions(xf, np.float32(scale.item()), d.cpu().numpy(),
                                                   clamp=True)
        probe = fvq.ops.div_full_probe(torch.from_numpy(xf).cuda(), scale.expand(xf.shape))
        np.savez_compressed(out / f"{name}.npz", q=raw(q), scale_bits=u32(scale), div_a=a,
                            div_b=b, div_q=qd)
        meta["cases"][name] = {"generator": gen.__name__, **kw,
                               "quotients_differing_from_ieee": n_diff, "code_changing": len(a),
                               "quotients_differing_from_div_full": int(
                                   (probe.view(torch.int32) != d.view(torch.int32)).sum().item())}

    # ---- QuantLinear('fp8'): scaled_mm + bias
    wb, bb = W.linear_params(256, 1536, seed=30, b_std=0.01)
    xb = W.gaussian(200, 1536, seed=31)
    tables = []
    lin = RefFp8Linear(to_dev(wb), to_dev(bb), tables)
    keep = {}
    y = lin.forward(to_dev(xb), keep, tables)
    np.savez_compressed(out / "f8_lin_200x1536x256.npz", y=raw(y).view(np.uint16),
                        s_bits=u32(keep["s"].reshape(-1)), sw_bits=u32(lin.scale.reshape(-1)),
                        **merged(tables))
    meta["cases"]["f8_lin_200x1536x256"] = {"x": "gaussian(200,1536,seed=31)",
                                            "w": "linear_params(256,1536,seed=30,b_std=0.01)",
                                            "qweight_sha256": sha(lin.qweight),
                                            "scale_sha256": sha(lin.scale)}

    # ---- FFN, small (full output) and one layer at 7680 tokens (sampled rows)
    w1, b1 = W.linear_params(W.D_FF, W.D_MODEL, seed=20, b_std=0.01)
    w2, b2 = W.linear_params(W.D_MODEL, W.D_FF, seed=21, b_std=0.01)
    w_tables = []
    l1 = RefFp8Linear(to_dev(w1), to_dev(b1), w_tables)
    l2 = RefFp8Linear(to_dev(w2), to_dev(b2), w_tables)
    weights_meta = {"w1": "linear_params(8960,1536,seed=20,b_std=0.01)",
                    "w2": "linear_params(1536,8960,seed=21,b_std=0.01)",
                    "qweight1_sha256": sha(l1.qweight), "scale1_sha256": sha(l1.scale),
                    "qweight2_sha256": sha(l2.qweight), "scale2_sha256": sha(l2.scale)}
    xb = W.student_t(64, W.D_MODEL, seed=1)
    keep = {}
    tables = list(w_tables)
    y = ref_ffn(to_dev(xb), l1, l2, keep, tables)
    np.savez_compressed(out / "f8_ffn_64.npz", y=raw(y).view(np.uint16),
                        h=raw(keep["h"]).view(np.uint16), **merged(tables))
    meta["cases"]["f8_ffn_64"] = {"x": "student_t(64,1536,seed=1)", **weights_meta,
                                  "h_q_sha256": sha(keep["qh"]), "h_s_sha256": sha(keep["sh"])}
    xb = W.student_t(W.M_ONE_LAYER, W.D_MODEL, seed=1)
    y = ref_ffn(to_dev(xb), l1, l2)
    rows = np.sort(np.random.default_rng(99).choice(W.M_ONE_LAYER, 64, replace=False))
    np.savez_compressed(out / "f8_ffn_7680_rows.npz", rows=rows,
                        y_rows=raw(y[torch.from_numpy(rows).cuda()]).view(np.uint16))
    meta["cases"]["f8_ffn_7680_rows"] = {"x": "student_t(7680,1536,seed=1)", **weights_meta,
                                         "y_fro": float(y.float().norm().item()), "y_sha256": sha(y)}
    (out / "golden_fp8_meta.json").write_text(json.dumps(meta, indent=1, sort_keys=True))
    print("wrote", len(meta["cases"]), "cases to", out)

    if args.time:
        res = time_reference(l1, l2)
        Path(args.time).write_text(json.dumps(res, indent=1))
        print(json.dumps(res, indent=1))


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
    res = {"device": torch.cuda.get_device_name(), "torch": torch.__version__}
    m = W.M_ONE_LAYER
    x = torch.randn(m, W.D_MODEL, device="cuda", dtype=torch.bfloat16)
    ms = _time(lambda: ref_ffn(x, l1, l2))
    res["ref_fp8_ffn_layer_7680"] = {"ms": ms, "tokens_per_s": m / ms * 1e3,
                                     "TFLOPs": m * W.FLOP_PER_TOKEN / ms / 1e9}
    h = torch.randn(m, W.D_FF, device="cuda", dtype=torch.bfloat16)
    res["ref_row_quant_7680x8960_ms"] = _time(lambda: ref_row_quant(h, keep_quotients=False))
    q, s, _ = ref_row_quant(x, keep_quotients=False)
    res["scaled_mm_gemm1_7680x8960x1536_ms"] = _time(
        lambda: torch._scaled_mm(q, l1.qweight.t(), scale_a=s, scale_b=l1.scale.t(),
                                 out_dtype=torch.bfloat16, use_fast_accum=False))
    qh, sh, _ = ref_row_quant(h, keep_quotients=False)
    res["scaled_mm_gemm2_7680x1536x8960_ms"] = _time(
        lambda: torch._scaled_mm(qh, l2.qweight.t(), scale_a=sh, scale_b=l2.scale.t(),
                                 out_dtype=torch.bfloat16, use_fast_accum=False))
    return res


if __name__ == "__main__":
    t0 = time.time()
    main()
    print(f"done in {time.time() - t0:.1f}s")
