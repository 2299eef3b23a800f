"""One FFN layer at the 30-layer stack workloads' sizes and at their per-rank row blocks.

The stack workloads split 15360 tokens (four 48x80 latent frames, N(0,1), seed 3) and
64800 tokens (two 135x240 frames, Student-t(4) x 0.5, seed 4) over 1/2/4/8 GPUs into
contiguous row blocks: 15360 / 7680 / 3840 / 1920 and 64800 / 32400 / 16200 / 8100 rows.
Each block is "the reference run on that shard" (per-shard global scales), and these
sizes reach code paths that the 7680-token layer does not: a ragged last 128-row tile
(8100, 16200, 32400 and 64800 rows), GEMM2 row counts that are not multiples of 256
(1920, 8100), few row blocks per SM in GEMM1's resident schedule (1920 rows: 15), and the
cooperative X quantizer on small grids.

Checked here, per block:
* against the reference's own NVFP4 FFN (golden rows made by tests/golden/make_golden.py
  with FlashInfer's kernels on a B200): the 64 seeded rows bit for bit, the output's
  Frobenius norm within the 5e-3 relative tolerance, and the global scale of x;
* against the CPU oracle with this GPU's measured reciprocals, decomposed so that each
  half is pinned on its own: X quantization bit-exact on sampled rows; GEMM1 + bias +
  GELU rows (the sampled rows and the row holding max |h|) within the GEMM tolerance;
  amax(h) equal to the maximum of the intermediate; the second linear on the GPU's own
  intermediate rows within the GEMM tolerance.
"""
import numpy as np
import pytest
import torch

from flashvsr_optimizations_b200 import ops, workloads as W
from flashvsr_optimizations_b200.ffn_quantization import NVFP4FFN, QuantLinear
from helpers import bits_to_dev, dev_to_bits, f32_from_bits, golden, golden_meta, gpu_rcp_table
from oracle import nvfp4_oracle as O

pytestmark = pytest.mark.gpu

FFN_TOL = 5e-3    # Frobenius-relative bar against the reference FFN
GEMM_TOL = 2e-3   # GEMM vs the float64 oracle, Frobenius-relative
ULPS = 2          # and per element, in bf16 units of the larger magnitude

CASES = {"ffn_c4_15360": (W.gaussian, dict(m=W.M_STACK, k=W.D_MODEL, seed=3)),
         "ffn_c5_64800": (W.student_t, dict(m=W.M_4K, k=W.D_MODEL, seed=4))}
SHARDS = [("ffn_c4_15360", r) for r in W.STACK_SHARD_ROWS[W.M_STACK]] + \
         [("ffn_c5_64800", r) for r in W.STACK_SHARD_ROWS[W.M_4K]]


def _linear(wb, bb):
    out_f, in_f = wb.shape
    lin = torch.nn.Linear(in_f, out_f, bias=True, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(bits_to_dev(wb))
        lin.bias.copy_(bits_to_dev(bb))
    return QuantLinear(lin, "nvfp4")


@pytest.fixture(scope="module")
def layer0():
    w1, b1, w2, b2 = W.stack_layer_params(0)
    ffn = NVFP4FFN(_linear(w1, b1), torch.nn.GELU(approximate="tanh"), _linear(w2, b2))
    return ffn, (w1, b1, w2, b2)


@pytest.fixture(scope="module")
def inputs():
    return {name: gen(**kw) for name, (gen, kw) in CASES.items()}


@pytest.fixture(scope="module")
def oracle_layer(layer0):
    _, (w1, b1, w2, b2) = layer0
    l1 = O.OracleQuantLinear(w1, b1, gpu_rcp_table)
    l2 = O.OracleQuantLinear(w2, b2, gpu_rcp_table)
    w1d = O.dequantize(l1.qweight, l1.scale, W.D_FF, W.D_MODEL).astype(np.float64)
    w2d = O.dequantize(l2.qweight, l2.scale, W.D_MODEL, W.D_FF).astype(np.float64)
    return l1, l2, w1d, w2d


def _ulps_ok(got: np.ndarray, want: np.ndarray) -> bool:
    """Every element within ULPS bf16 ulps of the oracle (2^-8 relative per ulp), plus an
    absolute slack of 1e-6 of the largest magnitude (the GEMM tests' measure)."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    ulp = np.maximum(np.abs(want), 1e-30) * 2.0 ** -8
    worst = np.max(np.abs(got - want) / (ulp + 1e-6 * np.abs(want).max()))
    return bool(worst <= ULPS)


@pytest.mark.parametrize("case,rows", SHARDS)
def test_shard_matches_reference_rows(layer0, inputs, case, rows):
    """The reference FFN on this shard (FlashInfer, per-shard scales): sampled rows bit
    for bit, the norm within 5e-3, the same global scale of x."""
    ffn, _ = layer0
    name = f"{case}_rows{rows}"
    fix = golden(name)
    meta = golden_meta()["cases"].get(name)
    if meta is None:
        pytest.skip(f"golden case {name} missing")
    x = bits_to_dev(inputs[case][:rows])
    assert int(ops.global_scale(x).cpu().numpy().view(np.uint32)[0]) == int(fix["g1_bits"][0])
    y = ffn(x)
    got = dev_to_bits(y[torch.from_numpy(fix["rows"]).cuda()])
    diff = int((got != fix["y_rows"]).sum())
    rel = O.frobenius_rel(O.bf16_bits_to_f32(got), O.bf16_bits_to_f32(fix["y_rows"]))
    assert rel <= FFN_TOL, (name, rel)
    assert diff == 0, f"{name}: {diff} of {got.size} sampled output values differ from the reference"
    fro = float(y.float().norm().item())
    assert abs(fro - meta["y_fro"]) / meta["y_fro"] <= FFN_TOL, (fro, meta["y_fro"])


@pytest.mark.parametrize("case,rows", [("ffn_c4_15360", 1920), ("ffn_c4_15360", 3840),
                                       ("ffn_c5_64800", 8100), ("ffn_c5_64800", 16200),
                                       ("ffn_c5_64800", 32400)])
def test_shard_matches_oracle(layer0, oracle_layer, inputs, case, rows):
    ffn, _ = layer0
    l1, l2, w1d, w2d = oracle_layer
    xb = np.ascontiguousarray(inputs[case][:rows])
    x = bits_to_dev(xb)
    pick = np.sort(np.random.default_rng(1000 + rows).choice(rows, 12, replace=False))
    pick = np.unique(np.concatenate([pick, [rows - 1]]))   # the ragged last tile's last row

    # X: global scale and codes of the sampled rows, bit-exact
    g_x = ops.global_scale(x)
    g_x_ref = O.global_scale(xb)
    assert f32_from_bits(g_x.cpu().numpy().view(np.uint32)) == g_x_ref
    q, s = ops.nvfp4_quantize(x, g_x)
    table_x = gpu_rcp_table(xb, g_x_ref)
    q_ref, s_ref = O.nvfp4_quantize(xb[pick], g_x_ref, rcp_table=table_x)
    assert np.array_equal(q[torch.from_numpy(pick).cuda()].cpu().numpy(), q_ref)
    sf_gpu = O.unswizzle_sf(s.cpu().numpy().reshape(-1), rows, W.D_MODEL)[pick]
    assert np.array_equal(sf_gpu, O.unswizzle_sf(s_ref, len(pick), W.D_MODEL))

    # GEMM1 + bias + GELU (+ amax of h): the same kernel as inside the FFN
    q1, q2 = ffn[0], ffn[2]
    h, amax_h = ops.nvfp4_gemm(q, s, g_x, q1.qweight, q1.scale, q1.global_sf, q1.bias, gelu=True)
    hmax = h.float().abs().max()
    assert float(amax_h.item()) == float(hmax.item())
    arg = int(h.float().abs().amax(dim=1).argmax().item())
    rows_h = np.unique(np.concatenate([pick, [arg]]))
    qa, sa = O.nvfp4_quantize(xb[rows_h], g_x_ref, rcp_table=table_x)
    alpha1 = O.gemm_alpha(g_x_ref, l1.global_sf)
    acc = O.dequantize(qa, sa, len(rows_h), W.D_MODEL).astype(np.float64) @ w1d.T
    h_ref = O.gelu_tanh_bf16(O.bias_add_bf16(O.round_bf16(alpha1 * acc.astype(np.float32)), l1.bias))
    h_gpu = O.bf16_bits_to_f32(dev_to_bits(h[torch.from_numpy(rows_h).cuda()]))
    assert O.frobenius_rel(h_gpu, h_ref) <= GEMM_TOL
    assert _ulps_ok(h_gpu, h_ref)

    # the second linear on the GPU's own intermediate rows, with the GPU's amax(h)
    g_h = O.global_scale_from_amax(np.float32(amax_h.item()))
    hb = dev_to_bits(h[torch.from_numpy(pick).cuda()])
    table_h = gpu_rcp_table(hb, g_h)
    qh, sh = O.nvfp4_quantize(hb, g_h, rcp_table=table_h)
    alpha2 = O.gemm_alpha(g_h, l2.global_sf)
    acc2 = O.dequantize(qh, sh, len(pick), W.D_FF).astype(np.float64) @ w2d.T
    y_ref = O.bias_add_bf16(O.round_bf16(alpha2 * acc2.astype(np.float32)), l2.bias)
    y = ffn(x)
    y_gpu = O.bf16_bits_to_f32(dev_to_bits(y[torch.from_numpy(pick).cuda()]))
    assert O.frobenius_rel(y_gpu, y_ref) <= GEMM_TOL, O.frobenius_rel(y_gpu, y_ref)
    assert _ulps_ok(y_gpu, y_ref)

    # the fused call is the composition of the steps just checked
    qh_full, sh_full, gh_full = ops.nvfp4_quantize_from_amax(h, amax_h)
    y_comp, _ = ops.nvfp4_gemm(qh_full, sh_full, gh_full, q2.qweight, q2.scale, q2.global_sf,
                               q2.bias, gelu=False)
    assert torch.equal(y, y_comp)
