"""Helpers shared by the tests (fixture loading, device transfer, rcp tables)."""
from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import GOLDEN


def golden_meta() -> dict:
    p = GOLDEN / "golden_meta.json"
    if not p.exists():
        pytest.skip("golden fixtures not generated yet (tests/golden/make_golden.py on a B200)")
    return json.loads(p.read_text())


def golden(name: str) -> dict:
    p = GOLDEN / f"{name}.npz"
    if not p.exists():
        pytest.skip(f"golden fixture {name} missing")
    with np.load(p) as z:
        return {k: z[k] for k in z.files}


def table_from(args: np.ndarray, res: np.ndarray) -> dict:
    return dict(zip(np.asarray(args, dtype=np.uint32).tolist(),
                    np.asarray(res, dtype=np.uint32).tolist()))


def f32_from_bits(b) -> np.float32:
    return np.asarray(b, dtype=np.uint32).view(np.float32).reshape(-1)[0]


def bits_to_dev(bits: np.ndarray):
    import torch
    return torch.from_numpy(np.ascontiguousarray(bits).astype(np.int16)).view(torch.bfloat16).cuda()


def dev_to_bits(t) -> np.ndarray:
    import torch
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def gpu_rcp_table(x_bits: np.ndarray, g: float) -> dict:
    """rcp.approx.ftz.f32 measured on the GPU for every argument the oracle needs."""
    import torch
    from oracle import nvfp4_oracle as O
    import flashvsr_optimizations_b200 as fvq
    args = np.array(O.rcp_arguments(x_bits, g), dtype=np.uint32)
    res = fvq.ops.rcp_approx_probe(torch.from_numpy(args.view(np.float32)).cuda())
    return table_from(args, res.cpu().numpy().view(np.uint32))
