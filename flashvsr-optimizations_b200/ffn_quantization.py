"""Drop-in replacement of the reference's ``ffn_quantization.py`` (NVFP4 and FP8 modes).

Same plugin API as the reference (ffn_quantization.py:35-86):

* ``global_scale(x)`` -> fp32 [1] encode scale ``2688 / max(amax(x), 1e-12)``;
* ``QuantLinear(linear, mode)`` with buffers ``qweight``, ``scale``,
  ``global_sf``, ``bias`` and attribute ``out_features``; ``forward`` maps
  bf16 ``[..., K]`` -> bf16 ``[..., N]`` on the current CUDA stream, without a
  host synchronisation;
* ``install_ffn(pipe, mode)`` swaps ``pipe.dit.blocks[i].ffn[0]`` and
  ``ffn[2]`` and returns the same metadata dict.

Additionally ``install_ffn`` (``fused=True``, the default) replaces each
block's ``ffn`` ``nn.Sequential`` by :class:`NVFP4FFN` (or :class:`FP8FFN`), a
subclass that keeps the same children (``[0]`` and ``[2]`` are the
``QuantLinear`` modules, ``[1]`` the GELU) but runs the whole
Linear-GELU-Linear chain as one call into the library, with GELU and the
intermediate's amax (per tensor for NVFP4, per row for FP8) computed in
GEMM1's epilogue.  Its result follows the reference's roundings and scales
exactly.

Modes: ``'nvfp4'`` (E2M1 W4A4, ffn_quantization.py:47-48, :62-67), ``'fp8'``
(E4M3 W8A8 with per-row scales, :44-46, :57-60), ``'bf16'`` (no swap).  Any
other mode raises ``ValueError(mode)`` like the reference
(ffn_quantization.py:50).
"""
from __future__ import annotations

import torch

from . import ops
from ._lib import load as load_library

__all__ = ["global_scale", "row_quant", "QuantLinear", "NVFP4FFN", "NVFP4FFNStack", "GraphedFFNStack",
           "FP8FFN", "install_ffn"]


def global_scale(x: torch.Tensor) -> torch.Tensor:
    """ffn_quantization.py:29-32."""
    return ops.global_scale(x.contiguous())


def row_quant(x: torch.Tensor):
    """ffn_quantization.py:22-26: (float8_e4m3fn [M, K], fp32 [M, 1] row scales)."""
    return ops.fp8_row_quant(x.contiguous())


def _quantize_weight(w: torch.Tensor):
    w = w.detach().to(torch.bfloat16).contiguous()
    g = ops.global_scale(w)
    q, s = ops.nvfp4_quantize(w, g)
    return q, s, g


class QuantLinear(torch.nn.Module):
    """W4A4 (``'nvfp4'``) or W8A8 (``'fp8'``) replacement of one ``nn.Linear``
    (ffn_quantization.py:35-70)."""

    def __init__(self, linear: torch.nn.Linear, mode: str):
        super().__init__()
        self.mode = mode
        self.out_features = linear.out_features
        self.in_features = linear.in_features
        bias = linear.bias.detach().clone().to(torch.bfloat16) if linear.bias is not None else None
        self.register_buffer("bias", bias)
        if mode not in ("fp8", "nvfp4"):
            raise ValueError(mode)
        w = linear.weight
        if not w.is_cuda:
            raise RuntimeError("QuantLinear: the weight must be on a CUDA device (no CPU path)")
        if mode == "fp8":
            q, s = row_quant(w.detach().to(torch.bfloat16))
        else:
            q, s, g = _quantize_weight(w)
            self.register_buffer("global_sf", g)
        self.register_buffer("qweight", q)
        self.register_buffer("scale", s)

    @classmethod
    def from_quantized(cls, qweight: torch.Tensor, scale: torch.Tensor, global_sf: torch.Tensor,
                       bias: torch.Tensor | None, in_features: int) -> "QuantLinear":
        """Build from already-quantized buffers (e.g. a saved state dict), no re-quantization."""
        self = cls.__new__(cls)
        torch.nn.Module.__init__(self)
        self.mode = "nvfp4"
        self.in_features = in_features
        self.out_features = qweight.shape[0]
        if qweight.shape[1] * 2 != in_features:
            raise ValueError("QuantLinear.from_quantized: qweight does not match in_features")
        self.register_buffer("bias", bias)
        self.register_buffer("global_sf", global_sf)
        self.register_buffer("qweight", qweight)
        self.register_buffer("scale", scale)
        return self

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        if self.mode == "fp8":
            out = ops.fp8_linear(x2, self.qweight, self.scale, self.bias)
        else:
            out = ops.nvfp4_linear(x2, self.qweight, self.scale, self.global_sf, self.bias)
        return out.reshape(*shape[:-1], self.out_features)

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, mode={self.mode}"


class NVFP4FFN(torch.nn.Sequential):
    """``nn.Sequential(QuantLinear, GELU(tanh), QuantLinear)`` run as one fused call.

    Indexing, iteration and state-dict keys are those of the Sequential it
    replaces; ``forward`` computes exactly what the Sequential of QuantLinear
    modules would, in four kernel launches (amax + quantize of x, GEMM1 with bias,
    GELU and the amax of the intermediate, quantize of the intermediate, GEMM2 with
    bias).
    """

    H_SCALINGS = ("exact", "static", "delayed")

    def __init__(self, lin1: QuantLinear, act: torch.nn.Module, lin2: QuantLinear):
        super().__init__(lin1, act, lin2)
        if lin1.out_features != lin2.in_features or lin2.out_features != lin1.in_features:
            raise ValueError("NVFP4FFN: linear shapes do not chain")
        self.h_scaling = "exact"
        self.headroom_log2 = 0
        self.rerun_on_saturation = False
        self._h_state = None      # fp32 [2]: the hint and the amax seen (swapped per call)
        self._h_flags = None      # int32 [1]
        self._h_turn = 0
        self._h_seeded = False

    def set_h_scaling(self, mode: str = "exact", amax=None, headroom_log2: int | None = None,
                      rerun_on_saturation: bool = False) -> "NVFP4FFN":
        """How the intermediate h = GELU(linear1(x)) is scaled for its NVFP4 quantization.

        * ``"exact"`` (default): the reference's scale 2688 / amax(h) of the whole tensor
          (ffn_quantization.py:63-64).  amax(h) is known only after GEMM1 has finished, so h
          makes one bf16 round trip through HBM (four launches); the output equals the
          reference's bit for bit.
        * ``"static"``: GEMM1's epilogue quantizes h itself with a provisional scale from
          `amax`, a calibrated estimate of max |h|: no bf16 intermediate, three launches.
        * ``"delayed"``: the same, with the max |h| the previous call saw as the estimate
          (its first call runs the exact path to seed it); default headroom 2x.

        The provisional scale differs from the exact one by other than a power of two, so
        the intermediate is quantized differently from the reference (the same number
        format and recipe, another scale grid): as close to the unquantized FFN as the
        reference is, not bit-identical to it.  A block whose scale saturates (h above
        hint x 2^headroom_log2) sets bit 0 of the device flags (``h_flags()``); with
        `rerun_on_saturation` the call then reads the flag (a host synchronisation) and
        reruns the exact path.
        """
        if mode not in self.H_SCALINGS:
            raise ValueError(mode)
        self.h_scaling = mode
        self.headroom_log2 = (1 if mode == "delayed" else 0) if headroom_log2 is None else int(headroom_log2)
        self.rerun_on_saturation = bool(rerun_on_saturation)
        dev = self[0].qweight.device
        self._h_state = torch.zeros(2, dtype=torch.float32, device=dev)
        self._h_flags = torch.zeros(1, dtype=torch.int32, device=dev)
        self._h_turn = 0
        self._h_seeded = False
        if mode == "static":
            if amax is None:
                raise ValueError("static h scaling needs amax (an estimate of max |h|)")
            self._h_state[0] = torch.as_tensor(amax, dtype=torch.float32).reshape(())
            self._h_seeded = True
        return self

    def h_flags(self, clear: bool = True) -> int:
        """The provisional-scale flags of the calls so far (1 saturated, 2 underflowed);
        reads the device (a host synchronisation)."""
        if self._h_flags is None:
            return 0
        v = int(self._h_flags.item())
        if clear:
            self._h_flags.zero_()
        return v

    def _exact_with_amax(self, x2: torch.Tensor):
        """The exact path as separate launches, returning max |h| as well (the same bits as
        fvq_nvfp4_ffn)."""
        l1, l2 = self[0], self[2]
        g = ops.global_scale(x2)
        q, s = ops.nvfp4_quantize(x2, g)
        h, amax_h = ops.nvfp4_gemm(q, s, g, l1.qweight, l1.scale, l1.global_sf, l1.bias, gelu=True)
        qh, sh, gh = ops.nvfp4_quantize_from_amax(h, amax_h)
        y, _ = ops.nvfp4_gemm(qh, sh, gh, l2.qweight, l2.scale, l2.global_sf, l2.bias, gelu=False)
        return y, amax_h

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        l1, l2 = self[0], self[2]
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        if self.h_scaling == "exact":
            y = ops.nvfp4_ffn(x2, l1.qweight, l1.scale, l1.global_sf, l1.bias,
                              l2.qweight, l2.scale, l2.global_sf, l2.bias)
        elif not self._h_seeded:
            y, amax_h = self._exact_with_amax(x2)
            self._h_state[0:1].copy_(amax_h)
            self._h_turn = 0
            self._h_seeded = True
        else:
            t = self._h_turn
            hint, seen = self._h_state[t:t + 1], self._h_state[1 - t:2 - t]
            y = ops.nvfp4_ffn_fused(x2, l1.qweight, l1.scale, l1.global_sf, l1.bias,
                                    l2.qweight, l2.scale, l2.global_sf, l2.bias,
                                    hint, self.headroom_log2, seen, self._h_flags)
            if self.h_scaling == "delayed":
                self._h_turn = 1 - t
            if self.rerun_on_saturation and self.h_flags(clear=False) & 1:
                self._h_flags.zero_()
                y, amax_h = self._exact_with_amax(x2)
                if self.h_scaling == "delayed":
                    self._h_state[self._h_turn:self._h_turn + 1].copy_(amax_h)
        return y.reshape(*shape[:-1], l2.out_features)

    def chained(self, x: torch.Tensor, x_amax: torch.Tensor | None = None):
        """(self(x), max |self(x)|) for a stack of FFNs that feed each other directly:
        x_amax, max |x| as the previous FFN's ``chained`` returned it, spares this call its
        own pass over x for the global scale (fvq_nvfp4_ffn_chain).  The exact h scaling
        only; the output equals ``self(x)`` bit for bit."""
        l1, l2 = self[0], self[2]
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        y, y_amax = ops.nvfp4_ffn_chain(x2, l1.qweight, l1.scale, l1.global_sf, l1.bias,
                                        l2.qweight, l2.scale, l2.global_sf, l2.bias, x_amax)
        return y.reshape(*shape[:-1], l2.out_features), y_amax

    def modulated(self, x: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor,
                  gate: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
        """The DiT block's FFN step around this module: x + gate * self(LN(x) * (1 + scale) +
        shift), LN without affine, each elementwise step in bf16 as torch rounds it; one library
        call (the LayerNorm and modulation in one kernel, the gated residual in the second
        GEMM's epilogue).  shift, scale, gate: bf16 vectors of d_model values."""
        l1, l2 = self[0], self[2]
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        y = ops.nvfp4_ffn_block(x2, shift, scale, gate, eps, l1.qweight, l1.scale, l1.global_sf,
                                l1.bias, l2.qweight, l2.scale, l2.global_sf, l2.bias)
        return y.reshape(shape)


class NVFP4FFNStack(torch.nn.ModuleList):
    """FFNs applied one after another, y = ffn_L(...ffn_1(x)), each NVFP4FFN handing the
    next the max |y| its second GEMM's epilogue already computed (``NVFP4FFN.chained``), so
    only the first quantizes its input with a separate amax pass.  The output equals running
    the modules one by one, bit for bit.  The FFN-only stack of the 30-layer benchmark
    workloads; the DiT pipeline itself puts attention between its FFNs."""

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        amax = None
        for ffn in self:
            x, amax = ffn.chained(x, amax)
        return x

    def graphed(self, x: torch.Tensor) -> "GraphedFFNStack":
        """This stack over the tensor ``x`` (a fixed buffer the caller refills), captured once
        into a CUDA graph: see :class:`GraphedFFNStack`."""
        return GraphedFFNStack(self, x)


class GraphedFFNStack:
    """An :class:`NVFP4FFNStack` over one input buffer, its launches (four per FFN) captured
    once into a CUDA graph and replayed: ``g()`` runs every layer on the current contents of
    the buffer given at capture, on the current CUDA stream, and returns the output tensor
    (the same tensor each time, overwritten by each replay).  No host work per layer (the
    30-layer stack at 1920 rows: 1.68 ms issued launch by launch, 1.64 ms replayed); the
    output equals ``stack(x)`` bit for bit.  The buffer, the weights and the library workspace the
    capture used stay referenced while this object lives.  Shapes are fixed: a new row count
    needs a new capture."""

    def __init__(self, stack: NVFP4FFNStack, x: torch.Tensor):
        if not x.is_cuda or x.dtype != torch.bfloat16 or not x.is_contiguous():
            raise ValueError("GraphedFFNStack: x must be a contiguous bf16 CUDA tensor")
        self.stack, self.x = stack, x
        dev = x.device
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.no_grad(), torch.cuda.stream(side):
            # warm-up on the capture stream: per-context kernel attributes and symbol
            # addresses are looked up once, and the library workspace of this stream is
            # allocated outside the capture (it must outlive the graph)
            for _ in range(2):
                stack(x)
            m = x.numel() // x.shape[-1]
            lin1 = stack[0][0]
            nbytes = load_library().fvq_nvfp4_ffn_workspace_bytes(m, lin1.in_features,
                                                                   lin1.out_features)
            self.workspace = ops.workspace(dev, nbytes)
        torch.cuda.current_stream(dev).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.no_grad(), torch.cuda.graph(self.graph, stream=side):
            self.out = stack(x)

    def __call__(self) -> torch.Tensor:
        self.graph.replay()
        return self.out


class FP8FFN(torch.nn.Sequential):
    """``nn.Sequential(QuantLinear('fp8'), GELU(tanh), QuantLinear('fp8'))`` run as one fused call.

    Same contract as :class:`NVFP4FFN`: the children and state-dict keys of
    the Sequential it replaces, and exactly the result of running them one
    after another (four kernel launches instead of seven).
    """

    def __init__(self, lin1: QuantLinear, act: torch.nn.Module, lin2: QuantLinear):
        super().__init__(lin1, act, lin2)
        if lin1.mode != "fp8" or lin2.mode != "fp8":
            raise ValueError("FP8FFN: both linears must be QuantLinear(mode='fp8')")
        if lin1.out_features != lin2.in_features or lin2.out_features != lin1.in_features:
            raise ValueError("FP8FFN: linear shapes do not chain")

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        l1, l2 = self[0], self[2]
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        y = ops.fp8_ffn(x2, l1.qweight, l1.scale, l1.bias, l2.qweight, l2.scale, l2.bias)
        return y.reshape(*shape[:-1], l2.out_features)


_FUSED = {"nvfp4": NVFP4FFN, "fp8": FP8FFN}


def _is_gelu_tanh(m: torch.nn.Module) -> bool:
    return isinstance(m, torch.nn.GELU) and getattr(m, "approximate", "none") == "tanh"


def install_ffn(pipe, mode: str, fused: bool = True) -> dict:
    """ffn_quantization.py:73-86, plus the fused whole-FFN module when ``fused``."""
    count = 0
    before = sum(p.numel() * p.element_size() for b in pipe.dit.blocks for p in b.ffn.parameters())
    fused_blocks = 0
    if mode != "bf16":
        for block in pipe.dit.blocks:
            for idx in (0, 2):
                block.ffn[idx] = QuantLinear(block.ffn[idx], mode)
                count += 1
            if fused and len(block.ffn) == 3 and _is_gelu_tanh(block.ffn[1]):
                block.ffn = _FUSED[mode](block.ffn[0], block.ffn[1], block.ffn[2])
                fused_blocks += 1
    after = sum(t.numel() * t.element_size() for b in pipe.dit.blocks
                for t in list(b.ffn.parameters()) + list(b.ffn.buffers()))
    return {
        "mode": mode, "quantized_linears": count, "ffn_bytes_before": before,
        "ffn_bytes_after": after,
        "fp8": ("E4M3 per-row W8A8; sm_100a tcgen05 kind::f8f6f4 GEMM with row-wise scales "
                "(libfvq); FP32 accumulation; BF16 output"),
        "nvfp4": ("E2M1 W4A4; 16-element E4M3 scales + dynamic tensor FP32 scale; sm_100a "
                  "tcgen05 block-scaled GEMM (libfvq); BF16 output"),
        "scope": "Only dit.blocks.*.ffn.{0,2}; GELU, bias, attention, conditioning, decoder remain BF16",
        "fused_ffn_blocks": fused_blocks,
    }
