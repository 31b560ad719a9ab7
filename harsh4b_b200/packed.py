"""Operator-level drop-in for the reference's PackedLinear (packed_linear.py:
92-106): ``PackedInt4Linear`` keeps a row-scaled packed int4 matrix in HBM
and computes ``x @ W.T (+ bias)`` for any input dtype and leading shape.

Like the reference module, the single-token case goes through a GEMV chosen
from a kernel registry (``KERNELS`` / ``KERNEL`` / ``set_kernel``,
packed_linear.py:20-28); ``"b200_int4"`` is this backend's fused
quantise + int4 GEMV. Each token's activation is quantised to int8 with its
own absmax scale (the reference CPU path's per-token contract), so a batch of
tokens gives exactly the rows the GEMV gives one token at a time.
"""
from __future__ import annotations

import torch

from . import ops


def _b200_int4(x: torch.Tensor, p: dict, bias: torch.Tensor | None = None) -> torch.Tensor:
    """One token: fp32 x[K] -> fp32 y[N] (quantise + int4 GEMV in one kernel)."""
    out, _, _ = ops.int4_gemv_fused_quant(x.reshape(-1).to(torch.float32).contiguous(), p["weights"], p["scales"])
    return out + bias if bias is not None else out


KERNELS = {"b200_int4": _b200_int4}
KERNEL = [_b200_int4]


def set_kernel(name: str) -> None:
    KERNEL[0] = KERNELS[name]


class PackedInt4Linear(torch.nn.Module):
    """y = x @ W.T + b with W = int4 codes (uint8[N, K/2], low nibble = even k)
    times fp32 row scales; x is quantised per token to int8 on the device."""

    def __init__(self, weights: torch.Tensor, scales: torch.Tensor, bias: torch.Tensor | None = None):
        super().__init__()
        if weights.dtype != torch.uint8 or weights.dim() != 2:
            raise ValueError("weights must be uint8[N, K/2]")
        if scales.dtype != torch.float32 or scales.shape != (weights.shape[0],):
            raise ValueError("scales must be float32[N]")
        if not weights.is_cuda or not scales.is_cuda:
            raise ValueError("PackedInt4Linear runs on the GPU only (harsh4b_b200 has no CPU fallback)")
        self.OC, self.IC = weights.shape[0], 2 * weights.shape[1]
        self.register_buffer("weights", weights.contiguous(), persistent=False)
        self.register_buffer("scales", scales.contiguous(), persistent=False)
        if bias is not None:
            self.register_buffer("bias", bias.to(torch.float32).contiguous(), persistent=False)
        else:
            self.bias = None

    def _p(self) -> dict:
        return {"weights": self.weights, "scales": self.scales, "shape": (self.OC, self.IC)}

    @torch.no_grad()
    def dequant(self) -> torch.Tensor:
        """W as fp32 [OC, IC] (testing aid)."""
        signed = self.weights.view(torch.int8)
        low = (signed << 4) >> 4
        high = signed >> 4
        codes = torch.stack([low, high], dim=-1).reshape(self.OC, self.IC).to(torch.float32)
        return codes * self.scales[:, None]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.shape[-1] != self.IC:
            raise ValueError(f"expected {self.IC} input features, got {x.shape[-1]}")
        in_dtype, lead = x.dtype, x.shape[:-1]
        rows = x.reshape(-1, self.IC).to(torch.float32).contiguous()
        if rows.shape[0] == 1:
            out = KERNEL[0](rows[0], self._p(), self.bias).reshape(1, self.OC)
        else:
            out = ops.int4_gemm_rows(rows, self.weights, self.scales)
            if self.bias is not None:
                out = out + self.bias
        return out.reshape(*lead, self.OC).to(in_dtype)
