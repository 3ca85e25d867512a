"""NF4Linear: frozen linear layer with an NF4 weight, computed by the fused kernels.

Drop-in for the reference's ``stratum.nf4_linear.NF4Linear``
(stratum/nf4_linear.py:17-47): same constructor ``NF4Linear(quantized,
quant_state, bias=None)``, same ``in_features`` / ``out_features``
(``quant_state.shape[1]`` / ``[0]``), same forward semantics
``F.linear(x, dequantize_4bit(quantized, quant_state), bias)``.  The reference
materialises the dequantized weight and calls cuBLAS; here the dequantization
happens inside the GEMM's mainloop and the weight never exists in HBM.

The reference pairs the frozen base layer with PEFT's ``lora.Linear``
(scripts/train.py:568-573: ``y = base(x) + scaling * B(A(x))``, dropout 0).
:meth:`NF4Linear.attach_lora` adds that adapter to this module, and the
low-rank update is folded into the same tensor-core accumulator (forward) and
the same fused input-gradient kernel (backward).  The weight is frozen: the
backward produces dX (and dA, dB for the adapter), never dW.
"""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn as nn

from . import ops
from .functional import QuantState, dequantize_4bit


class _NF4LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, lora_A, lora_B, packed, qs, bias, scaling):
        xa = None
        if lora_A is not None:
            x2 = x.reshape(-1, x.shape[-1])
            xa = ops.lora_down(x2, lora_A.to(x.dtype), scaling)
        y = ops.nf4_gemm_fwd(x, packed, qs, bias=bias, lora_A=lora_A, lora_B=lora_B, scaling=scaling, xa=xa)
        ctx.qs = qs
        ctx.scaling = scaling
        ctx.has_lora = lora_A is not None
        ctx.save_for_backward(x if lora_A is not None else None, xa, lora_A, lora_B, packed)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, xa, lora_A, lora_B, packed = ctx.saved_tensors
        qs, scaling = ctx.qs, ctx.scaling
        N = int(qs.shape[0])
        dy = dy.contiguous()
        dx = dA = dB = None
        if ctx.has_lora:
            dy2 = dy.reshape(-1, N)
            r = lora_A.shape[0]
            dyb = ops.lora_down(dy2, lora_B.t().to(dy.dtype), scaling)  # scaling * dy . B, padded
            if ctx.needs_input_grad[0]:
                dx = ops.nf4_gemm_dx(dy, packed, qs, lora_A=lora_A, lora_B=lora_B, scaling=scaling, dyb=dyb)
            x2 = x.reshape(-1, x.shape[-1])
            if ctx.needs_input_grad[1]:
                dA = (dyb[:, :r].t() @ x2).to(lora_A.dtype)  # scaling * B^T dy^T x
            if ctx.needs_input_grad[2]:
                dB = (dy2.t() @ xa[:, :r]).to(lora_B.dtype)  # dy^T (scaling * x A^T)
        elif ctx.needs_input_grad[0]:
            dx = ops.nf4_gemm_dx(dy, packed, qs)
        return dx, dA, dB, None, None, None, None


class NF4Linear(nn.Module):
    """Frozen Linear layer whose weight stays NF4 on the GPU.

    Args mirror the reference: ``quantized`` (packed uint8 payload),
    ``quant_state`` (:class:`~stratum_b200.functional.QuantState` with
    ``.shape == (out_features, in_features)``), optional frozen ``bias``.
    """

    def __init__(self, quantized: Optional[torch.Tensor], quant_state: Optional[QuantState],
                 bias: Optional[torch.Tensor] = None):
        super().__init__()
        self.quantized = quantized
        self.quant_state = quant_state
        if bias is not None:
            self.bias = nn.Parameter(bias.contiguous(), requires_grad=False)
        else:
            self.bias = None
        if quant_state is not None:
            self.in_features = quant_state.shape[1]
            self.out_features = quant_state.shape[0]
        self.lora_A: Optional[nn.Parameter] = None
        self.lora_B: Optional[nn.Parameter] = None
        self.scaling = 1.0
        self.streamed = False

    @classmethod
    def streamed_from(cls, weight: nn.Parameter, payload, bias: Optional[torch.Tensor] = None) -> "NF4Linear":
        """Fused-mode layer fed by the streaming contract (ensure_weights / free_weights).

        ``weight`` is the frozen placeholder parameter that carries the NF4
        payload (``stratum_b200.upload.NF4_ATTR``); ``ensure_weights`` uploads
        the packed bytes into this layer and ``free_weights`` drops them.
        """
        m = cls(None, None, bias=None)
        m.weight = weight
        weight.requires_grad_(False)
        if bias is not None:
            m.bias = bias if isinstance(bias, nn.Parameter) else nn.Parameter(bias, requires_grad=False)
            m.bias.requires_grad_(False)
        m.in_features = int(payload.shape[1])
        m.out_features = int(payload.shape[0])
        m.streamed = True
        return m

    def load_device_state(self, quantized: torch.Tensor, quant_state: QuantState) -> None:
        self.quantized = quantized
        self.quant_state = quant_state

    def device_state_on(self, device: torch.device) -> bool:
        return self.quantized is not None and self.quantized.device == device

    def drop_device_state(self) -> bool:
        had = self.quantized is not None
        self.quantized = None
        self.quant_state = None
        return had

    def attach_lora(self, r: int, alpha: float, dtype=torch.bfloat16, init_B_zero: bool = True,
                    device=None) -> "NF4Linear":
        """Add a PEFT-style adapter: A kaiming-uniform(a=sqrt 5) [r, in], B zeros [out, r], scaling alpha/r."""
        dev = device if device is not None else (self.quantized.device if self.quantized is not None else "cpu")
        A = torch.empty(r, self.in_features, dtype=torch.float32, device=dev)
        nn.init.kaiming_uniform_(A, a=math.sqrt(5))
        B = torch.zeros(self.out_features, r, dtype=torch.float32, device=dev)
        if not init_B_zero:
            nn.init.normal_(B, std=0.01)
        self.lora_A = nn.Parameter(A.to(dtype))
        self.lora_B = nn.Parameter(B.to(dtype))
        self.scaling = float(alpha) / float(r)
        return self

    @property
    def weight_dequantized(self) -> torch.Tensor:
        """The dequantized weight (materialised; for inspection and tests)."""
        return dequantize_4bit(self.quantized, self.quant_state)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.quantized is None:
            raise RuntimeError("NF4Linear: weights are not resident on the device; call ensure_weights() first")
        return _NF4LinearFn.apply(x, self.lora_A, self.lora_B, self.quantized, self.quant_state, self.bias,
                                  self.scaling)

    def extra_repr(self) -> str:
        lora = f", lora_r={self.lora_A.shape[0]}, scaling={self.scaling:g}" if self.lora_A is not None else ""
        return f"in_features={self.in_features}, out_features={self.out_features}, bias={self.bias is not None}{lora}"
