"""NF4Experts: routed expert MLPs whose frozen weights stay NF4 on the GPU.

Drop-in for HF ``Qwen3MoeExperts`` (transformers' modeling_qwen3_moe.py) as the
reference runs it: the 3-D frozen parameters ``gate_up_proj [E, 2I, H]`` and
``down_proj [E, H, I]`` are NF4-staged flattened to ``[-1, last]``
(stratum/upload.py:361-366) and, in the reference, dequantized in full before
the per-expert cuBLAS loop.  Same call: ``forward(hidden_states, top_k_index,
top_k_weights)``; same result::

    for each expert e:  h = silu(x_e . Wgu[e][:I]^T) * (x_e . Wgu[e][I:]^T)
                        out[tokens_e] += (h . Wd[e]^T) * top_k_weights

computed as: route (counting sort by expert) -> gather -> one grouped NF4 GEMM
with the SwiGLU epilogue -> one grouped NF4 GEMM -> weighted combine.  The
expert weights are frozen and not LoRA targets (the reference's PEFT config
targets module names ending in ``proj``, scripts/train.py:557-566), so the
backward produces the input gradient and the routing-weight gradient only.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from . import ops
from .functional import QuantState, dequantize_4bit, quantize_4bit


class _NF4ExpertsFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden, top_k_weights, routing, gu_packed, gu_qs, d_packed, d_qs):
        T, H = hidden.shape
        x_sorted = ops.moe_gather_rows(hidden, routing.token_of)
        if ctx.needs_input_grad[0]:  # the input gradient needs gate|up for the SwiGLU backward
            h, gu = ops.nf4_grouped_fwd(x_sorted, routing, gu_packed, gu_qs, swiglu=True, keep_gate_up=True)
        else:
            h, gu = ops.nf4_grouped_fwd(x_sorted, routing, gu_packed, gu_qs, swiglu=True), None
        o = ops.nf4_grouped_fwd(h, routing, d_packed, d_qs)
        w = top_k_weights.reshape(-1).to(torch.float32).contiguous()
        out = ops.moe_combine(o, routing, w)
        ctx.routing = routing
        ctx.qs = (gu_qs, d_qs)
        ctx.w_dtype = top_k_weights.dtype
        ctx.w_shape = top_k_weights.shape
        ctx.save_for_backward(w, gu, o if ctx.needs_input_grad[1] else None, gu_packed, d_packed)
        return out

    @staticmethod
    def backward(ctx, dout):
        w, gu, o, gu_packed, d_packed = ctx.saved_tensors
        routing = ctx.routing
        gu_qs, d_qs = ctx.qs
        dout = dout.contiguous()
        dy_sorted, dw = ops.moe_combine_grad(dout, routing, w, o)
        dhidden = None
        if ctx.needs_input_grad[0]:
            dh = ops.nf4_grouped_dx(dy_sorted, routing, d_packed, d_qs)
            dgu = ops.swiglu_grad(gu, dh)
            dx_sorted = ops.nf4_grouped_dx(dgu, routing, gu_packed, gu_qs)
            dhidden = ops.moe_combine(dx_sorted, routing, None)
        dweights = dw.view(ctx.w_shape).to(ctx.w_dtype) if dw is not None else None
        return dhidden, dweights, None, None, None, None, None


class NF4Experts(nn.Module):
    """Frozen routed experts with NF4 weights, computed by the grouped kernels.

    ``gate_up`` / ``down`` are the packed NF4 bytes of the flattened
    ``[E*2I, H]`` / ``[E*H, I]`` weights with their :class:`QuantState`\\ s
    (shapes ``(E*2I, H)`` / ``(E*H, I)``, blocksize 64).  ``hidden_act`` must be
    SiLU (Qwen3-MoE's ``"silu"``).
    """

    def __init__(self, num_experts: int, hidden_dim: int, intermediate_dim: int,
                 gate_up: Optional[torch.Tensor] = None, gate_up_state: Optional[QuantState] = None,
                 down: Optional[torch.Tensor] = None, down_state: Optional[QuantState] = None):
        super().__init__()
        self.num_experts = int(num_experts)
        self.hidden_dim = int(hidden_dim)
        self.intermediate_dim = int(intermediate_dim)
        self.gate_up = gate_up
        self.gate_up_state = gate_up_state
        self.down = down
        self.down_state = down_state
        self.streamed = False
        for qs, shape, what in ((gate_up_state, (self.num_experts * 2 * self.intermediate_dim, self.hidden_dim),
                                 "gate_up"),
                                (down_state, (self.num_experts * self.hidden_dim, self.intermediate_dim), "down")):
            if qs is not None and tuple(qs.shape) != shape:
                raise ValueError(f"NF4Experts: {what} quant state has shape {tuple(qs.shape)}, expected {shape}")

    @classmethod
    @torch.no_grad()
    def from_experts(cls, experts: nn.Module, *, device=None, compress_statistics: bool = False) -> "NF4Experts":
        """Quantize an HF ``Qwen3MoeExperts``-shaped module (``gate_up_proj [E, 2I, H]``,
        ``down_proj [E, H, I]``) on ``device`` (default: current CUDA device)."""
        act = getattr(experts, "act_fn", None)
        if act is not None and not isinstance(act, nn.SiLU) and type(act).__name__ not in ("SiLU", "SiLUActivation"):
            raise ValueError(f"NF4Experts: only SiLU experts are supported, got {type(act).__name__}")
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        gu = experts.gate_up_proj.detach()
        dn = experts.down_proj.detach()
        E, I2, H = gu.shape
        gq, gqs = quantize_4bit(gu.reshape(-1, H).to(dev), blocksize=64, compress_statistics=compress_statistics,
                                quant_type="nf4")
        dq, dqs = quantize_4bit(dn.reshape(-1, dn.shape[-1]).to(dev), blocksize=64,
                                compress_statistics=compress_statistics, quant_type="nf4")
        return cls(E, H, I2 // 2, gq, gqs, dq, dqs)

    @classmethod
    def streamed_from(cls, gate_up_weight: nn.Parameter, gate_up_payload, down_weight: nn.Parameter,
                      down_payload) -> "NF4Experts":
        """Experts fed by the streaming contract: ``gate_up_weight`` / ``down_weight`` are
        the frozen 3-D placeholder parameters carrying the NF4 payloads that
        ``upload.prepare_nf4`` attached (the reference's [-1, last] staging);
        ``ensure_weights`` uploads them into this module, ``free_weights`` drops them."""
        E, I2, H = (int(d) for d in gate_up_payload.shape)
        m = cls(E, H, I2 // 2)
        m.gate_up_weight = gate_up_weight
        m.down_weight = down_weight
        gate_up_weight.requires_grad_(False)
        down_weight.requires_grad_(False)
        if tuple(down_payload.shape) != (E, H, I2 // 2):
            raise ValueError(f"NF4Experts: down payload shape {tuple(down_payload.shape)} != {(E, H, I2 // 2)}")
        m.streamed = True
        return m

    def load_device_state(self, which: str, quantized: torch.Tensor, quant_state: QuantState) -> None:
        """Install one uploaded weight (``which`` = "gate_up_weight" or "down_weight"); the
        quant state's shape becomes the flattened [E*N_e, K] the grouped kernels take."""
        shape = tuple(int(d) for d in quant_state.shape)
        if len(shape) == 3:
            quant_state.shape = (shape[0] * shape[1], shape[2])
        if which == "gate_up_weight":
            self.gate_up, self.gate_up_state = quantized, quant_state
        elif which == "down_weight":
            self.down, self.down_state = quantized, quant_state
        else:
            raise ValueError(f"NF4Experts: unknown weight {which!r}")

    def device_state_on(self, which: str, device: torch.device) -> bool:
        t = self.gate_up if which == "gate_up_weight" else self.down
        return t is not None and t.device == device

    def drop_device_state(self, which: str) -> bool:
        if which == "gate_up_weight":
            had, self.gate_up, self.gate_up_state = self.gate_up is not None, None, None
        else:
            had, self.down, self.down_state = self.down is not None, None, None
        return had

    @property
    def resident(self) -> bool:
        return self.gate_up is not None and self.down is not None and self.gate_up.is_cuda

    def dequantized(self) -> tuple[torch.Tensor, torch.Tensor]:
        """The 3-D weights the reference materialises (for tests and inspection)."""
        E, H, I = self.num_experts, self.hidden_dim, self.intermediate_dim
        return (dequantize_4bit(self.gate_up, self.gate_up_state).reshape(E, 2 * I, H),
                dequantize_4bit(self.down, self.down_state).reshape(E, H, I))

    def forward(self, hidden_states: torch.Tensor, top_k_index: torch.Tensor,
                top_k_weights: torch.Tensor) -> torch.Tensor:
        if not self.resident:
            raise RuntimeError("NF4Experts: weights are not resident on a CUDA device (call ensure_weights first)")
        shape = hidden_states.shape
        x = hidden_states.reshape(-1, self.hidden_dim)
        if x.dtype not in (torch.bfloat16, torch.float16):
            raise ValueError(f"NF4Experts: hidden_states must be bf16 or fp16, got {x.dtype}")
        routing = ops.moe_route(top_k_index.reshape(x.shape[0], -1), self.num_experts)
        out = _NF4ExpertsFn.apply(x, top_k_weights, routing, self.gate_up, self.gate_up_state, self.down,
                                  self.down_state)
        return out.reshape(shape)

    def extra_repr(self) -> str:
        return (f"num_experts={self.num_experts}, hidden_dim={self.hidden_dim}, "
                f"intermediate_dim={self.intermediate_dim}, nf4")
