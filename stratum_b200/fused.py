"""Fused decoder-layer pieces around the NF4 GEMMs: RMSNorm, rotary, SwiGLU.

Drop-in modules for the parts of HF's Llama / Qwen3 decoder layers that the
reference runs as chains of small torch kernels (stratum/model/llama.py and
stratum/model/qwen3.py build those layers; the reference patches only their
attention kernel): ``FusedRMSNorm`` for ``LlamaRMSNorm`` / ``Qwen3RMSNorm``,
``FusedMLP`` for ``LlamaMLP`` (gate / up / down NF4Linears with one SwiGLU
kernel between them), ``FusedAttention`` for ``LlamaAttention`` /
``Qwen3Attention`` (q/k/v/o NF4Linears, optional per-head q/k RMSNorm, one
kernel that applies the rotary embedding and lays q and k out head-major for
the attention kernel, torch's SDPA -- cuDNN on B200 -- with GQA, one kernel
back to token-major for o_proj).  Each kernel reproduces the forward's bf16
roundings (csrc/fused_ops.cu); the backwards are the exact adjoints in fp32.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as TF

from . import _lib


def _call(name: str, *args) -> None:
    L = _lib.lib()
    _lib.check(getattr(L, name)(*args), name)


def _stream(t: torch.Tensor):
    return _lib.stream_of(t.device)


class _RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, eps):
        n = x.shape[-1]
        x2 = x.reshape(-1, n).contiguous()
        y = torch.empty_like(x2)
        rstd = torch.empty(x2.shape[0], dtype=torch.float32, device=x.device)
        with torch.cuda.device(x.device):
            _call("stratum_rmsnorm_fwd", _lib.ptr(x2), _lib.ptr(weight), _lib.DTYPE_CODE[x.dtype], x2.shape[0], n,
                  float(eps), _lib.ptr(y), _lib.ptr(rstd), _stream(x))
        ctx.save_for_backward(x2, weight, rstd)
        ctx.shape = x.shape
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, dy):
        x2, weight, rstd = ctx.saved_tensors
        n = x2.shape[1]
        dy2 = dy.reshape(-1, n).contiguous()
        dx = torch.empty_like(x2)
        with torch.cuda.device(dy.device):
            _call("stratum_rmsnorm_bwd", _lib.ptr(x2), _lib.ptr(weight), _lib.ptr(dy2), _lib.ptr(rstd),
                  _lib.DTYPE_CODE[dy.dtype], x2.shape[0], n, _lib.ptr(dx), _stream(dy))
        return dx.view(ctx.shape), None, None


class FusedRMSNorm(nn.Module):
    """``weight * round(x * rsqrt(mean(x^2) + eps))`` over the last dimension, frozen weight."""

    def __init__(self, weight: torch.Tensor, eps: float = 1e-6):
        super().__init__()
        self.weight = nn.Parameter(weight.detach().contiguous(), requires_grad=False)
        self.variance_epsilon = float(eps)

    @classmethod
    def from_hf(cls, norm: nn.Module) -> "FusedRMSNorm":
        return cls(norm.weight, getattr(norm, "variance_epsilon", getattr(norm, "eps", 1e-6)))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        _lib.require_cuda(x, "FusedRMSNorm")
        w = self.weight if self.weight.dtype == x.dtype else self.weight.to(x.dtype)
        return _RMSNormFn.apply(x, w, self.variance_epsilon)


class _SwiGLUFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, g, u):
        g, u = g.contiguous(), u.contiguous()
        h = torch.empty_like(g)
        with torch.cuda.device(g.device):
            _call("stratum_swiglu_fwd", _lib.ptr(g), _lib.ptr(u), _lib.DTYPE_CODE[g.dtype], g.numel(), _lib.ptr(h),
                  _stream(g))
        ctx.save_for_backward(g, u)
        return h

    @staticmethod
    def backward(ctx, dh):
        g, u = ctx.saved_tensors
        dh = dh.contiguous()
        dg, du = torch.empty_like(g), torch.empty_like(u)
        with torch.cuda.device(dh.device):
            _call("stratum_swiglu_bwd", _lib.ptr(g), _lib.ptr(u), _lib.ptr(dh), _lib.DTYPE_CODE[g.dtype], g.numel(),
                  _lib.ptr(dg), _lib.ptr(du), _stream(dh))
        return dg, du


def swiglu_backward_cat(gate: torch.Tensor, up: torch.Tensor, dh: torch.Tensor) -> torch.Tensor:
    """[dgate | dup] rows ([rows, 2I]) of ``h = silu(gate) * up`` with HF's roundings."""
    I = gate.shape[-1]
    g2, u2, d2 = (t.reshape(-1, I).contiguous() for t in (gate, up, dh))
    out = torch.empty((g2.shape[0], 2 * I), dtype=gate.dtype, device=gate.device)
    with torch.cuda.device(gate.device):
        _call("stratum_swiglu_bwd_cat", _lib.ptr(g2), _lib.ptr(u2), _lib.ptr(d2), _lib.DTYPE_CODE[gate.dtype],
              g2.shape[0], I, _lib.ptr(out), _stream(gate))
    return out


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """``silu(gate) * up`` with HF's bf16 roundings, one kernel each way."""
    _lib.require_cuda(gate, "swiglu")
    return _SwiGLUFn.apply(gate, up)


class _SwiGLUMLPFn(torch.autograd.Function):
    """The whole NF4 SwiGLU MLP with LoRA in three fused kernels:

    forward   gate and up GEMMs and one SwiGLU pass -- or, with ``fuse_forward``,
              one gate|up GEMM with the SwiGLU epilogue (h, plus 16-bit gate / up
              kept) -- then the down GEMM;
    backward  the down projection's input-gradient GEMM, one SwiGLU-backward pass
              writing [dgate | dup] rows, then one input-gradient pass through the
              stacked gate / up weights.  (The SwiGLU backward is not an epilogue of
              the down GEMM: its exp / divide per element would compete for issue
              slots with the NF4 decode on every SM and cost more than the
              standalone pass, which runs at HBM speed.)
    LoRA terms ride in the same accumulators (extra K chunks); dA / dB are small
    cuBLAS GEMMs as in NF4Linear."""

    @staticmethod
    def forward(ctx, x, Ag, Bg, Au, Bu, Ad, Bd, mods, fuse_forward):
        from . import ops

        gate, up, down = mods
        H = x.shape[-1]
        x2 = x.reshape(-1, H)
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        gw = (gate.quantized, gate.quant_state)
        uw = (up.quantized, up.quant_state)
        dw = (down.quantized, down.quant_state)
        xa_g = xa_u = None
        if fuse_forward:
            xa = ops.mlp_lora_down(x2, Ag, Au, gate.scaling, up.scaling) if Ag is not None else None
            h, g, u = ops.nf4_swiglu_fwd(x2, gw, uw, xa, Bg, Bu, keep_gate_up=True)
            if xa is not None:
                r, rp = Ag.shape[0], xa.shape[1] // 2
                xa_g, xa_u = xa[:, :r], xa[:, rp:rp + r]
        else:  # the two projections' GEMMs, then one SwiGLU pass
            if Ag is not None:
                xa_g = ops.lora_down(x2, Ag.to(x2.dtype), gate.scaling)
                xa_u = ops.lora_down(x2, Au.to(x2.dtype), up.scaling)
            g = ops.nf4_gemm_fwd(x2, gw[0], gw[1], lora_A=Ag, lora_B=Bg, scaling=gate.scaling, xa=xa_g)
            u = ops.nf4_gemm_fwd(x2, uw[0], uw[1], lora_A=Au, lora_B=Bu, scaling=up.scaling, xa=xa_u)
            h = torch.empty_like(g)
            with torch.cuda.device(g.device):
                _call("stratum_swiglu_fwd", _lib.ptr(g), _lib.ptr(u), _lib.DTYPE_CODE[g.dtype], g.numel(),
                      _lib.ptr(h), _stream(g))
            if Ag is not None:
                r = Ag.shape[0]
                xa_g, xa_u = xa_g[:, :r], xa_u[:, :r]
        xad = ops.lora_down(h, Ad.to(h.dtype), down.scaling) if Ad is not None else None
        y = ops.nf4_gemm_fwd(h, dw[0], dw[1], lora_A=Ad, lora_B=Bd, scaling=down.scaling, xa=xad)
        ctx.weights = (gw, uw, dw)
        ctx.scales = (gate.scaling, up.scaling, down.scaling)
        ctx.shape = x.shape
        ctx.save_for_backward(x2, xa_g, xa_u, g, u, h, xad, Ag, Bg, Au, Bu, Ad, Bd)
        return y.reshape(*x.shape[:-1], y.shape[-1])

    @staticmethod
    def backward(ctx, dy):
        from . import ops

        x2, xa_g, xa_u, g, u, h, xad, Ag, Bg, Au, Bu, Ad, Bd = ctx.saved_tensors
        gw, uw, dw = ctx.weights
        sg, su, sd = ctx.scales
        Hout = dy.shape[-1]
        dy2 = dy.reshape(-1, Hout)
        if not dy2.is_contiguous():
            dy2 = dy2.contiguous()
        I = g.shape[-1]
        grads = [None] * 6
        dyb_d = None
        if Ad is not None:
            rd = Ad.shape[0]
            dyb_d = ops.lora_down(dy2, Bd.t().to(dy2.dtype), sd)
            grads[4] = (dyb_d[:, :rd].t() @ h).to(Ad.dtype)
            grads[5] = (dy2.t() @ xad[:, :rd]).to(Bd.dtype)
        # dh through the down projection (its plain input-gradient kernel), then the
        # SwiGLU backward as one memory-bound pass writing [dgate | dup] rows
        dh = ops.nf4_gemm_dx(dy2, dw[0], dw[1], lora_A=Ad, lora_B=Bd, scaling=sd, dyb=dyb_d)
        dgu = swiglu_backward_cat(g, u, dh)
        del dh
        dg, du = dgu[:, :I], dgu[:, I:]
        dyb = A_cat = None
        if Ag is not None:
            r = Ag.shape[0]
            rp = -(-r // ops.LORA_CHUNK) * ops.LORA_CHUNK
            dyb = torch.zeros((dy2.shape[0], 2 * rp), dtype=dy2.dtype, device=dy2.device)
            dyb[:, :r] = ops.scaled_matmul(dg, Bg.to(dy2.dtype), sg)
            dyb[:, rp:rp + r] = ops.scaled_matmul(du, Bu.to(dy2.dtype), su)
            A_cat = torch.zeros((2 * rp, x2.shape[1]), dtype=dy2.dtype, device=dy2.device)
            A_cat[:r] = Ag
            A_cat[rp:rp + r] = Au
            grads[0] = (dyb[:, :r].t() @ x2).to(Ag.dtype)
            grads[1] = (dg.t() @ xa_g).to(Bg.dtype)
            grads[2] = (dyb[:, rp:rp + r].t() @ x2).to(Au.dtype)
            grads[3] = (du.t() @ xa_u).to(Bu.dtype)
        dx = None
        if ctx.needs_input_grad[0]:
            dx = ops.nf4_gemm_dx_pair(dgu, gw, uw, dyb, A_cat).reshape(ctx.shape)
        return (dx, *grads, None, None)


def _fusable(gate, up, down, x: torch.Tensor) -> bool:
    """Whether the three projections can run as the fused SwiGLU MLP kernels."""
    from .nf4_linear import NF4Linear

    mods = (gate, up, down)
    if not all(isinstance(m, NF4Linear) and m.quantized is not None and m.bias is None for m in mods):
        return False
    if x.dtype not in (torch.bfloat16, torch.float16) or x.device.type != "cuda":
        return False
    gq, uq, dq = gate.quant_state, up.quant_state, down.quant_state
    if any(q.blocksize != 64 or len(q.shape) != 2 for q in (gq, uq, dq)):
        return False
    I, H = int(gq.shape[0]), int(gq.shape[1])
    if tuple(uq.shape) != (I, H) or tuple(dq.shape) != (H, I) or I % 64 or H % 64:
        return False
    if bool(gq.nested) != bool(uq.nested):
        return False
    if (gate.lora_A is None) != (up.lora_A is None):
        return False
    if gate.lora_A is not None:
        r = gate.lora_A.shape[0]
        if r % 2 or up.lora_A.shape[0] != r or r > 128:
            return False
    if down.lora_A is not None and down.lora_A.shape[0] > 256:
        return False
    return True


class FusedMLP(nn.Module):
    """``down(swiglu(gate(x), up(x)))`` (LlamaMLP / Qwen3MLP with SiLU).

    With NF4Linear projections (blocksize 64, no bias, intermediate size a multiple
    of 64, gate and up LoRA of one even rank) the MLP runs through ``_SwiGLUMLPFn``,
    the dense counterpart of the reference's fused frozen MLP
    (stratum/model/mlp_opt.py:154-245): the backward takes the gate and up
    gradients through one stacked input-gradient GEMM fed by a single SwiGLU pass.
    ``fuse_forward=True`` also forms h in the gate|up GEMM's epilogue (one pass over
    x, gate and up never re-read); measured in the training pipeline on one B200 it
    wins at Qwen3-0.6B shapes and loses ~1% at Llama-3-8B shapes under the power
    cap, where the per-element exp / divide competes with the NF4 decode, so it is
    off by default.  Other projections run as three NF4Linears around one SwiGLU
    kernel."""

    def __init__(self, gate_proj: nn.Module, up_proj: nn.Module, down_proj: nn.Module, fuse: bool = True,
                 fuse_forward: bool = False):
        super().__init__()
        self.gate_proj, self.up_proj, self.down_proj = gate_proj, up_proj, down_proj
        self.fuse = fuse
        self.fuse_forward = fuse_forward

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        g, u, d = self.gate_proj, self.up_proj, self.down_proj
        if self.fuse and _fusable(g, u, d, x):
            return _SwiGLUMLPFn.apply(x, g.lora_A, g.lora_B, u.lora_A, u.lora_B, d.lora_A, d.lora_B, (g, u, d),
                                      bool(self.fuse_forward))
        return d(swiglu(g(x), u(x)))


class _HeadsFn(torch.autograd.Function):
    """[S, H*D] token-major -> [1, H, S, D] head-major, rotated when cos/sin are given."""

    @staticmethod
    def forward(ctx, x, cos, sin, H, D):
        S = x.shape[0]
        x = x.contiguous()
        y = torch.empty((1, H, S, D), dtype=x.dtype, device=x.device)
        with torch.cuda.device(x.device):
            _call("stratum_rope_to_heads", _lib.ptr(x), _lib.ptr(cos), _lib.ptr(sin), _lib.DTYPE_CODE[x.dtype], S, H,
                  D, _lib.ptr(y), _stream(x))
        ctx.save_for_backward(cos, sin) if cos is not None else ctx.save_for_backward()
        ctx.rot = cos is not None
        ctx.dims = (S, H, D)
        return y

    @staticmethod
    def backward(ctx, dy):
        S, H, D = ctx.dims
        cos, sin = ctx.saved_tensors if ctx.rot else (None, None)
        dy = dy.contiguous()
        dx = torch.empty((S, H * D), dtype=dy.dtype, device=dy.device)
        with torch.cuda.device(dy.device):
            _call("stratum_rope_from_heads", _lib.ptr(dy), _lib.ptr(cos), _lib.ptr(sin), _lib.DTYPE_CODE[dy.dtype], S,
                  H, D, _lib.ptr(dx), _stream(dy))
        return dx, None, None, None, None


class _TokensFn(torch.autograd.Function):
    """[1, H, S, D] head-major -> [S, H*D] token-major (no rotation)."""

    @staticmethod
    def forward(ctx, y):
        _, H, S, D = y.shape
        y = y.contiguous()
        x = torch.empty((S, H * D), dtype=y.dtype, device=y.device)
        with torch.cuda.device(y.device):
            _call("stratum_rope_from_heads", _lib.ptr(y), None, None, _lib.DTYPE_CODE[y.dtype], S, H, D, _lib.ptr(x),
                  _stream(y))
        ctx.dims = (S, H, D)
        return x

    @staticmethod
    def backward(ctx, dx):
        S, H, D = ctx.dims
        dx = dx.contiguous()
        dy = torch.empty((1, H, S, D), dtype=dx.dtype, device=dx.device)
        with torch.cuda.device(dx.device):
            _call("stratum_rope_to_heads", _lib.ptr(dx), None, None, _lib.DTYPE_CODE[dx.dtype], S, H, D, _lib.ptr(dy),
                  _stream(dx))
        return dy


def to_heads(x: torch.Tensor, H: int, D: int, cos: Optional[torch.Tensor] = None,
             sin: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``x`` [S, H*D] -> [1, H, S, D]; with ``cos``/``sin`` ([S, D]) the rotary embedding
    is applied as HF's ``apply_rotary_pos_emb`` does."""
    _lib.require_cuda(x, "to_heads")
    if cos is not None:
        cos = cos.reshape(-1, D).to(x.dtype).contiguous()
        sin = sin.reshape(-1, D).to(x.dtype).contiguous()
    return _HeadsFn.apply(x, cos, sin, H, D)


def to_tokens(y: torch.Tensor) -> torch.Tensor:
    """[1, H, S, D] -> [S, H*D]."""
    return _TokensFn.apply(y)


class FusedAttention(nn.Module):
    """Causal self-attention with NF4 projections (LlamaAttention / Qwen3Attention
    forward, no KV cache, no padding mask).  Returns ``(output, None)`` like HF."""

    def __init__(self, q_proj, k_proj, v_proj, o_proj, heads: int, kv_heads: int, head_dim: int,
                 q_norm: Optional[nn.Module] = None, k_norm: Optional[nn.Module] = None):
        super().__init__()
        self.q_proj, self.k_proj, self.v_proj, self.o_proj = q_proj, k_proj, v_proj, o_proj
        self.heads, self.kv_heads, self.head_dim = heads, kv_heads, head_dim
        self.q_norm, self.k_norm = q_norm, k_norm
        self.scaling = head_dim ** -0.5

    @classmethod
    def from_hf(cls, attn: nn.Module, heads: int, kv_heads: int, head_dim: int) -> "FusedAttention":
        qn = FusedRMSNorm.from_hf(attn.q_norm) if hasattr(attn, "q_norm") else None
        kn = FusedRMSNorm.from_hf(attn.k_norm) if hasattr(attn, "k_norm") else None
        return cls(attn.q_proj, attn.k_proj, attn.v_proj, attn.o_proj, heads, kv_heads, head_dim, qn, kn)

    def forward(self, hidden_states: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
                position_ids=None, past_key_values=None, use_cache=False, position_embeddings=None, **kwargs):
        if attention_mask is not None:
            raise ValueError("FusedAttention: causal attention only (no materialised mask)")
        if past_key_values is not None:
            raise ValueError("FusedAttention: no KV cache")
        B, S, _ = hidden_states.shape
        H, Hk, D = self.heads, self.kv_heads, self.head_dim
        cos, sin = position_embeddings
        q = self.q_proj(hidden_states)
        k = self.k_proj(hidden_states)
        v = self.v_proj(hidden_states)
        if self.q_norm is not None:
            q = self.q_norm(q.view(B, S, H, D)).view(B, S, H * D)
            k = self.k_norm(k.view(B, S, Hk, D)).view(B, S, Hk * D)
        outs = []
        for b in range(B):
            qh = to_heads(q[b], H, D, cos[b if cos.shape[0] > 1 else 0], sin[b if sin.shape[0] > 1 else 0])
            kh = to_heads(k[b], Hk, D, cos[b if cos.shape[0] > 1 else 0], sin[b if sin.shape[0] > 1 else 0])
            vh = to_heads(v[b], Hk, D)
            o = TF.scaled_dot_product_attention(qh, kh, vh, is_causal=True, scale=self.scaling, enable_gqa=(H != Hk))
            outs.append(to_tokens(o))
        o = torch.stack(outs, 0) if B > 1 else outs[0].unsqueeze(0)
        return self.o_proj(o), None


__all__ = ["FusedRMSNorm", "FusedMLP", "FusedAttention", "swiglu", "to_heads", "to_tokens"]
