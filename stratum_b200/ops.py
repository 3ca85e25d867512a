"""Tensor-level wrappers of the fused NF4 GEMM kernels (no autograd here).

``nf4_gemm_fwd`` is the forward of the reference's NF4Linear
(stratum/nf4_linear.py:43-47: dequantize_4bit then F.linear) with PEFT's LoRA
update (scripts/train.py:568-573) folded into the same tensor-core
accumulator.  Shapes follow F.linear: x [..., K], weight [N, K], y [..., N].
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as TF

from . import _lib, codebook
from .functional import QuantState

LORA_CHUNK = 64


def _weight_args(qs: QuantState, dev: torch.device):
    """(absmax, absmax_q, absmax2, code2, offset, code16) device pointers of a QuantState."""
    code = qs.code if qs.code is not None else codebook.nf4_code(dev)
    if code.device != dev or code.dtype != torch.float32:
        code = code.to(dev, torch.float32)
    if qs.nested:
        s2 = qs.state2
        return (None, qs.absmax, s2.absmax, s2.code, qs.offset, code)
    return (qs.absmax, None, None, None, None, code)


def lora_down(x2: torch.Tensor, lora_A: torch.Tensor, scaling: float) -> torch.Tensor:
    """xa = scaling * x . lora_A^T in x's dtype, zero-padded to a multiple of 64 columns."""
    xa = torch.matmul(x2, lora_A.t())
    if scaling != 1.0:
        xa = (xa.float() * scaling).to(x2.dtype)
    r = xa.shape[1]
    pad = (-r) % LORA_CHUNK
    if pad:
        xa = TF.pad(xa, (0, pad))
    return xa.contiguous()


def nf4_gemm_fwd(
    x: torch.Tensor,
    packed: torch.Tensor,
    qs: QuantState,
    bias: Optional[torch.Tensor] = None,
    lora_A: Optional[torch.Tensor] = None,
    lora_B: Optional[torch.Tensor] = None,
    scaling: float = 1.0,
    xa: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """y = x . W^T + bias + scaling * (x . lora_A^T) . lora_B^T with W in NF4 (fused kernel).

    ``xa`` may be passed precomputed (scaling already applied, padded to a
    multiple of 64 columns), e.g. when the backward needs it too.
    """
    _lib.require_cuda(x, "nf4_gemm_fwd")
    if x.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError(f"nf4_gemm_fwd: x must be bf16 or fp16, got {x.dtype}")
    if qs.blocksize != 64:
        raise ValueError(f"nf4_gemm_fwd: the fused kernel needs NF4 blocksize 64, got {qs.blocksize}")
    N, K = int(qs.shape[0]), int(qs.shape[-1])
    if len(qs.shape) != 2:
        raise ValueError(f"nf4_gemm_fwd: weight must be 2-D, got shape {qs.shape}")
    if x.shape[-1] != K:
        raise ValueError(f"nf4_gemm_fwd: x has {x.shape[-1]} features, weight expects {K}")
    dev = x.device
    x2 = x.reshape(-1, K)
    if not x2.is_contiguous() or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    T = x2.shape[0]
    y = torch.empty((T, N), dtype=x.dtype, device=dev)
    r = 0
    lb = None
    if lora_B is not None:
        r = int(lora_B.shape[1])
        if xa is None:
            xa = lora_down(x2, lora_A, scaling)
        lb = lora_B if (lora_B.dtype == x.dtype and lora_B.is_contiguous()) else lora_B.to(x.dtype).contiguous()
        if r % 2:
            # the kernel reads rank pairs; an odd rank gets one zero column
            lb = TF.pad(lb, (0, 1))
            r += 1
    if bias is not None and (bias.device != dev or not bias.is_contiguous()):
        bias = bias.to(dev).contiguous()
    absmax, absmax_q, absmax2, code2, offset, code16 = _weight_args(qs, dev)
    L = _lib.lib()
    with torch.cuda.device(dev):
        _lib.check(
            L.stratum_nf4_gemm_fwd(
                _lib.ptr(x2), _lib.DTYPE_CODE[x.dtype], T, K, _lib.ptr(packed), _lib.ptr(absmax), _lib.ptr(absmax_q),
                _lib.ptr(absmax2), _lib.ptr(code2), _lib.ptr(offset), _lib.ptr(code16), N, _lib.ptr(bias),
                _lib.DTYPE_CODE.get(bias.dtype, 0) if bias is not None else 0, _lib.ptr(xa), _lib.ptr(lb), r,
                _lib.ptr(y), _lib.stream_of(dev),
            ),
            "nf4_gemm_fwd",
        )
    return y.reshape(*x.shape[:-1], N)


def nf4_gemm_dx(
    dy: torch.Tensor,
    packed: torch.Tensor,
    qs: QuantState,
    lora_A: Optional[torch.Tensor] = None,
    lora_B: Optional[torch.Tensor] = None,
    scaling: float = 1.0,
    dyb: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """dx = dy . W + scaling * (dy . lora_B) . lora_A with W in NF4 (fused kernel).

    ``dyb`` may be passed precomputed (= scaling * dy . lora_B, padded to a
    multiple of 64 columns), e.g. when dA needs it too.
    """
    _lib.require_cuda(dy, "nf4_gemm_dx")
    if dy.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError(f"nf4_gemm_dx: dy must be bf16 or fp16, got {dy.dtype}")
    if qs.blocksize != 64 or len(qs.shape) != 2:
        raise ValueError("nf4_gemm_dx: needs a 2-D NF4 weight with blocksize 64")
    N, K = int(qs.shape[0]), int(qs.shape[1])
    if dy.shape[-1] != N:
        raise ValueError(f"nf4_gemm_dx: dy has {dy.shape[-1]} features, weight has {N} rows")
    dev = dy.device
    dy2 = dy.reshape(-1, N)
    if not dy2.is_contiguous() or dy2.data_ptr() % 16:
        dy2 = dy2.contiguous()
    T = dy2.shape[0]
    dx = torch.empty((T, K), dtype=dy.dtype, device=dev)
    r = 0
    la = None
    if lora_A is not None:
        r = int(lora_A.shape[0])
        if dyb is None:
            dyb = lora_down(dy2, lora_B.t(), scaling)
        la = lora_A if (lora_A.dtype == dy.dtype and lora_A.is_contiguous()) else lora_A.to(dy.dtype).contiguous()
    absmax, absmax_q, absmax2, code2, offset, code16 = _weight_args(qs, dev)
    L = _lib.lib()
    with torch.cuda.device(dev):
        _lib.check(
            L.stratum_nf4_gemm_dx(
                _lib.ptr(dy2), _lib.DTYPE_CODE[dy.dtype], T, N, _lib.ptr(packed), _lib.ptr(absmax), _lib.ptr(absmax_q),
                _lib.ptr(absmax2), _lib.ptr(code2), _lib.ptr(offset), _lib.ptr(code16), K, _lib.ptr(dyb), _lib.ptr(la), r,
                _lib.ptr(dx), _lib.stream_of(dev),
            ),
            "nf4_gemm_dx",
        )
    return dx.reshape(*dy.shape[:-1], K)
