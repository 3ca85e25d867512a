"""Tensor-level wrappers of the fused NF4 GEMM kernels (no autograd here).

``nf4_gemm_fwd`` is the forward of the reference's NF4Linear
(stratum/nf4_linear.py:43-47: dequantize_4bit then F.linear) with PEFT's LoRA
update (scripts/train.py:568-573) folded into the same tensor-core
accumulator.  Shapes follow F.linear: x [..., K], weight [N, K], y [..., N].
"""

from __future__ import annotations

import os
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
    if scaling != 1.0:  # the scale rides on cuBLAS's alpha (beta = 0: the buffer is not read)
        xa = torch.addmm(torch.empty((x2.shape[0], lora_A.shape[0]), dtype=x2.dtype, device=x2.device), x2,
                         lora_A.t(), beta=0, alpha=scaling)
    else:
        xa = torch.matmul(x2, lora_A.t())
    r = xa.shape[1]
    pad = (-r) % LORA_CHUNK
    if pad:
        xa = TF.pad(xa, (0, pad))
    return xa.contiguous()


_GEMM_KERNELS = {"auto": 0, "pair": 1, "single": 2}


_gemm_kernel_chosen = False  # set_gemm_kernel was called by the user


def set_gemm_kernel(which: str) -> None:
    """Kernel for every later NF4 forward and input-gradient GEMM in this process:
    ``"auto"`` (by estimated makespan), ``"pair"`` (512-token x 256-column tiles on
    CTA pairs sharing 2-SM MMAs) or ``"single"`` (the one-SM kernels)."""
    global _gemm_kernel_chosen
    if which not in _GEMM_KERNELS:
        raise ValueError(f"set_gemm_kernel: expected one of {sorted(_GEMM_KERNELS)}, got {which!r}")
    _lib.check(_lib.lib().stratum_nf4_gemm_set_kernel(_GEMM_KERNELS[which]), "set_gemm_kernel")
    _gemm_kernel_chosen = True


def multirank_gemm_default() -> None:
    """One-SM GEMM kernels for one rank of a multi-rank pipeline, unless the kernel
    was chosen explicitly (``set_gemm_kernel`` or ``STRATUM_NF4_GEMM``).  In MoE
    pipeline runs the grouped expert input-gradient kernel sometimes finds foreign
    data in its barrier words and its bounded wait gives up. On two GPUs that
    happened in 9 of 39 steps beside the CTA-pair kernels (one run also ended in a
    launch failure) and in 1 of 14 beside the one-SM kernels."""
    if _gemm_kernel_chosen or os.environ.get("STRATUM_NF4_GEMM"):
        return
    _lib.check(_lib.lib().stratum_nf4_gemm_set_kernel(_GEMM_KERNELS["single"]), "multirank_gemm_default")


def nf4_gemm_fwd(
    x: torch.Tensor,
    packed: torch.Tensor,
    qs: QuantState,
    bias: Optional[torch.Tensor] = None,
    lora_A: Optional[torch.Tensor] = None,
    lora_B: Optional[torch.Tensor] = None,
    scaling: float = 1.0,
    xa: Optional[torch.Tensor] = None,
    out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """y = x . W^T + bias + scaling * (x . lora_A^T) . lora_B^T with W in NF4 (fused kernel).

    ``xa`` may be passed precomputed (scaling already applied, padded to a
    multiple of 64 columns), e.g. when the backward needs it too.  ``out``: a
    contiguous, 16-byte aligned [rows, N] tensor of x's dtype and device to write y into.
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
    if out is None:
        y = torch.empty((T, N), dtype=x.dtype, device=dev)
    else:
        if (out.dtype != x.dtype or out.device != dev or out.numel() != T * N or not out.is_contiguous()
                or out.data_ptr() % 16):
            raise ValueError(f"nf4_gemm_fwd: out must be a contiguous, 16-byte aligned {x.dtype} tensor of "
                             f"{T * N} elements on {dev}")
        y = out.view(T, N)
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
    out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """dx = dy . W + scaling * (dy . lora_B) . lora_A with W in NF4 (fused kernel).

    ``dyb`` may be passed precomputed (= scaling * dy . lora_B, padded to a
    multiple of 64 columns), e.g. when dA needs it too.  ``out``: a contiguous,
    16-byte aligned [rows, K] tensor of dy's dtype and device to write dx into.
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
    if out is None:
        dx = torch.empty((T, K), dtype=dy.dtype, device=dev)
    else:
        if (out.dtype != dy.dtype or out.device != dev or out.numel() != T * K or not out.is_contiguous()
                or out.data_ptr() % 16):
            raise ValueError(f"nf4_gemm_dx: out must be a contiguous, 16-byte aligned {dy.dtype} tensor of "
                             f"{T}x{K} elements on {dev}")
        dx = out
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
    return dx if out is not None else dx.reshape(*dy.shape[:-1], K)


# --------------------------------------------------------------------------------
# fused SwiGLU MLP (dense): one gate|up GEMM with the SwiGLU epilogue, and the
# matching input gradients
# --------------------------------------------------------------------------------

def _nf4_weight(packed: torch.Tensor, qs: QuantState, dev: torch.device, keep: list) -> "_lib.NF4Weight":
    absmax, absmax_q, absmax2, code2, offset, code16 = _weight_args(qs, dev)
    keep += [t for t in (packed, absmax, absmax_q, absmax2, code2, offset, code16) if t is not None]
    w = _lib.NF4Weight()
    w.packed = packed.data_ptr()
    w.absmax = 0 if absmax is None else absmax.data_ptr()
    w.absmax_q = 0 if absmax_q is None else absmax_q.data_ptr()
    w.absmax2 = 0 if absmax2 is None else absmax2.data_ptr()
    w.code2 = 0 if code2 is None else code2.data_ptr()
    w.offset = 0 if offset is None else offset.data_ptr()
    return w


def _addr(w) -> "ctypes.c_void_p":
    import ctypes

    return ctypes.c_void_p(ctypes.addressof(w))


def mlp_lora_down(x2: torch.Tensor, A_gate: torch.Tensor, A_up: torch.Tensor, s_gate: float,
                  s_up: float) -> torch.Tensor:
    """xa = [s_gate x A_gate^T | 0 | s_up x A_up^T | 0] with each half ceil(r/64)*64 wide."""
    r = int(A_gate.shape[0])
    rp = -(-r // LORA_CHUNK) * LORA_CHUNK
    xa = torch.zeros((x2.shape[0], 2 * rp), dtype=x2.dtype, device=x2.device)
    for c0, A, s in ((0, A_gate, s_gate), (rp, A_up, s_up)):
        xa[:, c0:c0 + r] = scaled_matmul(x2, A.to(x2.dtype).t(), s)
    return xa


def scaled_matmul(a: torch.Tensor, b: torch.Tensor, s: float) -> torch.Tensor:
    """s * (a @ b) with the scale applied in cuBLAS's fp32 epilogue (one rounding)."""
    if s == 1.0:
        return torch.matmul(a, b)
    return torch.addmm(torch.empty((a.shape[0], b.shape[1]), dtype=a.dtype, device=a.device), a, b, beta=0, alpha=s)


def nf4_swiglu_fwd(x: torch.Tensor, gate: tuple, up: tuple, xa: Optional[torch.Tensor] = None,
                   lora_B_gate: Optional[torch.Tensor] = None, lora_B_up: Optional[torch.Tensor] = None,
                   keep_gate_up: bool = True):
    """h = silu(x Wg^T + LoRA_g) * (x Wu^T + LoRA_u) with HF's bf16 roundings, one fused kernel.

    ``gate`` / ``up``: ``(packed, QuantState)`` of two NF4 weights [I, K] (blocksize 64,
    I % 64 == 0); ``xa`` from :func:`mlp_lora_down` with the LoRA B matrices [I, r].
    Returns ``(h, gate_out, up_out)`` ([rows, I]; the last two None unless kept)."""
    _lib.require_cuda(x, "nf4_swiglu_fwd")
    (gp, gqs), (upk, uqs) = gate, up
    I, K = int(gqs.shape[0]), int(gqs.shape[1])
    if tuple(uqs.shape) != (I, K) or gqs.blocksize != 64 or uqs.blocksize != 64:
        raise ValueError("nf4_swiglu_fwd: gate and up must be [I, K] NF4 weights with blocksize 64")
    dev = x.device
    x2 = x.reshape(-1, K)
    if not x2.is_contiguous() or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    T = x2.shape[0]
    h = torch.empty((T, I), dtype=x.dtype, device=dev)
    g_out = torch.empty((T, I), dtype=x.dtype, device=dev) if keep_gate_up else None
    u_out = torch.empty((T, I), dtype=x.dtype, device=dev) if keep_gate_up else None
    r = 0
    lbg = lbu = None
    if lora_B_gate is not None:
        r = int(lora_B_gate.shape[1])
        if r % 2:
            raise ValueError("nf4_swiglu_fwd: the LoRA rank must be even")
        lbg = lora_B_gate.to(x.dtype).contiguous()
        lbu = lora_B_up.to(x.dtype).contiguous()
    keep: list = []
    wg = _nf4_weight(gp, gqs, dev, keep)
    wu = _nf4_weight(upk, uqs, dev, keep)
    code16 = keep[-1]
    L = _lib.lib()
    with torch.cuda.device(dev):
        _lib.check(L.stratum_nf4_gemm_swiglu_fwd(
            _lib.ptr(x2), _lib.DTYPE_CODE[x.dtype], T, K, _addr(wg), _addr(wu), _lib.ptr(code16), I, _lib.ptr(xa),
            _lib.ptr(lbg), _lib.ptr(lbu), r, _lib.ptr(h), _lib.ptr(g_out), _lib.ptr(u_out), _lib.stream_of(dev)),
            "nf4_swiglu_fwd")
    shp = x.shape[:-1]
    return (h.reshape(*shp, I), None if g_out is None else g_out.reshape(*shp, I),
            None if u_out is None else u_out.reshape(*shp, I))


def nf4_gemm_dx_pair(dy: torch.Tensor, w0: tuple, w1: tuple, dyb: Optional[torch.Tensor] = None,
                     lora_A: Optional[torch.Tensor] = None) -> torch.Tensor:
    """dx = dy [W0; W1] + dyb lora_A for two NF4 weights stacked along their rows
    (dy [rows, N0 + N1]), one fused input-gradient pass."""
    _lib.require_cuda(dy, "nf4_gemm_dx_pair")
    (p0, q0), (p1, q1) = w0, w1
    N0, K = int(q0.shape[0]), int(q0.shape[1])
    N1 = int(q1.shape[0])
    if int(q1.shape[1]) != K:
        raise ValueError("nf4_gemm_dx_pair: the weights need the same number of columns")
    dev = dy.device
    dy2 = dy.reshape(-1, N0 + N1)
    if not dy2.is_contiguous() or dy2.data_ptr() % 16:
        dy2 = dy2.contiguous()
    T = dy2.shape[0]
    dx = torch.empty((T, K), dtype=dy.dtype, device=dev)
    r = 0
    la = None
    if lora_A is not None:
        r = int(lora_A.shape[0])
        la = lora_A.to(dy.dtype).contiguous()
    keep: list = []
    a = _nf4_weight(p0, q0, dev, keep)
    b = _nf4_weight(p1, q1, dev, keep)
    code16 = keep[-1]
    L = _lib.lib()
    with torch.cuda.device(dev):
        _lib.check(L.stratum_nf4_gemm_dx_pair(
            _lib.ptr(dy2), _lib.DTYPE_CODE[dy.dtype], T, _addr(a), N0, _addr(b), N1, _lib.ptr(code16), K, _lib.ptr(dyb),
            _lib.ptr(la), r, _lib.ptr(dx), _lib.stream_of(dev)), "nf4_gemm_dx_pair")
    return dx.reshape(*dy.shape[:-1], K)


# --------------------------------------------------------------------------------
# routed experts (include/stratum_moe.h)
# --------------------------------------------------------------------------------

class Routing:
    """Expert-sorted layout of the router's (token, slot) pairs.

    ``order[p]`` is the flat pair ``t*k + slot`` of sorted row ``p``, ``inv`` its
    inverse, ``token_of[p] = order[p] // k``; expert ``e`` owns sorted rows
    ``offsets[e]:offsets[e+1]``.  Pairs whose expert id lies outside
    ``[0, n_experts)`` are dropped (sorted after ``offsets[E]``), as HF's
    ``Qwen3MoeExperts.forward`` skips ``expert_idx == num_experts``.
    """

    __slots__ = ("order", "inv", "token_of", "offsets", "T", "k", "n_experts")

    def __init__(self, order, inv, token_of, offsets, T, k, n_experts):
        self.order, self.inv, self.token_of, self.offsets = order, inv, token_of, offsets
        self.T, self.k, self.n_experts = T, k, n_experts

    @property
    def rows(self) -> int:
        return self.T * self.k


def moe_route(top_k_index: torch.Tensor, n_experts: int) -> Routing:
    """Stable counting sort of ``top_k_index`` ([T, k] expert ids) by expert, on the GPU."""
    _lib.require_cuda(top_k_index, "moe_route")
    if top_k_index.dim() != 2:
        raise ValueError(f"moe_route: top_k_index must be [T, k], got {tuple(top_k_index.shape)}")
    dev = top_k_index.device
    idx = top_k_index.to(torch.int64).contiguous()
    T, k = int(idx.shape[0]), int(idx.shape[1])
    n = T * k
    order = torch.empty(n, dtype=torch.int32, device=dev)
    inv = torch.empty(n, dtype=torch.int32, device=dev)
    token_of = torch.empty(n, dtype=torch.int32, device=dev)
    offsets = torch.empty(n_experts + 1, dtype=torch.int32, device=dev)
    L = _lib.lib()
    ws_bytes = int(L.stratum_moe_route_workspace_bytes(n, n_experts))
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _lib.check(L.stratum_moe_route(_lib.ptr(idx), T, k, n_experts, _lib.ptr(order), _lib.ptr(inv),
                                       _lib.ptr(token_of), _lib.ptr(offsets), _lib.ptr(ws), ws_bytes,
                                       _lib.stream_of(dev)), "moe_route")
    return Routing(order, inv, token_of, offsets, T, k, n_experts)


def moe_gather_rows(src: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    """``src[idx]`` for a 2-D ``src`` with 16-byte rows (the expert dispatch gather)."""
    _lib.require_cuda(src, "moe_gather_rows")
    src = src.contiguous()
    dst = torch.empty((idx.numel(), src.shape[1]), dtype=src.dtype, device=src.device)
    L = _lib.lib()
    with torch.cuda.device(src.device):
        _lib.check(L.stratum_moe_gather_rows(_lib.ptr(src), src.shape[1] * src.element_size(), _lib.ptr(idx),
                                             idx.numel(), _lib.ptr(dst), _lib.stream_of(src.device)),
                   "moe_gather_rows")
    return dst


def _table(rows: int, n_experts: int, weight_dim: int, dev: torch.device) -> tuple[torch.Tensor, int]:
    nbytes = int(_lib.lib().stratum_nf4_grouped_table_bytes(rows, n_experts, weight_dim))
    return torch.empty(nbytes, dtype=torch.uint8, device=dev), nbytes


def _expert_weight_shape(qs: QuantState, n_experts: int, what: str) -> tuple[int, int]:
    """(N_e, K) of a flattened [E*N_e, K] NF4 expert weight."""
    if qs.blocksize != 64 or len(qs.shape) != 2:
        raise ValueError(f"{what}: needs a flattened 2-D NF4 expert weight with blocksize 64")
    rows, K = int(qs.shape[0]), int(qs.shape[1])
    if rows % n_experts:
        raise ValueError(f"{what}: {rows} weight rows do not split into {n_experts} experts")
    return rows // n_experts, K


def nf4_grouped_fwd(x_sorted: torch.Tensor, routing: Routing, packed: torch.Tensor, qs: QuantState, *,
                    swiglu: bool = False, rw: Optional[torch.Tensor] = None, keep_gate_up: bool = False):
    """Grouped expert forward over expert-sorted rows (one launch for every expert).

    ``qs.shape`` is ``(E*N_e, K)``.  Plain: returns ``x_sorted . W[e]^T`` (times
    ``rw``, per sorted row, when given).  ``swiglu``: the weight is gate_up_proj and
    the result is ``silu(gate) * up`` ([rows, N_e/2]); with ``keep_gate_up`` the
    gate|up activations ([rows, N_e]) are returned as well.
    """
    _lib.require_cuda(x_sorted, "nf4_grouped_fwd")
    if x_sorted.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError(f"nf4_grouped_fwd: x must be bf16 or fp16, got {x_sorted.dtype}")
    E = routing.n_experts
    N_e, K = _expert_weight_shape(qs, E, "nf4_grouped_fwd")
    if x_sorted.shape[-1] != K or x_sorted.shape[0] != routing.rows:
        raise ValueError(f"nf4_grouped_fwd: x_sorted {tuple(x_sorted.shape)} does not match [{routing.rows}, {K}]")
    dev = x_sorted.device
    x2 = x_sorted.contiguous()
    rows = x2.shape[0]
    y = torch.empty((rows, N_e // 2 if swiglu else N_e), dtype=x2.dtype, device=dev)
    gu = torch.empty((rows, N_e), dtype=x2.dtype, device=dev) if (swiglu and keep_gate_up) else None
    if rw is not None:
        rw = rw.to(device=dev, dtype=torch.float32).contiguous()
    table, tbytes = _table(rows, E, max(N_e, K), dev)
    absmax, absmax_q, absmax2, code2, offset, code16 = _weight_args(qs, dev)
    L = _lib.lib()
    with torch.cuda.device(dev):
        _lib.check(
            L.stratum_nf4_grouped_fwd(
                _lib.ptr(x2), _lib.DTYPE_CODE[x2.dtype], rows, K, _lib.ptr(routing.offsets), E, _lib.ptr(packed),
                _lib.ptr(absmax), _lib.ptr(absmax_q), _lib.ptr(absmax2), _lib.ptr(code2), _lib.ptr(offset),
                _lib.ptr(code16), N_e, int(swiglu), _lib.ptr(rw), _lib.ptr(y), _lib.ptr(gu), _lib.ptr(table), tbytes,
                _lib.stream_of(dev)),
            "nf4_grouped_fwd",
        )
    return (y, gu) if keep_gate_up else y


def nf4_grouped_dx(dy_sorted: torch.Tensor, routing: Routing, packed: torch.Tensor, qs: QuantState) -> torch.Tensor:
    """Grouped expert input gradient: ``dy_sorted . W[e]`` for every sorted row."""
    _lib.require_cuda(dy_sorted, "nf4_grouped_dx")
    if dy_sorted.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError(f"nf4_grouped_dx: dy must be bf16 or fp16, got {dy_sorted.dtype}")
    E = routing.n_experts
    N_e, K = _expert_weight_shape(qs, E, "nf4_grouped_dx")
    if dy_sorted.shape[-1] != N_e or dy_sorted.shape[0] != routing.rows:
        raise ValueError(f"nf4_grouped_dx: dy_sorted {tuple(dy_sorted.shape)} does not match [{routing.rows}, {N_e}]")
    dev = dy_sorted.device
    dy2 = dy_sorted.contiguous()
    rows = dy2.shape[0]
    dx = torch.empty((rows, K), dtype=dy2.dtype, device=dev)
    table, tbytes = _table(rows, E, max(N_e, K), dev)
    absmax, absmax_q, absmax2, code2, offset, code16 = _weight_args(qs, dev)
    L = _lib.lib()
    with torch.cuda.device(dev):
        _lib.check(
            L.stratum_nf4_grouped_dx(
                _lib.ptr(dy2), _lib.DTYPE_CODE[dy2.dtype], rows, N_e, _lib.ptr(routing.offsets), E, _lib.ptr(packed),
                _lib.ptr(absmax), _lib.ptr(absmax_q), _lib.ptr(absmax2), _lib.ptr(code2), _lib.ptr(offset),
                _lib.ptr(code16), K, _lib.ptr(dx), _lib.ptr(table), tbytes, _lib.stream_of(dev)),
            "nf4_grouped_dx",
        )
    return dx


def moe_combine(rows: torch.Tensor, routing: Routing, weights: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``out[t] = sum_s weights[t, s] * rows[inv[t*k+s]]`` (fp32 sum), [T, width] in ``rows.dtype``."""
    _lib.require_cuda(rows, "moe_combine")
    dev = rows.device
    rows = rows.contiguous()
    width = rows.shape[1]
    out = torch.empty((routing.T, width), dtype=rows.dtype, device=dev)
    if weights is not None:
        weights = weights.reshape(-1).to(device=dev, dtype=torch.float32).contiguous()
    L = _lib.lib()
    with torch.cuda.device(dev):
        _lib.check(L.stratum_moe_combine(_lib.ptr(rows), _lib.DTYPE_CODE[rows.dtype], _lib.ptr(routing.inv),
                                         _lib.ptr(weights), _lib.ptr(routing.offsets), routing.n_experts, routing.T,
                                         routing.k, width, _lib.ptr(out), _lib.stream_of(dev)), "moe_combine")
    return out


def moe_combine_grad(dout: torch.Tensor, routing: Routing, weights: Optional[torch.Tensor],
                     rows: Optional[torch.Tensor]) -> tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Backward of :func:`moe_combine`: (dy_sorted, dweights [T*k] fp32 or None when ``rows`` is None)."""
    _lib.require_cuda(dout, "moe_combine_grad")
    dev = dout.device
    dout = dout.contiguous()
    width = dout.shape[1]
    dy_sorted = torch.empty((routing.rows, width), dtype=dout.dtype, device=dev)
    dw = torch.empty(routing.rows, dtype=torch.float32, device=dev) if rows is not None else None
    if weights is not None:
        weights = weights.reshape(-1).to(device=dev, dtype=torch.float32).contiguous()
    L = _lib.lib()
    with torch.cuda.device(dev):
        _lib.check(L.stratum_moe_combine_grad(_lib.ptr(dout), _lib.DTYPE_CODE[dout.dtype], _lib.ptr(routing.order),
                                              _lib.ptr(routing.token_of), _lib.ptr(weights), _lib.ptr(routing.offsets),
                                              routing.n_experts, _lib.ptr(rows), routing.rows, width,
                                              _lib.ptr(dy_sorted), _lib.ptr(dw), _lib.stream_of(dev)),
                   "moe_combine_grad")
    return dy_sorted, dw


def swiglu_grad(gate_up: torch.Tensor, dh: torch.Tensor) -> torch.Tensor:
    """d(gate|up) of ``h = silu(gate) * up`` given the saved gate|up and dh."""
    _lib.require_cuda(gate_up, "swiglu_grad")
    rows, inter = int(dh.shape[0]), int(dh.shape[1])
    if tuple(gate_up.shape) != (rows, 2 * inter):
        raise ValueError(f"swiglu_grad: gate_up {tuple(gate_up.shape)} does not match dh {tuple(dh.shape)}")
    gate_up, dh = gate_up.contiguous(), dh.contiguous()
    dgu = torch.empty_like(gate_up)
    L = _lib.lib()
    with torch.cuda.device(dh.device):
        _lib.check(L.stratum_swiglu_grad(_lib.ptr(gate_up), _lib.ptr(dh),
                                         _lib.DTYPE_CODE[dh.dtype], rows, inter, _lib.ptr(dgu),
                                         _lib.stream_of(dh.device)), "swiglu_grad")
    return dgu
