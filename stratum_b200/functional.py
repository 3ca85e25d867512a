"""bitsandbytes-compatible NF4 codec entry points backed by the sm_100a kernels.

The reference calls ``bitsandbytes.functional.quantize_4bit`` /
``dequantize_4bit`` / ``QuantState`` (stratum/upload.py:193-222, :355-369,
:922-946, :1021-1040; stratum/nf4_linear.py:44-46).  This module keeps those
names and argument meanings so the call sites read the same, and routes every
call to ``libstratum_nf4.so``.  There is no CPU implementation: a CPU tensor is
processed on the current CUDA device and the result is returned on the CPU
(the device the caller passed), and without a CUDA device the call raises.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib, codebook

SUPPORTED_QUANT_BLOCKSIZES = (32, 64, 128, 256)
DQ_BLOCKSIZE = 256


class QuantState:
    """Metadata of an NF4-quantized tensor (mirrors bitsandbytes' QuantState).

    ``absmax`` is float32 [nb], or uint8 [nb] when ``state2`` is set (double
    quantization; then ``offset`` is a float32 scalar tensor and ``state2``
    holds absmax2 [ceil(nb/256)] and the 256-entry dynamic code).
    """

    def __init__(
        self,
        absmax: torch.Tensor,
        shape=None,
        code: Optional[torch.Tensor] = None,
        blocksize: Optional[int] = None,
        quant_type: Optional[str] = None,
        dtype: Optional[torch.dtype] = None,
        offset: Optional[torch.Tensor] = None,
        state2: Optional["QuantState"] = None,
    ):
        self.absmax = absmax
        self.shape = tuple(shape) if shape is not None else None
        self.code = code
        self.blocksize = blocksize
        self.quant_type = quant_type
        self.dtype = dtype
        self.offset = offset
        self.state2 = state2
        self.nested = state2 is not None

    def to(self, device) -> "QuantState":
        dev = torch.device(device)
        self.absmax = self.absmax.to(dev, non_blocking=True)
        if self.code is not None:
            self.code = self.code.to(dev, non_blocking=True)
        if self.offset is not None:
            self.offset = self.offset.to(dev, non_blocking=True)
        if self.state2 is not None:
            self.state2.to(dev)
        return self

    def __repr__(self) -> str:
        return (
            f"QuantState(shape={self.shape}, dtype={self.dtype}, blocksize={self.blocksize}, "
            f"quant_type={self.quant_type!r}, nested={self.nested})"
        )


def _check_quant_type(quant_type: str) -> None:
    if quant_type != "nf4":
        raise ValueError(f"quant_type {quant_type!r} is not supported: this build implements NF4 only")


def _compute_device(t: torch.Tensor, what: str) -> torch.device:
    if t.device.type == "cuda":
        return t.device
    if not torch.cuda.is_available():
        raise RuntimeError(f"{what}: no CUDA device; the NF4 kernels have no CPU fallback")
    return torch.device("cuda", torch.cuda.current_device())


def _f32_on(t: torch.Tensor, dev: torch.device) -> torch.Tensor:
    if t.device != dev or t.dtype != torch.float32 or not t.is_contiguous():
        t = t.to(device=dev, dtype=torch.float32).contiguous()
    return t


@torch.no_grad()
def quantize_4bit(
    A: torch.Tensor,
    absmax: Optional[torch.Tensor] = None,
    out: Optional[torch.Tensor] = None,
    blocksize: int = 64,
    compress_statistics: bool = False,
    quant_type: str = "nf4",
    quant_storage: torch.dtype = torch.uint8,
    *,
    thresholds: str = "cuda",
) -> tuple[torch.Tensor, QuantState]:
    """Blockwise NF4 quantization of ``A`` (fp16/bf16/fp32, any shape).

    Returns ``(packed, state)`` with ``packed`` uint8 of shape
    ``((n + 1) // 2, 1)`` like bitsandbytes.  ``thresholds`` picks the
    decision-threshold convention (see :mod:`stratum_b200.codebook`).
    """
    _check_quant_type(quant_type)
    if quant_storage != torch.uint8:
        raise ValueError("quant_storage must be torch.uint8")
    if blocksize not in SUPPORTED_QUANT_BLOCKSIZES:
        raise ValueError(f"blocksize {blocksize} not in {SUPPORTED_QUANT_BLOCKSIZES}")
    if A.dtype not in _lib.DTYPE_CODE:
        raise ValueError(f"quantize_4bit: unsupported dtype {A.dtype}")
    home = A.device
    dev = _compute_device(A, "quantize_4bit")
    src = A.detach().to(dev, non_blocking=True).contiguous()
    n = src.numel()
    nb = (n + blocksize - 1) // blocksize
    packed = out if out is not None else torch.empty(((n + 1) // 2, 1), dtype=torch.uint8, device=dev)
    am = torch.empty(nb, dtype=torch.float32, device=dev)
    L = _lib.lib()
    with torch.cuda.device(dev):
        st = _lib.stream_of(dev)
        _lib.check(
            L.stratum_nf4_quantize(
                _lib.ptr(src), _lib.DTYPE_CODE[src.dtype], n, blocksize,
                _lib.ptr(codebook.nf4_thresholds(dev, thresholds)), _lib.ptr(packed), _lib.ptr(am), st,
            ),
            "quantize_4bit",
        )
        code = codebook.nf4_code(dev)
        if compress_statistics:
            absmax_q = torch.empty(nb, dtype=torch.uint8, device=dev)
            absmax2 = torch.empty((nb + DQ_BLOCKSIZE - 1) // DQ_BLOCKSIZE, dtype=torch.float32, device=dev)
            offset = torch.empty((), dtype=torch.float32, device=dev)
            ws_bytes = int(L.stratum_nf4_dq_workspace_bytes(nb))
            ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
            _lib.check(
                L.stratum_nf4_quantize_absmax_dq(
                    _lib.ptr(am), nb, DQ_BLOCKSIZE, _lib.ptr(codebook.dynamic_thresholds(dev)),
                    _lib.ptr(absmax_q), _lib.ptr(absmax2), _lib.ptr(offset), _lib.ptr(ws), ws_bytes, st,
                ),
                "quantize_4bit(compress_statistics=True)",
            )
            state2 = QuantState(absmax=absmax2, code=codebook.dynamic_code(dev), blocksize=DQ_BLOCKSIZE, dtype=torch.float32)
            state = QuantState(absmax_q, A.shape, code, blocksize, quant_type, A.dtype, offset=offset, state2=state2)
        else:
            state = QuantState(am, A.shape, code, blocksize, quant_type, A.dtype)
    if home != dev:
        packed = packed.to(home)
        state.to(home)
        if home.type == "cpu":
            torch.cuda.current_stream(dev).synchronize()
    return packed, state


@torch.no_grad()
def dequantize_4bit(
    A: torch.Tensor,
    quant_state: Optional[QuantState] = None,
    absmax: Optional[torch.Tensor] = None,
    out: Optional[torch.Tensor] = None,
    blocksize: int = 64,
    quant_type: str = "nf4",
    *,
    out_dtype: Optional[torch.dtype] = None,
) -> torch.Tensor:
    """Blockwise NF4 dequantization to ``quant_state.dtype`` in ``quant_state.shape``.

    ``out_dtype`` overrides the output dtype (fp16/bf16/fp32) without touching
    the state, e.g. to dequantize an fp16 payload straight to bf16.
    """
    if quant_state is None:
        raise ValueError("dequantize_4bit: quant_state is required")
    qs = quant_state
    _check_quant_type(qs.quant_type or quant_type)
    home = A.device
    dev = _compute_device(A, "dequantize_4bit")
    packed = A.to(dev, non_blocking=True)
    if not packed.is_contiguous():
        packed = packed.contiguous()
    shape = tuple(qs.shape)
    n = 1
    for s in shape:
        n *= int(s)
    dtype = out_dtype or qs.dtype or torch.float16
    if dtype not in _lib.DTYPE_CODE:
        raise ValueError(f"dequantize_4bit: unsupported output dtype {dtype}")
    if packed.numel() < (n + 1) // 2:
        raise ValueError(f"dequantize_4bit: packed has {packed.numel()} bytes, need {(n + 1) // 2}")
    res = out if out is not None else torch.empty(shape, dtype=dtype, device=dev)
    if res.dtype != dtype or res.numel() != n or res.device != dev or not res.is_contiguous():
        raise ValueError("dequantize_4bit: out has the wrong dtype, size, device or layout")
    code = qs.code if qs.code is not None else codebook.nf4_code(dev)
    code = _f32_on(code, dev)
    if code.numel() != 16:
        raise ValueError(f"dequantize_4bit: NF4 code must have 16 entries, got {code.numel()}")
    L = _lib.lib()
    with torch.cuda.device(dev):
        st = _lib.stream_of(dev)
        if qs.nested:
            s2 = qs.state2
            absmax_q = qs.absmax.to(dev, non_blocking=True)
            if absmax_q.dtype != torch.uint8:
                raise ValueError("dequantize_4bit: nested state needs uint8 absmax")
            absmax2 = _f32_on(s2.absmax, dev)
            code2 = _f32_on(s2.code, dev)
            offset = _f32_on(qs.offset.reshape(()), dev)
            _lib.check(
                L.stratum_nf4_dequantize_dq(
                    _lib.ptr(packed), _lib.ptr(absmax_q), _lib.ptr(absmax2), _lib.ptr(code2), _lib.ptr(offset),
                    int(s2.blocksize), _lib.ptr(code), n, int(qs.blocksize), _lib.ptr(res), _lib.DTYPE_CODE[dtype], st,
                ),
                "dequantize_4bit",
            )
        else:
            am = _f32_on(qs.absmax, dev)
            _lib.check(
                L.stratum_nf4_dequantize(
                    _lib.ptr(packed), _lib.ptr(am), _lib.ptr(code), n, int(qs.blocksize), _lib.ptr(res),
                    _lib.DTYPE_CODE[dtype], st,
                ),
                "dequantize_4bit",
            )
    if home != dev:
        res = res.to(home)
    return res


class _Nf4Tensor(__import__("ctypes").Structure):
    """``stratum_nf4_tensor`` of include/stratum_nf4.h."""

    _fields_ = [("packed", _lib._vp), ("absmax", _lib._vp), ("absmax_q", _lib._vp), ("absmax2", _lib._vp),
                ("code2", _lib._vp), ("offset", _lib._vp), ("n", _lib._i64), ("out", _lib._vp)]


def dequantize_4bit_many(items, *, out_dtype: Optional[torch.dtype] = None) -> list[torch.Tensor]:
    """Dequantize several NF4 tensors with one launch per 32 of the same kind.

    ``items``: sequence of ``(A, quant_state)`` or ``(A, quant_state, out)``, all on
    one CUDA device with the same blocksize and NF4 code.  Returns the outputs
    (``quant_state.dtype`` / ``out_dtype``, ``quant_state.shape``), equal to what
    :func:`dequantize_4bit` returns for each.  Used by ``upload.ensure_weights``
    to dequantize a whole layer at once.
    """
    items = list(items)
    if not items:
        return []
    first_qs = items[0][1]
    dev = _compute_device(items[0][0], "dequantize_4bit_many")
    bs = int(first_qs.blocksize)
    bs2 = 256
    dtype = out_dtype or first_qs.dtype or torch.float16
    if dtype not in _lib.DTYPE_CODE:
        raise ValueError(f"dequantize_4bit_many: unsupported output dtype {dtype}")
    code = first_qs.code if first_qs.code is not None else codebook.nf4_code(dev)
    code = _f32_on(code, dev)
    keep: list[torch.Tensor] = [code]
    descs = (_Nf4Tensor * len(items))()
    outs: list[torch.Tensor] = []
    for i, item in enumerate(items):
        A, qs = item[0], item[1]
        out = item[2] if len(item) > 2 else None
        _check_quant_type(qs.quant_type or "nf4")
        if int(qs.blocksize) != bs:
            raise ValueError("dequantize_4bit_many: all tensors need the same blocksize")
        if A.device != dev:
            raise ValueError("dequantize_4bit_many: all tensors must be on one device")
        shape = tuple(qs.shape)
        n = 1
        for s in shape:
            n *= int(s)
        packed = A if A.is_contiguous() else A.contiguous()
        if packed.numel() < (n + 1) // 2:
            raise ValueError(f"dequantize_4bit_many: tensor {i}: packed has {packed.numel()} bytes, need {(n + 1) // 2}")
        res = out if out is not None else torch.empty(shape, dtype=dtype, device=dev)
        if res.dtype != dtype or res.numel() != n or res.device != dev or not res.is_contiguous():
            raise ValueError(f"dequantize_4bit_many: tensor {i}: out has the wrong dtype, size, device or layout")
        d = descs[i]
        d.packed, d.n, d.out = packed.data_ptr(), n, res.data_ptr()
        keep += [packed, res]
        if qs.nested:
            s2 = qs.state2
            bs2 = int(s2.blocksize)
            aq = qs.absmax.to(dev, non_blocking=True)
            a2, c2, off = _f32_on(s2.absmax, dev), _f32_on(s2.code, dev), _f32_on(qs.offset.reshape(()), dev)
            keep += [aq, a2, c2, off]
            d.absmax_q, d.absmax2, d.code2, d.offset = aq.data_ptr(), a2.data_ptr(), c2.data_ptr(), off.data_ptr()
        else:
            am = _f32_on(qs.absmax, dev)
            keep.append(am)
            d.absmax = am.data_ptr()
        outs.append(res)
    L = _lib.lib()
    with torch.cuda.device(dev):
        _lib.check(L.stratum_nf4_dequantize_many(__import__("ctypes").cast(descs, _lib._vp), len(items), _lib.ptr(code),
                                                 bs, bs2, _lib.DTYPE_CODE[dtype],
                                                 _lib.stream_of(dev)), "dequantize_4bit_many")
    del keep
    return outs
