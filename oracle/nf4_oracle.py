"""CPU oracle for the NF4 frozen-weight path.  TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline legs may import it.
The product path (``stratum_b200``) never imports, links or executes anything
under ``oracle/``.

PARITY UNPINNED.  The reference (h4rm0n1c/stratum) does not implement the NF4
arithmetic itself.  It calls ``bitsandbytes.functional.quantize_4bit`` and
``dequantize_4bit`` (stratum/upload.py:355-369, :1021-1040;
stratum/nf4_linear.py:44-46).  bitsandbytes is an unpinned, un-vendored
dependency (pyproject.toml:19, Dockerfile:51) that is absent here and on the GPU
box, and the reference's own tests replace it with a zero-returning fake
(tests/test_upload.py:361-398), so no golden vector pins the codec numbers.
This file restates the published algorithm instead:

* the 16 NF4 levels of QLoRA (Dettmers et al. 2023, arXiv 2305.14314,
  Appendix E), which bitsandbytes uses for ``quant_type="nf4"``;
* bitsandbytes' blockwise 4-bit quantizer: per-block absmax over ``blocksize``
  consecutive elements of the flattened tensor, scale by the fp32 reciprocal of
  the absmax, pick the level by comparing against the fp32 midpoints between
  adjacent levels with strict ``>`` (an all-zero block gives 0*inf = NaN, which
  fails every comparison and lands on level 0), two codes per byte with the
  first element in the high nibble, padding elements of a ragged tail quantized
  as 0.0;
* bitsandbytes' blockwise dequantizer: ``out = dtype(fp32(level[q] * absmax))``;
* double quantization (``compress_statistics=True``): offset = mean(absmax),
  8-bit blockwise quantization (blocksize 256) of ``absmax - offset`` with the
  signed dynamic code (Dettmers et al. 2021, "8-bit Optimizers via Block-wise
  Quantization"), dequantized as ``fp32(fp32(code2[q] * absmax2) + offset)``.

The reference itself never enables double quantization (it hard-codes
``compress_statistics=False`` at stratum/upload.py:368 and :726), so the
double-quant definitions below (the mean's summation order and the
nearest-code rule) are this framework's own, stated exactly so that the GPU
kernels can be held bit-exact to them.
"""

from __future__ import annotations

import math

import numpy as np

# QLoRA NF4 levels (arXiv 2305.14314, Appendix E).  Every value is an exact
# float32; index 7 is 0.0, index 0 is -1.0 and index 15 is 1.0.
NF4_LEVELS = np.array(
    [
        -1.0,
        -0.6961928009986877,
        -0.5250730514526367,
        -0.39491748809814453,
        -0.28444138169288635,
        -0.18477343022823334,
        -0.09105003625154495,
        0.0,
        0.07958029955625534,
        0.16093020141124725,
        0.24611230194568634,
        0.33791524171829224,
        0.44070982933044434,
        0.5626170039176941,
        0.7229568362236023,
        1.0,
    ],
    dtype=np.float32,
)


def midpoints_f32(levels: np.ndarray) -> np.ndarray:
    """fp32 thresholds: each midpoint of adjacent sorted levels, computed in
    float64 and rounded once to float32 (round-to-nearest-even).

    This is what a float32 tensor compared against Python-float thresholds
    gets (the threshold is cast float64 -> float32), i.e. bitsandbytes'
    torch-level CPU quantizer.
    """
    lv = levels.astype(np.float64)
    return ((lv[:-1] + lv[1:]) * 0.5).astype(np.float32)


def _nearest_f32_to_fraction(target, guess: np.float32) -> np.float32:
    from fractions import Fraction

    cands = [np.nextafter(guess, np.float32(-np.inf)), guess, np.nextafter(guess, np.float32(np.inf))]
    def key(c):
        d = abs(Fraction(float(c)) - target)
        odd = int(np.asarray(c, np.float32).view(np.uint32)) & 1
        return (d, odd)  # ties go to the even mantissa
    return min(cands, key=key)


def decimal_literal_thresholds(levels: np.ndarray) -> np.ndarray:
    """fp32 thresholds as the bitsandbytes CUDA decision tree has them.

    That tree writes each midpoint as a float literal: the shortest decimal
    that round-trips the float64 midpoint (Python ``repr``), suffixed ``f``,
    which the compiler rounds directly from decimal to float32.  Where the
    float64 midpoint is an exact float32 tie, the decimal sits slightly off
    the tie and may round to the other neighbour than
    :func:`midpoints_f32` does (4 of the 15 NF4 thresholds differ by one
    float32 ulp).
    """
    from decimal import Decimal
    from fractions import Fraction

    lv = levels.astype(np.float64)
    out = []
    for i in range(lv.size - 1):
        m = float((lv[i] + lv[i + 1]) * 0.5)
        exact = Fraction(Decimal(repr(m)))
        out.append(_nearest_f32_to_fraction(exact, np.float32(m)))
    return np.array(out, dtype=np.float32)


# Default: the CUDA-kernel thresholds (bitsandbytes' reference kernel).
NF4_THRESHOLDS_CUDA = decimal_literal_thresholds(NF4_LEVELS)
NF4_THRESHOLDS_MIDPOINT = midpoints_f32(NF4_LEVELS)
NF4_THRESHOLDS = NF4_THRESHOLDS_CUDA


def nearest_code(scaled: np.ndarray, thresholds: np.ndarray) -> np.ndarray:
    """Index of the nearest level: the number of thresholds strictly below x.

    Equivalent to the bitsandbytes NF4 decision tree (a chain of ``x > t``
    tests).  NaN compares false everywhere and maps to index 0.
    """
    s = np.asarray(scaled, dtype=np.float32)
    idx = np.searchsorted(thresholds, s, side="left").astype(np.uint8)
    idx[np.isnan(s)] = 0
    return idx


def _as_f32_flat(a) -> np.ndarray:
    """Flatten fp16/bf16/fp32 input (numpy array or torch tensor) to fp32."""
    try:
        import torch

        if isinstance(a, torch.Tensor):
            return a.detach().reshape(-1).to(torch.float32).cpu().numpy()
    except ImportError:  # pragma: no cover - torch is always present here
        pass
    return np.asarray(a).reshape(-1).astype(np.float32)


def blockwise_absmax(x: np.ndarray, blocksize: int) -> np.ndarray:
    """Per-block max |x| over ``blocksize`` consecutive elements (ragged tail ok)."""
    n = x.size
    nb = (n + blocksize - 1) // blocksize
    pad = nb * blocksize - n
    xp = np.concatenate([np.abs(x), np.zeros(pad, np.float32)]) if pad else np.abs(x)
    return xp.reshape(nb, blocksize).max(axis=1).astype(np.float32)


def quantize_nf4(a, blocksize: int = 64, thresholds: np.ndarray | None = None):
    """NF4-quantize ``a`` (any shape, fp16/bf16/fp32); returns (packed u8 [ceil(n/2)], absmax f32 [nb]).

    Follows bitsandbytes' blockwise 4-bit quantizer as called at
    stratum/upload.py:367-369 (blocksize 64, quant_type "nf4").
    ``thresholds`` defaults to :data:`NF4_THRESHOLDS` (the CUDA-kernel set).
    """
    thresholds = NF4_THRESHOLDS if thresholds is None else np.asarray(thresholds, np.float32)
    x = _as_f32_flat(a)
    n = x.size
    nb = (n + blocksize - 1) // blocksize
    absmax = blockwise_absmax(x, blocksize)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        inv = np.float32(1.0) / absmax  # fp32 reciprocal, inf for zero blocks
        pad = nb * blocksize - n
        xp = np.concatenate([x, np.zeros(pad, np.float32)]) if pad else x
        scaled = (xp.reshape(nb, blocksize) * inv[:, None]).reshape(-1)[: n + (n & 1)]
    q = nearest_code(scaled, thresholds)
    packed = ((q[0::2] << 4) | q[1::2]).astype(np.uint8)
    return packed, absmax


def unpack_nibbles(packed: np.ndarray, n: int) -> np.ndarray:
    """Codes in element order (first element of each byte is its high nibble)."""
    p = np.asarray(packed, dtype=np.uint8).reshape(-1)
    q = np.empty(p.size * 2, np.uint8)
    q[0::2] = p >> 4
    q[1::2] = p & 0x0F
    return q[:n]


def dequantize_nf4(packed, absmax, n: int, blocksize: int = 64, levels=NF4_LEVELS, out_dtype="float16"):
    """``out[i] = out_dtype(fp32(levels[q_i] * absmax[i // blocksize]))``.

    bitsandbytes' blockwise dequantizer as called at stratum/upload.py:1038 and
    stratum/nf4_linear.py:44-46.  Returns a numpy array of ``out_dtype``
    ("float16", "bfloat16" as raw uint16 bits via :func:`f32_to_bf16_bits`, or
    "float32").
    """
    q = unpack_nibbles(packed, n)
    am = np.asarray(absmax, dtype=np.float32).reshape(-1)
    blk = np.arange(n) // blocksize
    v = (np.asarray(levels, np.float32)[q] * am[blk]).astype(np.float32)
    if out_dtype == "float32":
        return v
    if out_dtype == "float16":
        return v.astype(np.float16)
    if out_dtype == "bfloat16":
        return f32_to_bf16_bits(v)
    raise ValueError(out_dtype)


def f32_to_bf16_bits(v: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bfloat16, returned as uint16 bit patterns."""
    u = np.asarray(v, np.float32).view(np.uint32).astype(np.uint64)
    is_nan = np.isnan(np.asarray(v, np.float32))
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    out = rounded.astype(np.uint16)
    out[is_nan] = ((u[is_nan] >> 16) | 0x40).astype(np.uint16)
    return out


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------------------
# Double quantization of the absmax (compress_statistics=True)
# ---------------------------------------------------------------------------

def dynamic_code_signed() -> np.ndarray:
    """The signed 8-bit dynamic code (256 sorted float32 values).

    Restates bitsandbytes' dynamic data type (Dettmers et al. 2021): for each
    decimal exponent e = 0..6 the interval [0.1, 1] is split into 2**e equal
    parts (float32 linspace of 2**e + 1 points); the part midpoints, scaled by
    10**(e-6), are taken with both signs; 0 and 1.0 complete the 256 values.
    The arithmetic is float32 throughout (linspace, midpoint, scale), like the
    torch implementation it restates.
    """
    import torch

    vals: list[float] = []
    for e in range(7):
        pts = torch.linspace(0.1, 1.0, 2**e + 1, dtype=torch.float32)
        mids = (pts[:-1] + pts[1:]) / 2.0
        scaled = (10 ** (e - 6)) * mids
        vals += scaled.tolist()
        vals += (-(10 ** (e - 6)) * mids).tolist()
    vals += [0.0, 1.0]
    assert len(vals) == 256
    return np.sort(np.array(vals, dtype=np.float32))


DQ_BLOCKSIZE = 256
MEAN_CHUNK = 1024


def dq_mean(absmax: np.ndarray) -> np.float32:
    """Deterministic mean of the absmax vector used as the double-quant offset.

    Sequential float64 sums over consecutive chunks of 1024 elements, then a
    sequential float64 sum of the chunk sums, divided by n in float64 and
    rounded once to float32.  The GPU kernel performs the same operations in
    the same order, so the offset is bit-identical.
    """
    a = np.asarray(absmax, np.float32).astype(np.float64)
    n = a.size
    total = 0.0
    for c0 in range(0, n, MEAN_CHUNK):
        chunk = a[c0 : c0 + MEAN_CHUNK]
        part = float(np.cumsum(chunk)[-1]) if chunk.size else 0.0
        total = total + part
    return np.float32(total / n)


def quantize_absmax_dq(absmax: np.ndarray, code2: np.ndarray | None = None, blocksize2: int = DQ_BLOCKSIZE):
    """Double-quantize a float32 absmax vector.

    Returns (absmax_q u8 [nb], absmax2 f32 [ceil(nb/256)], code2 f32 [256], offset f32).
    ``absmax_q[b]`` is the nearest entry of the sorted code to
    ``(absmax[b] - offset) * (1 / absmax2[b // 256])`` under the same
    strict-midpoint rule as the NF4 levels.
    """
    code2 = dynamic_code_signed() if code2 is None else np.asarray(code2, np.float32)
    am = np.asarray(absmax, np.float32)
    offset = dq_mean(am)
    centered = (am - offset).astype(np.float32)
    absmax2 = blockwise_absmax(centered, blocksize2)
    nb2 = absmax2.size
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        inv2 = np.float32(1.0) / absmax2
        pad = nb2 * blocksize2 - am.size
        cp = np.concatenate([centered, np.zeros(pad, np.float32)]) if pad else centered
        scaled = (cp.reshape(nb2, blocksize2) * inv2[:, None]).reshape(-1)[: am.size]
    q = nearest_code(scaled, midpoints_f32(code2))
    return q.astype(np.uint8), absmax2, code2, offset


def dequantize_absmax_dq(absmax_q, absmax2, code2, offset, blocksize2: int = DQ_BLOCKSIZE) -> np.ndarray:
    q = np.asarray(absmax_q, np.uint8).reshape(-1)
    blk = np.arange(q.size) // blocksize2
    v = (np.asarray(code2, np.float32)[q] * np.asarray(absmax2, np.float32)[blk]).astype(np.float32)
    return (v + np.float32(offset)).astype(np.float32)


def quantize_nf4_dq(a, blocksize: int = 64):
    """NF4 + double quant.  Returns (packed, absmax_q, absmax2, code2, offset)."""
    packed, absmax = quantize_nf4(a, blocksize)
    absmax_q, absmax2, code2, offset = quantize_absmax_dq(absmax)
    return packed, absmax_q, absmax2, code2, offset


def dequantize_nf4_dq(packed, absmax_q, absmax2, code2, offset, n, blocksize=64, out_dtype="float16"):
    absmax = dequantize_absmax_dq(absmax_q, absmax2, code2, offset)
    return dequantize_nf4(packed, absmax, n, blocksize, out_dtype=out_dtype)


# ---------------------------------------------------------------------------
# Floating-point references for the GEMM / LoRA path (torch fp32 on CPU)
# ---------------------------------------------------------------------------

def nf4_linear_reference(x, w_deq, bias=None, lora_A=None, lora_B=None, scaling=1.0, dy=None):
    """fp32 reference of ``NF4Linear`` + PEFT LoRA, forward and backward.

    y = x @ W^T + bias + scaling * (x @ A^T) @ B^T  (PEFT lora.Linear with
    dropout 0; scaling = alpha / r, scripts/train.py:568-573), W frozen.
    Returns dict with y and, when ``dy`` is given, dx, dA, dB (all fp32).
    """
    import torch

    xf = x.detach().to(torch.float32).clone().requires_grad_(dy is not None)
    wf = w_deq.detach().to(torch.float32)
    y = xf @ wf.t()
    if bias is not None:
        y = y + bias.detach().to(torch.float32)
    a_f = b_f = None
    if lora_A is not None:
        a_f = lora_A.detach().to(torch.float32).clone().requires_grad_(dy is not None)
        b_f = lora_B.detach().to(torch.float32).clone().requires_grad_(dy is not None)
        y = y + scaling * ((xf @ a_f.t()) @ b_f.t())
    out = {"y": y.detach()}
    if dy is not None:
        y.backward(dy.detach().to(torch.float32))
        out["dx"] = xf.grad
        if a_f is not None:
            out["dA"] = a_f.grad
            out["dB"] = b_f.grad
    return out


def relative_error(a, b) -> float:
    """||a - b|| / max(||b||, tiny) in float64 (Frobenius)."""
    import torch

    a64 = a.detach().to(torch.float64).cpu()
    b64 = b.detach().to(torch.float64).cpu()
    den = max(float(torch.linalg.vector_norm(b64)), 1e-30)
    return float(torch.linalg.vector_norm(a64 - b64)) / den


def threshold_ties() -> list[int]:
    """Indices of NF4 midpoints that are exact float32 ties (halfway between two float32s).

    Only at these indices can the two threshold conventions
    (:data:`NF4_THRESHOLDS_CUDA`, :data:`NF4_THRESHOLDS_MIDPOINT`) differ.
    """
    from fractions import Fraction

    lv = NF4_LEVELS.astype(np.float64)
    ties = []
    for i in range(15):
        m = (lv[i] + lv[i + 1]) * 0.5
        f = np.float32(m)
        for nb in (np.nextafter(f, np.float32(-np.inf)), np.nextafter(f, np.float32(np.inf))):
            if Fraction(float(m)) == (Fraction(float(f)) + Fraction(float(nb))) / 2:
                ties.append(i)
    return ties
