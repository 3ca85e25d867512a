"""NF4 codebook tables used by the kernels (levels, thresholds, dynamic code).

The kernels take these as small device tensors, so callers can choose between
the two threshold conventions bitsandbytes has:

* ``"cuda"`` (default): the midpoints as bitsandbytes' CUDA decision tree
  writes them, float literals rounded directly from their shortest decimal
  form to float32;
* ``"midpoint"``: each float64 midpoint rounded once to float32, which is
  what bitsandbytes' torch-level CPU quantizer compares against.

They differ by one float32 ulp at 4 of the 15 thresholds (indices 0, 8, 12,
14); only a scaled weight that lands exactly on one of those four values is
quantized differently.
"""

from __future__ import annotations

import threading
from decimal import Decimal
from fractions import Fraction

import numpy as np
import torch

# QLoRA NF4 levels (arXiv 2305.14314, Appendix E); bitsandbytes quant_type "nf4".
NF4_LEVELS = (
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
)

THRESHOLD_CONVENTIONS = ("cuda", "midpoint")


def nf4_levels_np() -> np.ndarray:
    return np.array(NF4_LEVELS, dtype=np.float32)


def _round_fraction_to_f32(target: Fraction, guess: float) -> np.float32:
    g = np.float32(guess)
    cands = (np.nextafter(g, np.float32(-np.inf)), g, np.nextafter(g, np.float32(np.inf)))
    return min(cands, key=lambda c: (abs(Fraction(float(c)) - target), int(np.asarray(c).view(np.uint32)) & 1))


def thresholds_np(levels=None, convention: str = "cuda") -> np.ndarray:
    """Sorted float32 thresholds between adjacent levels (len(levels) - 1 values)."""
    lv = np.asarray(nf4_levels_np() if levels is None else levels, np.float32).astype(np.float64)
    mids = (lv[:-1] + lv[1:]) * 0.5
    if convention == "midpoint":
        return mids.astype(np.float32)
    if convention == "cuda":
        return np.array(
            [_round_fraction_to_f32(Fraction(Decimal(repr(float(m)))), float(m)) for m in mids], dtype=np.float32
        )
    raise ValueError(f"unknown threshold convention {convention!r}; expected one of {THRESHOLD_CONVENTIONS}")


def dynamic_code_np() -> np.ndarray:
    """Signed 8-bit dynamic code (256 sorted float32 values) for double quantization.

    bitsandbytes' dynamic data type with 7 exponent bits: for decimal
    exponents e = 0..6 the interval [0.1, 1] is cut into 2**e equal parts
    (float32 linspace) whose midpoints, scaled by 10**(e - 6), are taken with
    both signs; 0 and 1 complete the table.
    """
    vals: list[float] = []
    for e in range(7):
        pts = torch.linspace(0.1, 1.0, 2**e + 1, dtype=torch.float32)
        mids = (pts[:-1] + pts[1:]) / 2.0
        vals += ((10 ** (e - 6)) * mids).tolist()
        vals += (-(10 ** (e - 6)) * mids).tolist()
    vals += [0.0, 1.0]
    return np.sort(np.array(vals, dtype=np.float32))


def dynamic_thresholds_np() -> np.ndarray:
    c = dynamic_code_np().astype(np.float64)
    return ((c[:-1] + c[1:]) * 0.5).astype(np.float32)


_cache: dict = {}
_lock = threading.Lock()


def _device_key(device) -> torch.device:
    d = torch.device(device)
    if d.type == "cuda" and d.index is None:
        d = torch.device("cuda", torch.cuda.current_device())
    return d


def _cached(name: str, device, make) -> torch.Tensor:
    d = _device_key(device)
    key = (name, d)
    t = _cache.get(key)
    if t is None:
        with _lock:
            t = _cache.get(key)
            if t is None:
                t = torch.from_numpy(make()).to(d)
                _cache[key] = t
    return t


def nf4_code(device="cpu") -> torch.Tensor:
    """The 16 NF4 levels as a float32 tensor (what QuantState.code holds)."""
    return _cached("levels", device, nf4_levels_np)


def nf4_thresholds(device, convention: str = "cuda") -> torch.Tensor:
    if convention not in THRESHOLD_CONVENTIONS:
        raise ValueError(f"unknown threshold convention {convention!r}; expected one of {THRESHOLD_CONVENTIONS}")
    return _cached(f"thr-{convention}", device, lambda: thresholds_np(convention=convention))


def dynamic_code(device="cpu") -> torch.Tensor:
    return _cached("code2", device, dynamic_code_np)


def dynamic_thresholds(device) -> torch.Tensor:
    return _cached("thr2", device, dynamic_thresholds_np)
