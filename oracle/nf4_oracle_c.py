"""ctypes wrapper of the C oracle (oracle/nf4_oracle.c).  TEST INFRASTRUCTURE ONLY.

Used by tests/ for full-size bit-exact checks and by bench.py's CPU-baseline
legs for timing on all host cores.  Parity unpinned: see oracle/nf4_oracle.py.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

from . import nf4_oracle as O

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "libnf4_oracle.so"

_F32, _F16, _BF16 = 0, 1, 2
_vp = ctypes.c_void_p


def build() -> Path:
    src = HERE / "nf4_oracle.c"
    if not LIB.exists() or LIB.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


class OracleC:
    def __init__(self, path: Path):
        self.lib = ctypes.CDLL(str(path))
        L = self.lib
        L.nf4o_quantize.argtypes = [_vp, ctypes.c_int, ctypes.c_int64, ctypes.c_int, _vp, _vp, _vp, ctypes.c_int]
        L.nf4o_dequantize.argtypes = [_vp, _vp, _vp, ctypes.c_int64, ctypes.c_int, _vp, ctypes.c_int, ctypes.c_int]
        L.nf4o_quantize_absmax_dq.argtypes = [_vp, ctypes.c_int64, ctypes.c_int, _vp, _vp, _vp, _vp, ctypes.c_int]
        L.nf4o_dequantize_dq.argtypes = [_vp, _vp, _vp, _vp, ctypes.c_float, ctypes.c_int, _vp, ctypes.c_int64,
                                         ctypes.c_int, _vp, ctypes.c_int, ctypes.c_int]
        L.nf4o_dq_mean.argtypes = [_vp, ctypes.c_int64]
        L.nf4o_dq_mean.restype = ctypes.c_float
        self.threads = len(os.sched_getaffinity(0))

    @staticmethod
    def _p(a: np.ndarray):
        return ctypes.c_void_p(a.ctypes.data)

    @staticmethod
    def _src(x):
        """numpy view + dtype code of fp16/bf16/fp32 input (torch tensors accepted)."""
        try:
            import torch

            if isinstance(x, torch.Tensor):
                x = x.detach().contiguous().cpu()
                if x.dtype == torch.bfloat16:
                    return x.view(torch.int16).numpy().view(np.uint16).reshape(-1), _BF16
                x = x.numpy()
        except ImportError:  # pragma: no cover
            pass
        x = np.ascontiguousarray(x).reshape(-1)
        if x.dtype == np.float16:
            return x, _F16
        if x.dtype == np.float32:
            return x, _F32
        raise TypeError(x.dtype)

    def quantize(self, x, blocksize=64, thresholds=None, threads=None):
        a, code = self._src(x)
        n = a.size
        thr = np.ascontiguousarray(O.NF4_THRESHOLDS if thresholds is None else thresholds, np.float32)
        packed = np.empty((n + 1) // 2, np.uint8)
        absmax = np.empty((n + blocksize - 1) // blocksize, np.float32)
        self.lib.nf4o_quantize(self._p(a), code, n, blocksize, self._p(thr), self._p(packed), self._p(absmax),
                               threads or self.threads)
        return packed, absmax

    def dequantize(self, packed, absmax, n, blocksize=64, out_dtype="float16", threads=None):
        lv = np.ascontiguousarray(O.NF4_LEVELS)
        out, code = self._out(n, out_dtype)
        self.lib.nf4o_dequantize(self._p(np.ascontiguousarray(packed)), self._p(np.ascontiguousarray(absmax, np.float32)),
                                 self._p(lv), n, blocksize, self._p(out), code, threads or self.threads)
        return out

    def quantize_absmax_dq(self, absmax, threads=None):
        am = np.ascontiguousarray(absmax, np.float32)
        code2 = O.dynamic_code_signed()
        thr2 = np.ascontiguousarray(O.midpoints_f32(code2))
        q = np.empty(am.size, np.uint8)
        a2 = np.empty((am.size + 255) // 256, np.float32)
        off = np.empty(1, np.float32)
        self.lib.nf4o_quantize_absmax_dq(self._p(am), am.size, 256, self._p(thr2), self._p(q), self._p(a2),
                                         self._p(off), threads or self.threads)
        return q, a2, code2, np.float32(off[0])

    def dequantize_dq(self, packed, absmax_q, absmax2, code2, offset, n, blocksize=64, out_dtype="float16", threads=None):
        lv = np.ascontiguousarray(O.NF4_LEVELS)
        out, code = self._out(n, out_dtype)
        self.lib.nf4o_dequantize_dq(self._p(np.ascontiguousarray(packed)), self._p(np.ascontiguousarray(absmax_q)),
                                    self._p(np.ascontiguousarray(absmax2, np.float32)),
                                    self._p(np.ascontiguousarray(code2, np.float32)), float(offset), 256, self._p(lv), n,
                                    blocksize, self._p(out), code, threads or self.threads)
        return out

    @staticmethod
    def _out(n, out_dtype):
        if out_dtype == "float16":
            return np.empty(n, np.float16), _F16
        if out_dtype == "bfloat16":
            return np.empty(n, np.uint16), _BF16
        if out_dtype == "float32":
            return np.empty(n, np.float32), _F32
        raise ValueError(out_dtype)


_instance = None


def load() -> OracleC:
    global _instance
    if _instance is None:
        _instance = OracleC(build())
    return _instance
