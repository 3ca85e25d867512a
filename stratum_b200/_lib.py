"""ctypes binding of libstratum_nf4.so (the C ABI in include/stratum_nf4.h).

There is no CPU fallback: every product entry point goes through this library,
and a missing library or a missing CUDA device raises instead of degrading.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libstratum_nf4.so"

STRATUM_OK = 0
STRATUM_ERR_INVALID = 1
STRATUM_ERR_UNSUPPORTED = 2
STRATUM_ERR_CUDA = 3
STRATUM_ERR_TIMEOUT = 4
STRATUM_ERR_NCCL = 5

DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_f32 = ctypes.c_float
_sz = ctypes.c_size_t

# name -> (restype, argtypes); must match include/stratum_nf4.h
SIGNATURES: dict[str, tuple] = {
    "stratum_abi_version": (_int, []),
    "stratum_last_error": (ctypes.c_char_p, []),
    "stratum_launch_count": (ctypes.c_uint64, []),
    "stratum_device_status_detail": (_int, [_vp, _vp]),
    "stratum_device_status_record": (_int, [_vp, _int, _vp]),
    "stratum_set_wait_limit_ns": (_int, [ctypes.c_uint64, _vp]),
    "stratum_wait_selftest": (_int, [_vp]),
    "stratum_nf4_gemm_set_kernel": (_int, [_int]),
    "stratum_set_device": (_int, [_int]),
    "stratum_nf4_quantize": (_int, [_vp, _int, _i64, _int, _vp, _vp, _vp, _vp]),
    "stratum_nf4_dq_workspace_bytes": (_sz, [_i64]),
    "stratum_nf4_quantize_absmax_dq": (_int, [_vp, _i64, _int, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "stratum_nf4_dequantize": (_int, [_vp, _vp, _vp, _i64, _int, _vp, _int, _vp]),
    "stratum_nf4_dequantize_dq": (_int, [_vp, _vp, _vp, _vp, _vp, _int, _vp, _i64, _int, _vp, _int, _vp]),
    "stratum_device_status": (_int, [ctypes.POINTER(ctypes.c_int), _int, _vp]),
    "stratum_nf4_quantize_dq_noalloc": (_int, [_vp, _int, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "stratum_nf4_dequantize_many": (_int, [_vp, _int, _vp, _int, _int, _int, _vp]),
    "stratum_nf4_gemm_fwd": (_int, [_vp, _int, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _vp, _int, _vp,
                                    _vp, _int, _vp, _vp]),
    "stratum_nf4_gemm_dx": (_int, [_vp, _int, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _vp, _vp, _int,
                                   _vp, _vp]),
    "stratum_nf4_gemm_swiglu_fwd": (_int, [_vp, _int, _i64, _i64, _vp, _vp, _vp, _i64, _vp, _vp, _vp, _int, _vp, _vp,
                                           _vp, _vp]),
    "stratum_nf4_gemm_dx_pair": (_int, [_vp, _int, _i64, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _int, _vp, _vp]),
    # include/stratum_moe.h
    "stratum_moe_route_workspace_bytes": (_sz, [_i64, _int]),
    "stratum_moe_route": (_int, [_vp, _i64, _int, _int, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "stratum_moe_gather_rows": (_int, [_vp, _i64, _vp, _i64, _vp, _vp]),
    "stratum_nf4_grouped_table_bytes": (_sz, [_i64, _int, _i64]),
    "stratum_nf4_grouped_fwd": (_int, [_vp, _int, _i64, _int, _vp, _int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _int,
                                       _int, _vp, _vp, _vp, _vp, _sz, _vp]),
    "stratum_nf4_grouped_dx": (_int, [_vp, _int, _i64, _int, _vp, _int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _int,
                                      _vp, _vp, _sz, _vp]),
    "stratum_moe_combine": (_int, [_vp, _int, _vp, _vp, _vp, _int, _i64, _int, _i64, _vp, _vp]),
    "stratum_moe_combine_grad": (_int, [_vp, _int, _vp, _vp, _vp, _vp, _int, _vp, _i64, _i64, _vp, _vp, _vp]),
    "stratum_swiglu_grad": (_int, [_vp, _vp, _int, _i64, _i64, _vp, _vp]),
    # include/stratum_layers.h
    "stratum_rmsnorm_fwd": (_int, [_vp, _vp, _int, _i64, _i64, _f32, _vp, _vp, _vp]),
    "stratum_rmsnorm_bwd": (_int, [_vp, _vp, _vp, _vp, _int, _i64, _i64, _vp, _vp]),
    "stratum_rope_to_heads": (_int, [_vp, _vp, _vp, _int, _int, _int, _int, _vp, _vp]),
    "stratum_rope_from_heads": (_int, [_vp, _vp, _vp, _int, _int, _int, _int, _vp, _vp]),
    "stratum_swiglu_fwd": (_int, [_vp, _vp, _int, _i64, _vp, _vp]),
    "stratum_swiglu_bwd": (_int, [_vp, _vp, _vp, _int, _i64, _vp, _vp, _vp]),
    "stratum_swiglu_bwd_cat": (_int, [_vp, _vp, _vp, _int, _i64, _i64, _vp, _vp]),
    "stratum_ce_fwd_grad": (_int, [_vp, _int, _vp, _i64, _i64, _i64, _f32, _vp, _vp]),
}

ABI_VERSION = 1

_lib = None
_lock = threading.Lock()


class StratumError(RuntimeError):
    """A CUDA, NCCL or timeout failure reported by the native library."""


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        from . import _build

        try:
            _build.build()
        except Exception as exc:  # no nvcc: fail loudly, never fall back
            raise RuntimeError(
                f"{LIB_PATH.name} is not built and could not be built ({exc}); "
                "run `python -m stratum_b200._build` on a machine with nvcc"
            ) from exc
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    ver = lib.stratum_abi_version()
    if ver != ABI_VERSION:
        raise RuntimeError(f"{LIB_PATH.name} ABI version {ver} != expected {ABI_VERSION}; rebuild it")
    return lib


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                _lib = _load()
    return _lib


def check(rc: int, what: str) -> None:
    if rc == STRATUM_OK:
        return
    msg = lib().stratum_last_error().decode(errors="replace")
    if rc in (STRATUM_ERR_INVALID, STRATUM_ERR_UNSUPPORTED):
        raise ValueError(f"{what}: {msg}")
    raise StratumError(f"{what}: {msg} (status {rc})")


def ptr(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def stream_of(device: torch.device) -> ctypes.c_void_p:
    """The caller's current stream on ``device``.  The library runs each call on the
    stream's device; for torch's legacy default stream (handle 0), and while the
    stream is being captured into a CUDA graph (when its device cannot be queried),
    the library's own current device is selected here first."""
    dev = torch.device(device)
    index = dev.index if dev.index is not None else torch.cuda.current_device()
    handle = torch.cuda.current_stream(dev).cuda_stream
    # always: a call on another stream may have switched the library's device
    if handle == 0 or torch.cuda.is_current_stream_capturing():
        check(lib().stratum_set_device(index), "set_device")
    return ctypes.c_void_p(handle)


class NF4Weight(ctypes.Structure):
    """``stratum_nf4_weight`` of include/stratum_nf4.h."""

    _fields_ = [("packed", _vp), ("absmax", _vp), ("absmax_q", _vp), ("absmax2", _vp), ("code2", _vp),
                ("offset", _vp)]


def require_cuda(t: torch.Tensor, what: str) -> None:
    if t.device.type != "cuda":
        raise RuntimeError(f"{what}: tensor on {t.device}; the NF4 kernels run on CUDA only (no CPU fallback)")


def device_status(device=None, reset: bool = True) -> int:
    """Status word of the GEMM kernels on ``device`` (0 = no bounded wait gave up)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    out = ctypes.c_int(0)
    with torch.cuda.device(dev):
        check(lib().stratum_device_status(ctypes.byref(out), int(reset), stream_of(dev)), "device_status")
    return out.value


STATUS_WORDS = 72  # ints in the status record (include/stratum_nf4.h)
BAR_BELOW, BAR_ABOVE = 17, 9  # shared-memory words snapshotted around the barrier waited on


def device_status_record(device=None) -> list:
    """The GEMM kernels' whole diagnostic record on ``device`` (see
    ``stratum_device_status_record``), without clearing it."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    rec = (ctypes.c_int * STATUS_WORDS)()
    with torch.cuda.device(dev):
        check(lib().stratum_device_status_record(ctypes.cast(rec, ctypes.c_void_p), STATUS_WORDS, stream_of(dev)),
              "device_status_record")
    return list(rec)


def set_wait_limit_ns(ns: int, device=None) -> None:
    """Limit of the GEMM kernels' bounded device-side waits on ``device`` (0 = the 2 s default)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        check(lib().stratum_set_wait_limit_ns(int(ns), stream_of(dev)), "set_wait_limit_ns")


def wait_selftest(device=None) -> None:
    """Enqueue one bounded wait that gives up (status 0x1f0 after the limit in force)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        check(lib().stratum_wait_selftest(stream_of(dev)), "wait_selftest")


def _u64(lo: int, hi: int) -> int:
    return (lo & 0xffffffff) | ((hi & 0xffffffff) << 32)


def describe_status_record(d: list) -> str:
    """Readable form of a record from :func:`device_status_record` (empty when it
    holds no wait that gave up or rejected tile record)."""
    st = d[0]
    if st != 0 and (st & 0xf00) == 0x100:
        text = (f"first wait to give up: block {d[1]}, thread {d[2]}, SM {d[7]}, parity {d[3]}, barrier at shared "
                f"offset 0x{d[4] & 0xffffffff:x}, state 0x{_u64(d[5], d[6]):016x}; the wait lasted "
                f"{_u64(d[8], d[9]) / 1e9:.3f} s by %globaltimer and {d[10] & 0xffffffff} SM cycles")
        n = BAR_BELOW + 1 + BAR_ABOVE
        if len(d) >= 12 + 2 * n:
            snap = [_u64(d[12 + 2 * i], d[13 + 2 * i]) for i in range(n)]
            text += (f"; shared-memory words from {BAR_BELOW} below it to {BAR_ABOVE} above: "
                     + " ".join(f"{v:016x}" for v in snap))
        return text
    if st == 0x202 and d[6] != 0:
        return f"bad tile record: block {d[1]}, tile {d[2]}: expert {d[3]}, column tile {d[4]}, tokens [{d[5]}, {d[6]})"
    return ""


def check_device_status(what: str, device=None) -> None:
    """Raise :class:`StratumError` if a GEMM kernel on ``device`` gave up a bounded wait
    (or rejected its tile table) since the last read.  The read clears the word, so
    after the error the caller may retry; the results of the failed step are invalid."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    rec = device_status_record(dev)
    st = device_status(dev)
    if st != 0:
        where = describe_status_record(rec) if rec[0] == st else ""
        raise StratumError(f"{what}: a device-side wait timed out or a tile table was rejected (status 0x{st:x})"
                           f"{'; ' + where if where else ''}; the kernel unwound and its outputs are invalid "
                           f"(the status word is now cleared)")


def launch_count() -> int:
    return int(lib().stratum_launch_count())
