"""Bounded device-side waits: a wait that is never satisfied gives up after the
configured limit, reports where it was through the status record, and leaves the
CUDA context usable.  The wait is on a barrier nothing arrives on (a flag no one
sets); no fault, trap or hang is involved."""

import pytest
import torch

from stratum_b200 import _lib, ops, workloads
from stratum_b200.functional import dequantize_4bit, quantize_4bit

pytestmark = pytest.mark.gpu

SELFTEST = 0x1F0


def _u64(lo, hi):
    return (lo & 0xFFFFFFFF) | ((hi & 0xFFFFFFFF) << 32)


def test_wait_gives_up_after_the_limit_and_reports_it():
    torch.cuda.set_device(0)
    _lib.device_status()  # start from a clear word
    limit = 20_000_000  # 20 ms
    _lib.set_wait_limit_ns(limit)
    try:
        _lib.wait_selftest()
        torch.cuda.synchronize()
        rec = _lib.device_status_record()
        assert rec[0] == SELFTEST
        assert rec[1] == 0 and rec[2] == 0 and rec[3] == 0  # block 0, thread 0, parity 0
        waited_ns = _u64(rec[8], rec[9])
        assert limit <= waited_ns < 1_000_000_000
        assert rec[10] != 0  # SM cycles elapsed in the wait
        # the barrier waited on is initialised for one arrival and never completed
        assert _u64(rec[5], rec[6]) == _u64(rec[12 + 2 * _lib.BAR_BELOW], rec[13 + 2 * _lib.BAR_BELOW])
        assert "first wait to give up" in _lib.describe_status_record(rec)
        assert _lib.device_status() == SELFTEST  # the read clears it
        assert _lib.device_status() == 0
        with pytest.raises(_lib.StratumError, match="0x1f0"):
            _lib.wait_selftest()
            _lib.check_device_status("selftest")
    finally:
        _lib.set_wait_limit_ns(0)
    assert _lib.device_status() == 0


def test_context_usable_after_a_wait_gave_up():
    torch.cuda.set_device(0)
    _lib.set_wait_limit_ns(5_000_000)
    try:
        _lib.wait_selftest()
        torch.cuda.synchronize()
    finally:
        _lib.set_wait_limit_ns(0)
    assert _lib.device_status() == SELFTEST
    # a GEMM after the cleared error runs to completion with the default limit
    w = workloads.codec_weight((512, 1024), seed=3)
    packed, qs = quantize_4bit(w, blocksize=64)
    x = torch.randn(256, 1024, device="cuda", dtype=torch.bfloat16)
    y = ops.nf4_gemm_fwd(x, packed, qs)
    ref = x.float() @ dequantize_4bit(packed, qs, out_dtype=torch.float32).to(torch.bfloat16).float().t()
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    rel = (y.float() - ref).norm() / ref.norm()
    assert rel < 1e-2


def test_wait_limit_bounds_are_checked():
    torch.cuda.set_device(0)
    with pytest.raises(ValueError):
        _lib.set_wait_limit_ns(1000)  # below 1 ms
    with pytest.raises(ValueError):
        _lib.set_wait_limit_ns(120_000_000_000)  # above 60 s
