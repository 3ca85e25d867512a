"""The allocation-free double-quant quantizer (stratum_nf4_quantize_dq_noalloc).

It exists for callers of the C ABI that cannot hand the library a device
workspace: an FFI host that only owns the buffers it passes in, or code that
must not allocate at that point.  Its scratch is a fixed array inside the
library, shared by every call.  This test calls it through the C ABI three
times in a row (a large input, then a smaller one, so the second call runs over
scratch the first left behind, then one whose last NF4 block is partial) and
checks each result bit for bit against the regular entry points given a
caller-allocated workspace -- the codec's tolerance is exact.  It also checks
the size limit and that an empty input is a no-op.

Named so pytest collects it last; it passes alone and after the other tests.
"""

import ctypes

import pytest
import torch

from stratum_b200 import _lib, codebook, workloads

pytestmark = pytest.mark.gpu

DEV = "cuda"
MAX_ELEMS = (1 << 20) * 64  # the entry point's fixed scratch: 2^20 blocks of 64


def _regular(w):
    """Outputs of stratum_nf4_quantize + stratum_nf4_quantize_absmax_dq with allocated scratch."""
    L = _lib.lib()
    n = w.numel()
    nb = (n + 63) // 64
    st = _lib.stream_of(w.device)
    packed = torch.empty((n + 1) // 2, dtype=torch.uint8, device=DEV)
    absmax = torch.empty(nb, dtype=torch.float32, device=DEV)
    _lib.check(L.stratum_nf4_quantize(_lib.ptr(w), _lib.DTYPE_CODE[w.dtype], n, 64,
                                      _lib.ptr(codebook.nf4_thresholds(DEV)), _lib.ptr(packed), _lib.ptr(absmax), st),
               "quantize")
    q = torch.empty(nb, dtype=torch.uint8, device=DEV)
    a2 = torch.empty((nb + 255) // 256, dtype=torch.float32, device=DEV)
    off = torch.empty((), dtype=torch.float32, device=DEV)
    ws_bytes = int(L.stratum_nf4_dq_workspace_bytes(nb))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=DEV)
    _lib.check(L.stratum_nf4_quantize_absmax_dq(_lib.ptr(absmax), nb, 256, _lib.ptr(codebook.dynamic_thresholds(DEV)),
                                                _lib.ptr(q), _lib.ptr(a2), _lib.ptr(off), _lib.ptr(ws), ws_bytes, st),
               "quantize_absmax_dq")
    return packed, q, a2, off


def _no_alloc(w):
    L = _lib.lib()
    n = w.numel()
    nb = (n + 63) // 64
    packed = torch.full(((n + 1) // 2,), 0xEE, dtype=torch.uint8, device=DEV)
    q = torch.full((nb,), 0xEE, dtype=torch.uint8, device=DEV)
    a2 = torch.full(((nb + 255) // 256,), -1.0, dtype=torch.float32, device=DEV)
    off = torch.full((), -1.0, dtype=torch.float32, device=DEV)
    _lib.check(L.stratum_nf4_quantize_dq_noalloc(_lib.ptr(w), _lib.DTYPE_CODE[w.dtype], n,
                                                 _lib.ptr(codebook.nf4_thresholds(DEV)),
                                                 _lib.ptr(codebook.dynamic_thresholds(DEV)), _lib.ptr(packed),
                                                 _lib.ptr(q), _lib.ptr(a2), _lib.ptr(off), _lib.stream_of(w.device)),
               "quantize_dq_noalloc")
    return packed, q, a2, off


def test_no_alloc_matches_regular_entry_points_on_two_calls_in_a_row():
    big = workloads.codec_weight((14336, 4096), seed=21)  # 58.7 M elements, close to the limit
    small = workloads.codec_weight((1000, 4096 + 192), seed=22).to(torch.bfloat16)  # ragged block count
    # a partial final NF4 block (n % 64 == 37) and an odd element count (half-filled last byte)
    tail = workloads.codec_weight((64 * 1000 + 37,), seed=23)
    for w in (big, small, tail):
        got = _no_alloc(w)
        ref = _regular(w)
        torch.cuda.synchronize()
        for g, r, what in zip(got, ref, ("packed", "absmax_q", "absmax2", "offset")):
            assert torch.equal(g, r), f"{what} differs for n={w.numel()}"


def test_no_alloc_rejects_sizes_above_its_scratch():
    L = _lib.lib()
    dummy = torch.empty(16, dtype=torch.uint8, device=DEV)
    rc = L.stratum_nf4_quantize_dq_noalloc(_lib.ptr(dummy), 1, MAX_ELEMS + 1, _lib.ptr(dummy), _lib.ptr(dummy),
                                           _lib.ptr(dummy), _lib.ptr(dummy), _lib.ptr(dummy), _lib.ptr(dummy),
                                           _lib.stream_of(dummy.device))
    assert rc == _lib.STRATUM_ERR_INVALID
    assert b"fixed scratch" in L.stratum_last_error()


def test_no_alloc_empty_input_is_a_no_op():
    L = _lib.lib()
    dummy = torch.full((16,), 0xEE, dtype=torch.uint8, device=DEV)
    rc = L.stratum_nf4_quantize_dq_noalloc(_lib.ptr(dummy), 1, 0, _lib.ptr(dummy), _lib.ptr(dummy), _lib.ptr(dummy),
                                           _lib.ptr(dummy), _lib.ptr(dummy), _lib.ptr(dummy),
                                           _lib.stream_of(dummy.device))
    assert rc == _lib.STRATUM_OK
    torch.cuda.synchronize()
    assert bool((dummy == 0xEE).all())
