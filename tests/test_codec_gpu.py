"""GPU parity of the NF4 codec kernels (K1 quantize, K2 dequantize, double quant)
against the CPU oracle: bit-exact for packed nibbles, absmax and dequantized
values.  Small cases compare with the numpy restatement, full config-2 sizes
with the C restatement plus size-independent properties."""

import numpy as np
import pytest
import torch

from oracle import nf4_oracle as O
from stratum_b200 import functional as F
from stratum_b200 import workloads

pytestmark = pytest.mark.gpu

DEV = "cuda"
DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}


def _np_bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().contiguous().cpu()
    if t.dtype in (torch.float16, torch.bfloat16):
        return t.view(torch.int16).numpy().view(np.uint16).reshape(-1)
    return t.view(torch.int32).numpy().view(np.uint32).reshape(-1)


def _oracle_bits(arr: np.ndarray, od: str) -> np.ndarray:
    if od == "bfloat16":
        return arr.view(np.uint16)
    if od == "float16":
        return arr.view(np.uint16)
    return arr.view(np.uint32)


def _thr(conv):
    return O.NF4_THRESHOLDS_CUDA if conv == "cuda" else O.NF4_THRESHOLDS_MIDPOINT


def _check_roundtrip(w: torch.Tensor, blocksize: int, conv: str = "cuda"):
    packed, st = F.quantize_4bit(w, blocksize=blocksize, thresholds=conv)
    p_o, a_o = O.quantize_nf4(w, blocksize, _thr(conv))
    assert packed.shape == ((w.numel() + 1) // 2, 1) and packed.dtype == torch.uint8
    assert np.array_equal(packed.cpu().numpy().reshape(-1), p_o), "packed nibbles differ from oracle"
    assert np.array_equal(st.absmax.cpu().numpy(), a_o), "absmax differs from oracle"
    assert st.shape == tuple(w.shape) and st.dtype == w.dtype and st.blocksize == blocksize
    for od in ("float16", "bfloat16", "float32"):
        d = F.dequantize_4bit(packed, st, out_dtype=DTYPES[od])
        assert d.shape == w.shape and d.dtype == DTYPES[od]
        ref = O.dequantize_nf4(p_o, a_o, w.numel(), blocksize, out_dtype=od)
        assert np.array_equal(_np_bits(d), _oracle_bits(ref, od)), f"dequant {od} differs from oracle"


@pytest.mark.parametrize("dtype", ["float16", "bfloat16", "float32"])
@pytest.mark.parametrize("blocksize", [32, 64, 128, 256])
def test_codec_matches_oracle_small(dtype, blocksize):
    g = torch.Generator(device=DEV).manual_seed(blocksize)
    w = (torch.randn(96, 8 * blocksize, generator=g, device=DEV) * 0.02).to(DTYPES[dtype])
    w[3] = 0  # whole zero rows -> zero blocks
    w[5, 7] = 1.0  # outlier
    _check_roundtrip(w, blocksize)


@pytest.mark.parametrize("conv", ["cuda", "midpoint"])
def test_threshold_conventions(conv):
    # values exactly on the thresholds (absmax 1 -> scale 1), where the conventions differ
    thr = np.concatenate([O.NF4_THRESHOLDS_CUDA, O.NF4_THRESHOLDS_MIDPOINT])
    vals = np.concatenate([thr, np.nextafter(thr, 2), np.nextafter(thr, -2)]).astype(np.float32)
    x = np.ones(64 * 2, np.float32)
    x[: vals.size] = vals
    _check_roundtrip(torch.from_numpy(x).to(DEV), 64, conv)


@pytest.mark.parametrize("n", [1, 2, 3, 7, 8, 9, 63, 64, 65, 127, 128, 129, 1000, 4096 + 24, 65536 + 2])
def test_ragged_sizes(n):
    g = torch.Generator(device=DEV).manual_seed(n)
    w = (torch.randn(n, generator=g, device=DEV) * 0.02).to(torch.float16)
    _check_roundtrip(w, 64)


def test_edge_values():
    # NaN/inf inputs are out of contract (the absmax reduction ignores NaN like fmaxf); all values finite here
    x = torch.zeros(64 * 8, dtype=torch.float32)
    x[64:128] = 1e-30  # tiny (subnormal-range products)
    x[128:192] = torch.linspace(-3e38, 3e38, 64, dtype=torch.float64).to(torch.float32)  # huge, finite
    x[192:256] = 7.5  # constant block
    x[256:320] = -0.0
    x[320] = 1e-45  # one denormal, rest zero
    x[384:448] = torch.tensor(O.NF4_LEVELS).repeat(4) * 3.0
    assert torch.isfinite(x).all()
    _check_roundtrip(x.to(DEV), 64)


def test_empty_tensor():
    w = torch.empty(0, 4, dtype=torch.float16, device=DEV)
    packed, st = F.quantize_4bit(w)
    assert packed.numel() == 0 and st.absmax.numel() == 0
    d = F.dequantize_4bit(packed, st)
    assert d.shape == (0, 4)


def test_unaligned_output_and_cpu_input():
    g = torch.Generator().manual_seed(3)
    w = (torch.randn(64, 192, generator=g) * 0.02).to(torch.float16)  # CPU input -> CPU outputs
    packed, st = F.quantize_4bit(w)
    assert packed.device.type == "cpu" and st.absmax.device.type == "cpu"
    p_o, a_o = O.quantize_nf4(w, 64)
    assert np.array_equal(packed.numpy().reshape(-1), p_o) and np.array_equal(st.absmax.numpy(), a_o)
    # dequant into a 2-byte-offset view: takes the unaligned kernel
    buf = torch.full((w.numel() + 1,), 7.0, dtype=torch.float16, device=DEV)
    out = buf[1:]
    F.dequantize_4bit(packed.to(DEV), st.to(DEV), out=out.view(w.shape))
    ref = O.dequantize_nf4(p_o, a_o, w.numel(), 64)
    assert np.array_equal(_np_bits(out), ref.view(np.uint16))
    assert buf[0].item() == 7.0


def test_canary_guard_bands():
    n = 4096 * 3 + 40
    w = (torch.randn(n, device=DEV) * 0.02).to(torch.bfloat16)
    guard = 4096
    pk = torch.full((guard + (n + 1) // 2 + guard,), 0xA5, dtype=torch.uint8, device=DEV)
    am = torch.full((guard + (n + 63) // 64 + guard,), -123.0, dtype=torch.float32, device=DEV)
    from stratum_b200 import _lib, codebook

    L = _lib.lib()
    _lib.check(L.stratum_nf4_quantize(_lib.ptr(w), 2, n, 64, _lib.ptr(codebook.nf4_thresholds(DEV)),
                                      _lib.ptr(pk[guard:]), _lib.ptr(am[guard:]), _lib.stream_of(w.device)), "q")
    out = torch.full((guard + n + guard,), 5.0, dtype=torch.float16, device=DEV)
    _lib.check(L.stratum_nf4_dequantize(_lib.ptr(pk[guard:]), _lib.ptr(am[guard:]), _lib.ptr(codebook.nf4_code(DEV)),
                                        n, 64, _lib.ptr(out[guard:]), 1, _lib.stream_of(w.device)), "dq")
    torch.cuda.synchronize()
    assert torch.all(pk[:guard] == 0xA5) and torch.all(pk[guard + (n + 1) // 2:] == 0xA5)
    assert torch.all(am[:guard] == -123.0) and torch.all(am[guard + (n + 63) // 64:] == -123.0)
    assert torch.all(out[:guard] == 5.0) and torch.all(out[guard + n:] == 5.0)


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
def test_double_quant_matches_oracle(dtype):
    w = workloads.codec_weight((1024, 4096 + 64 * 3), seed=11, dtype=DTYPES[dtype])
    packed, st = F.quantize_4bit(w, compress_statistics=True)
    assert st.nested and st.absmax.dtype == torch.uint8 and st.state2.blocksize == 256
    p_o, aq, a2, c2, off = O.quantize_nf4_dq(w, 64)
    assert np.array_equal(packed.cpu().numpy().reshape(-1), p_o)
    assert np.array_equal(st.offset.cpu().numpy().reshape(-1), np.array([off], np.float32))
    assert np.array_equal(st.absmax.cpu().numpy(), aq)
    assert np.array_equal(st.state2.absmax.cpu().numpy(), a2)
    assert np.array_equal(st.state2.code.cpu().numpy(), c2)
    for od in ("float16", "bfloat16", "float32"):
        d = F.dequantize_4bit(packed, st, out_dtype=DTYPES[od])
        ref = O.dequantize_nf4_dq(p_o, aq, a2, c2, off, w.numel(), out_dtype=od)
        assert np.array_equal(_np_bits(d), _oracle_bits(ref, od))


@pytest.mark.parametrize("shape", workloads.CODEC_SHAPES + (workloads.LINEAR1_WEIGHT,))
def test_config_sizes_bit_exact_and_idempotent(oracle_c, shape):
    w = workloads.codec_weight(shape, seed=0)
    packed, st = F.quantize_4bit(w)
    p_c, a_c = oracle_c.quantize(w.cpu(), 64)
    assert np.array_equal(packed.cpu().numpy().reshape(-1), p_c)
    assert np.array_equal(st.absmax.cpu().numpy(), a_c)
    d16 = F.dequantize_4bit(packed, st)
    ref16 = oracle_c.dequantize(p_c, a_c, w.numel(), 64, "float16")
    assert np.array_equal(_np_bits(d16), ref16.view(np.uint16))
    # size-independent property: re-quantizing the fp32 dequant reproduces the code exactly
    d32 = F.dequantize_4bit(packed, st, out_dtype=torch.float32)
    packed2, st2 = F.quantize_4bit(d32)
    assert torch.equal(packed2, packed) and torch.equal(st2.absmax, st.absmax)
    # double quant at full size against the C oracle
    packed_dq, st_dq = F.quantize_4bit(w, compress_statistics=True)
    q_c, a2_c, c2_c, off_c = oracle_c.quantize_absmax_dq(a_c)
    assert np.array_equal(st_dq.absmax.cpu().numpy(), q_c)
    assert np.array_equal(st_dq.state2.absmax.cpu().numpy(), a2_c)
    assert st_dq.offset.item() == float(off_c)
    dq16 = F.dequantize_4bit(packed_dq, st_dq, out_dtype=torch.bfloat16)
    ref_dq = oracle_c.dequantize_dq(p_c, q_c, a2_c, c2_c, off_c, w.numel(), 64, "bfloat16")
    assert np.array_equal(_np_bits(dq16), ref_dq)


def test_dequantize_many_matches_single_tensor_calls():
    """One batched launch per 32 tensors of a kind gives exactly the per-tensor results:
    plain and double-quant mixed, sizes that take the one-by-one fallback (n % 64 != 0),
    and more than 32 tensors (several launches)."""
    g = torch.Generator(device="cuda").manual_seed(77)
    shapes = [(4096, 4096), (1000, 1000), (64, 64), (7, 9)] + [(256, 320)] * 36 + [(14336, 512)]
    items, refs = [], []
    for i, shp in enumerate(shapes):
        w = (torch.randn(*shp, generator=g, device="cuda") * 0.02).half()
        packed, qs = F.quantize_4bit(w, compress_statistics=(i % 3 == 1))
        items.append((packed, qs))
        refs.append(F.dequantize_4bit(packed, qs, out_dtype=torch.bfloat16))
    outs = F.dequantize_4bit_many(items, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    for i, (o, r) in enumerate(zip(outs, refs)):
        assert torch.equal(o, r), f"tensor {i} {shapes[i]}"
