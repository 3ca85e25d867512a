"""CPU tests of the oracle itself: known answers from the NF4 definition, the two
threshold conventions, C vs numpy restatements, double quant, and the product's
codebook tables against the oracle's."""

import numpy as np
import pytest
import torch

from oracle import nf4_oracle as O


def test_levels_are_the_qlora_table():
    lv = O.NF4_LEVELS
    assert lv.dtype == np.float32 and lv.size == 16
    assert lv[0] == -1.0 and lv[7] == 0.0 and lv[15] == 1.0
    assert np.all(np.diff(lv) > 0)
    # every level is an exact float32 (no rounding when stored)
    assert np.array_equal(lv.astype(np.float64).astype(np.float32), lv)


def test_threshold_conventions_differ_only_at_float32_ties():
    cuda, mid = O.NF4_THRESHOLDS_CUDA, O.NF4_THRESHOLDS_MIDPOINT
    diff = np.nonzero(cuda != mid)[0].tolist()
    assert diff == [0, 8, 12, 14]
    assert set(diff) <= set(O.threshold_ties())
    # one float32 ulp apart where they differ
    for i in diff:
        assert np.nextafter(cuda[i], mid[i]) == mid[i]
    # both conventions are sorted and strictly between neighbouring levels
    for thr in (cuda, mid):
        assert np.all(np.diff(thr) > 0)
        assert np.all(thr > O.NF4_LEVELS[:-1]) and np.all(thr < O.NF4_LEVELS[1:])


def test_known_answers_levels_map_to_themselves():
    absmax = np.float32(0.5)
    x = (O.NF4_LEVELS * absmax).astype(np.float32)
    x = np.concatenate([x, x[::-1], x, x[::-1]])  # one block of 64
    packed, am = O.quantize_nf4(x, 64)
    assert am[0] == absmax
    q = O.unpack_nibbles(packed, 64)
    assert q.tolist() == list(range(16)) + list(range(15, -1, -1)) + list(range(16)) + list(range(15, -1, -1))
    deq = O.dequantize_nf4(packed, am, 64, 64, out_dtype="float32")
    assert np.array_equal(deq, x)


def test_known_answers_threshold_neighbourhood():
    thr = O.NF4_THRESHOLDS
    vals, want = [], []
    for i, t in enumerate(thr):
        vals += [t, np.nextafter(t, np.float32(2))]
        want += [i, i + 1]  # strict ">": exactly at the threshold stays below
    x = np.array(vals + [1.0] * (64 - len(vals)), np.float32)  # absmax 1.0 -> scale 1
    packed, am = O.quantize_nf4(x, 64)
    q = O.unpack_nibbles(packed, 64)
    assert q[: len(want)].tolist() == want
    assert np.all(q[len(want):] == 15)


def test_zero_block_and_odd_tail():
    x = np.zeros(64 + 3, np.float32)
    x[64:] = [0.25, -0.5, 0.125]
    packed, am = O.quantize_nf4(x, 64)
    assert am.tolist() == [0.0, 0.5]
    q = O.unpack_nibbles(packed, 68)
    assert np.all(q[:64] == 0)  # 0 * inf = NaN -> level 0
    assert q[64:67].tolist() == [12, 0, 10]  # 0.5, -1.0, 0.25 (rounded to nearest level)
    assert q[67] == 7  # padding element quantized as 0.0
    assert packed.size == 34
    deq = O.dequantize_nf4(packed, am, 67, 64, out_dtype="float32")
    assert np.all(deq[:64] == 0.0) and np.all(np.signbit(deq[:64]))  # -1 * 0 = -0.0


def test_bf16_rounding_helper():
    v = np.array([1.0, 1.00390625, 1.005859375, -3.1415926, 65504.0], np.float32)
    bits = O.f32_to_bf16_bits(v)
    ref = torch.from_numpy(v).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(bits, ref)


@pytest.mark.parametrize("dtype", ["float16", "bfloat16", "float32"])
@pytest.mark.parametrize("blocksize", [32, 64, 128, 256])
@pytest.mark.parametrize("conv", ["cuda", "midpoint"])
def test_c_oracle_matches_numpy(oracle_c, dtype, blocksize, conv):
    g = torch.Generator().manual_seed(1234 + blocksize)
    n = 7 * blocksize * 5 + 13
    x = torch.randn(n, generator=g, dtype=torch.float32) * 0.02
    x[:blocksize] = 0
    x = x.to(getattr(torch, dtype))
    thr = O.NF4_THRESHOLDS_CUDA if conv == "cuda" else O.NF4_THRESHOLDS_MIDPOINT
    p_np, a_np = O.quantize_nf4(x, blocksize, thr)
    p_c, a_c = oracle_c.quantize(x, blocksize, thr)
    assert np.array_equal(p_np, p_c) and np.array_equal(a_np, a_c)
    for od in ("float16", "bfloat16", "float32"):
        d_np = O.dequantize_nf4(p_np, a_np, n, blocksize, out_dtype=od)
        d_c = oracle_c.dequantize(p_c, a_c, n, blocksize, out_dtype=od)
        assert np.array_equal(d_np.view(np.uint8), d_c.view(np.uint8))


def test_dynamic_code_shape_and_order():
    c = O.dynamic_code_signed()
    assert c.size == 256 and c.dtype == np.float32
    assert np.all(np.diff(c) > 0)
    assert c[-1] == 1.0 and 0.0 in c
    assert -1.0 < c[0] < -0.99


def test_double_quant_c_matches_numpy_and_reconstructs(oracle_c):
    g = torch.Generator().manual_seed(7)
    w = (torch.randn(4096 * 33, generator=g) * 0.02).to(torch.float16)
    _, am = O.quantize_nf4(w, 64)
    q, a2, c2, off = O.quantize_absmax_dq(am)
    qc, a2c, c2c, offc = oracle_c.quantize_absmax_dq(am)
    assert np.array_equal(q, qc) and np.array_equal(a2, a2c) and off == offc
    assert off == np.float32(O.dq_mean(am))
    rec = O.dequantize_absmax_dq(q, a2, c2, off)
    assert np.max(np.abs(rec - am)) <= 0.02 * np.max(np.abs(am - off))
    packed, _ = O.quantize_nf4(w, 64)
    d_np = O.dequantize_nf4_dq(packed, q, a2, c2, off, w.numel())
    d_c = oracle_c.dequantize_dq(packed, q, a2, c2, off, w.numel())
    assert np.array_equal(d_np.view(np.uint16), d_c.view(np.uint16))


def test_product_codebook_matches_oracle():
    from stratum_b200 import codebook

    assert np.array_equal(codebook.nf4_levels_np(), O.NF4_LEVELS)
    assert np.array_equal(codebook.thresholds_np(convention="cuda"), O.NF4_THRESHOLDS_CUDA)
    assert np.array_equal(codebook.thresholds_np(convention="midpoint"), O.NF4_THRESHOLDS_MIDPOINT)
    assert np.array_equal(codebook.dynamic_code_np(), O.dynamic_code_signed())
    assert np.array_equal(codebook.dynamic_thresholds_np(), O.midpoints_f32(O.dynamic_code_signed()))
