"""GPU parity of the fused NF4 GEMM (forward, LoRA epilogue, bias, double quant)
against an fp32 reference built from the oracle-exact dequantized weight.

Tolerance: ||y - y_ref|| / ||y_ref|| <= 1e-2 (bf16 inputs, fp32 accumulate),
the bar the reference path is held to; the measured error is ~2e-3 (one bf16
rounding of the output)."""

import pytest
import torch

from oracle.nf4_oracle import relative_error
from stratum_b200 import _lib, ops
from stratum_b200 import functional as F

pytestmark = pytest.mark.gpu

DEV = "cuda"
TOL = 1e-2


@pytest.fixture(autouse=True, params=["single", "pair"])
def gemm_kernel(request):
    """Every test runs on both kernels: one-SM tiles and CTA pairs."""
    ops.set_gemm_kernel(request.param)
    yield request.param
    ops.set_gemm_kernel("auto")


def _make(N, K, T, dtype=torch.bfloat16, seed=0, dq=False, rank=0, bias=False):
    g = torch.Generator(device=DEV).manual_seed(seed)
    w = (torch.randn(N, K, generator=g, device=DEV) * 0.02).to(torch.float16)
    packed, qs = F.quantize_4bit(w, compress_statistics=dq)
    w_deq = F.dequantize_4bit(packed, qs, out_dtype=torch.float32)  # bit-exact to the oracle (codec tests)
    x = torch.randn(T, K, generator=g, device=DEV).to(dtype)
    b = (torch.randn(N, generator=g, device=DEV) * 0.1).to(dtype) if bias else None
    A = B = None
    if rank:
        A = ((torch.rand(rank, K, generator=g, device=DEV) * 2 - 1) / K**0.5).to(dtype)
        B = (torch.randn(N, rank, generator=g, device=DEV) * 0.01).to(dtype)
    return w, packed, qs, w_deq, x, b, A, B


def _ref(x, w_deq, b, A, B, scaling, dtype):
    # the weight as the kernel sees it: rounded once to the activation dtype
    wq = w_deq.to(dtype).float()
    y = x.float() @ wq.t()
    if b is not None:
        y = y + b.float()
    if A is not None:
        y = y + scaling * ((x.float() @ A.float().t()) @ B.float().t())
    return y


@pytest.mark.parametrize(
    "T,N,K",
    [(256, 128, 64), (1, 128, 128), (300, 200, 192), (513, 384, 256), (1024, 5632, 2048), (2048, 4096, 4096)],
)
def test_fwd_plain(T, N, K):
    _, packed, qs, w_deq, x, _, _, _ = _make(N, K, T)
    y = ops.nf4_gemm_fwd(x, packed, qs)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    err = relative_error(y.float(), _ref(x, w_deq, None, None, None, 1.0, torch.bfloat16))
    assert err < TOL, f"rel err {err}"
    assert err < 4e-3, f"rel err {err} (expected ~2e-3)"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rank,dq,bias", [(16, False, True), (64, True, False), (32, False, False), (96, True, True)])
def test_fwd_lora_bias_dq(dtype, rank, dq, bias):
    T, N, K = 640, 384, 512
    scaling = 2.0
    _, packed, qs, w_deq, x, b, A, B = _make(N, K, T, dtype=dtype, dq=dq, rank=rank, bias=bias, seed=rank)
    y = ops.nf4_gemm_fwd(x, packed, qs, bias=b, lora_A=A, lora_B=B, scaling=scaling)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    ref = _ref(x, w_deq, b, A, B, scaling, dtype)
    err = relative_error(y.float(), ref)
    assert err < TOL, f"rel err {err}"
    # LoRA is really applied: its contribution is far above the tolerance
    if A is not None:
        base = _ref(x, w_deq, b, None, None, scaling, dtype)
        assert relative_error(base, ref) > 5 * err


def test_fwd_exact_against_cublas_on_dequantized_weight():
    # same bf16 weight values in both: the fused kernel == dequant + bf16 GEMM up to accumulation order
    T, N, K = 512, 1024, 1024
    _, packed, qs, _, x, _, _, _ = _make(N, K, T, seed=3)
    w16 = F.dequantize_4bit(packed, qs, out_dtype=torch.bfloat16)
    y = ops.nf4_gemm_fwd(x, packed, qs)
    y_ref = (x.float() @ w16.float().t())
    assert relative_error(y.float(), y_ref) < 4e-3


def test_fwd_config5_shape_smoke():
    # the 14336x4096 (down-proj shaped) weight at T = 4096 tokens
    T, N, K = 4096, 4096, 14336
    _, packed, qs, w_deq, x, _, _, _ = _make(N, K, T, seed=5)
    y = ops.nf4_gemm_fwd(x, packed, qs)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    rows = torch.randint(0, T, (64,), device=DEV)
    ref = x[rows].float() @ w_deq.to(torch.bfloat16).float().t()
    assert relative_error(y[rows].float(), ref) < 4e-3


def test_fwd_many_tiles_per_cta_every_tile():
    T, N, K = 8192, 4096, 2048
    _, packed, qs, w_deq, x, _, _, _ = _make(N, K, T, seed=13)
    ref = x.float() @ w_deq.to(torch.bfloat16).float().t()
    for _ in range(2):
        y = ops.nf4_gemm_fwd(x, packed, qs).float()
        err = (y - ref).reshape(T // 256, 256, N // 128, 128)
        den = ref.reshape(T // 256, 256, N // 128, 128).pow(2).sum(dim=(1, 3)).sqrt()
        assert (err.pow(2).sum(dim=(1, 3)).sqrt() / den).max().item() < 4e-3


@pytest.mark.parametrize(
    "T,N,K",
    [
        (129, 1288, 128),  # N % 256 == 8: the second CTA of the last pair tile has no rows
        (300, 200, 192),   # one pair tile: second MMA partial, second CTA's rows partly past N
        (777, 1030, 64),   # N % 8 != 0: element-store epilogue
        (1, 1288, 64),     # one token
        (1100, 520, 320),  # last token tile of 76 tokens
    ],
)
def test_fwd_ragged_tiles(T, N, K):
    _, packed, qs, w_deq, x, b, _, _ = _make(N, K, T, seed=T, bias=True)
    y = ops.nf4_gemm_fwd(x, packed, qs, bias=b)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    err = relative_error(y.float(), _ref(x, w_deq, b, None, None, 1.0, torch.bfloat16))
    assert err < 4e-3, f"rel err {err}"
