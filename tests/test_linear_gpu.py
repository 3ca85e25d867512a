"""GPU parity of the fused NF4 input-gradient kernel and the NF4Linear module
(forward + backward with LoRA) against the fp32 oracle reference
(oracle/nf4_oracle.py: nf4_linear_reference) on the oracle-exact weight.

Tolerance: relative Frobenius error <= 1e-2 for y, dX, dA, dB (bf16 inputs,
fp32 accumulation)."""

import pytest
import torch

from oracle.nf4_oracle import nf4_linear_reference, relative_error
from stratum_b200 import _lib, ops, workloads
from stratum_b200 import functional as F
from stratum_b200.nf4_linear import NF4Linear

pytestmark = pytest.mark.gpu

DEV = "cuda"
TOL = 1e-2


@pytest.fixture(autouse=True, params=["single", "pair"])
def gemm_kernel(request):
    """Every test runs on both kernels: one-SM tiles and CTA pairs."""
    ops.set_gemm_kernel(request.param)
    yield request.param
    ops.set_gemm_kernel("auto")


def _weight(N, K, seed=0, dq=False):
    g = torch.Generator(device=DEV).manual_seed(seed)
    w = (torch.randn(N, K, generator=g, device=DEV) * 0.02).to(torch.float16)
    packed, qs = F.quantize_4bit(w, compress_statistics=dq)
    return packed, qs, F.dequantize_4bit(packed, qs, out_dtype=torch.float32)


@pytest.mark.parametrize("T,N,K", [(256, 128, 128), (300, 200, 192), (1, 64, 64), (1024, 5632, 2048),
                                   (2048, 4096, 4096), (777, 1032, 320)])
def test_dx_plain(T, N, K):
    packed, qs, w = _weight(N, K, seed=T)
    g = torch.Generator(device=DEV).manual_seed(1)
    dy = torch.randn(T, N, generator=g, device=DEV).to(torch.bfloat16)
    dx = ops.nf4_gemm_dx(dy, packed, qs)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    ref = dy.float() @ w.to(torch.bfloat16).float()
    err = relative_error(dx.float(), ref)
    assert err < 4e-3, f"rel err {err}"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rank,dq", [(16, False), (64, True), (96, False)])
def test_dx_lora(dtype, rank, dq):
    T, N, K = 520, 384, 512
    scaling = 2.0
    packed, qs, w = _weight(N, K, seed=rank, dq=dq)
    g = torch.Generator(device=DEV).manual_seed(2)
    dy = torch.randn(T, N, generator=g, device=DEV).to(dtype)
    A = ((torch.rand(rank, K, generator=g, device=DEV) * 2 - 1) / K**0.5).to(dtype)
    B = (torch.randn(N, rank, generator=g, device=DEV) * 0.05).to(dtype)
    dx = ops.nf4_gemm_dx(dy, packed, qs, lora_A=A, lora_B=B, scaling=scaling)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    ref = dy.float() @ w.to(dtype).float() + scaling * ((dy.float() @ B.float()) @ A.float())
    assert relative_error(dx.float(), ref) < TOL


def _check_module(x, w_deq, mod, dy, scaling):
    xx = x.clone().requires_grad_(True)
    y = mod(xx)
    y.backward(dy)
    ref = nf4_linear_reference(x.cpu(), w_deq.cpu(), None if mod.bias is None else mod.bias.cpu(),
                               None if mod.lora_A is None else mod.lora_A.detach().cpu(),
                               None if mod.lora_B is None else mod.lora_B.detach().cpu(), scaling, dy.cpu())
    assert relative_error(y.float().cpu(), ref["y"]) < TOL
    assert relative_error(xx.grad.float().cpu(), ref["dx"]) < TOL
    if mod.lora_A is not None:
        assert relative_error(mod.lora_A.grad.float().cpu(), ref["dA"]) < TOL
        assert relative_error(mod.lora_B.grad.float().cpu(), ref["dB"]) < TOL


def test_nf4linear_config1_forward_backward():
    """W 5632x2048 fp16 ~N(0,0.02) -> NF4 bs64, LoRA r=16 alpha=32,
    x bf16 [2,512,2048] ~N(0,1), dY ~N(0,1): y, dX, dA, dB within 1e-2 of fp32."""
    w, A, B, x, dy = workloads.linear_inputs(device=DEV)
    packed, qs = F.quantize_4bit(w)
    w_deq = F.dequantize_4bit(packed, qs, out_dtype=torch.float32)
    mod = NF4Linear(packed, qs)
    mod.attach_lora(workloads.LINEAR1_RANK, workloads.LINEAR1_ALPHA)
    with torch.no_grad():
        mod.lora_A.copy_(A)
        mod.lora_B.copy_(B)
    assert mod.in_features == 2048 and mod.out_features == 5632
    # the weight as the bf16 kernel sees it: rounded once to bf16
    _check_module(x, w_deq.to(torch.bfloat16).float(), mod, dy, mod.scaling)


def test_nf4linear_plain_bias_fp16():
    g = torch.Generator(device=DEV).manual_seed(9)
    packed, qs, w = _weight(384, 256, seed=9)
    bias = (torch.randn(384, generator=g, device=DEV) * 0.1).to(torch.float16)
    mod = NF4Linear(packed, qs, bias=bias)
    x = torch.randn(3, 100, 256, generator=g, device=DEV).to(torch.float16)
    dy = torch.randn(3, 100, 384, generator=g, device=DEV).to(torch.float16)
    _check_module(x, w.to(torch.float16).float(), mod, dy, 1.0)
    assert not mod.bias.requires_grad and mod.bias.grad is None


def test_nf4linear_matches_reference_semantics():
    # reference NF4Linear.forward == F.linear(x, dequantize_4bit(q, state), bias)
    packed, qs, w = _weight(256, 512, seed=4)
    mod = NF4Linear(packed, qs)
    x = torch.randn(64, 512, device=DEV).to(torch.bfloat16)
    y = mod(x)
    y_ref = torch.nn.functional.linear(x, mod.weight_dequantized.to(torch.bfloat16))
    assert relative_error(y.float(), y_ref.float()) < 4e-3


@pytest.mark.parametrize("T,N,K", [(4096, 1024, 8192), (2048, 4096, 4096)])
def test_dx_many_tiles_per_cta_every_tile(T, N, K):
    """Every 256x128 output tile checked, over repeated launches: several tiles per CTA
    exercise the rings' reuse and the double-buffered accumulator."""
    packed, qs, w = _weight(N, K, seed=11)
    g = torch.Generator(device=DEV).manual_seed(12)
    dy = torch.randn(T, N, generator=g, device=DEV).to(torch.bfloat16)
    ref = dy.float() @ w.to(torch.bfloat16).float()
    for _ in range(3):
        dx = ops.nf4_gemm_dx(dy, packed, qs).float()
        err = (dx - ref).reshape(T // 256, 256, K // 128, 128)
        den = ref.reshape(T // 256, 256, K // 128, 128).pow(2).sum(dim=(1, 3)).sqrt()
        per_tile = err.pow(2).sum(dim=(1, 3)).sqrt() / den
        assert per_tile.max().item() < 4e-3, f"worst tile {per_tile.max().item()}"
