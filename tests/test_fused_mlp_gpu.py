"""GPU parity of the fused NF4 SwiGLU MLP (FusedMLP's three-kernel path).

* The gate|up GEMM with the SwiGLU epilogue reproduces, bit for bit, the
  unfused path it replaces (the gate and up NF4 GEMMs, then the SwiGLU kernel):
  each output row is the same dot product over the same dequantized weights.
* The SwiGLU backward written as [dgate | dup] rows (the dY of the stacked
  gate/up input gradient) equals the two-output SwiGLU backward kernel bit for
  bit.
* The whole MLP (forward, input gradient, LoRA gradients) is within 1e-2
  relative (Frobenius) of an fp32 reference on the exact dequantized weights,
  and within 1e-2 of HF's LlamaMLP run on the same weights with the adapters
  added as PEFT does.
"""

import pytest
import torch
import torch.nn.functional as TF

from oracle.nf4_oracle import relative_error
from stratum_b200 import fused as FZ
from stratum_b200 import functional as F
from stratum_b200 import ops
from stratum_b200.nf4_linear import NF4Linear

pytestmark = pytest.mark.gpu

DEV = "cuda"
CASES = [  # (tokens, hidden, intermediate, lora rank, double quant)
    (1000, 512, 1024, 16, False),
    (256, 1024, 3072, 0, True),
    (777, 512, 1536, 64, True),
]


def _linear(out_f, in_f, g, dq, r, lora_seed):
    w = (torch.randn(out_f, in_f, generator=g, device=DEV) * 0.02).half()
    packed, qs = F.quantize_4bit(w, compress_statistics=dq)
    m = NF4Linear(packed, qs)
    if r:
        m.attach_lora(r, alpha=2.0 * r, init_B_zero=False, device=DEV)
        with torch.no_grad():  # a visible adapter term
            gl = torch.Generator(device=DEV).manual_seed(lora_seed)
            m.lora_B.copy_(torch.randn(m.lora_B.shape, generator=gl, device=DEV) * 0.05)
    return m


def _mlp(H, I, r, dq, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    gate = _linear(I, H, g, dq, r, seed + 1)
    up = _linear(I, H, g, dq, r, seed + 2)
    down = _linear(H, I, g, dq, r, seed + 3)
    return gate, up, down


def _w(m):
    return F.dequantize_4bit(m.quantized, m.quant_state, out_dtype=torch.float32)


def _ref_fp32(x, gate, up, down):
    """fp32 reference of the MLP with PEFT LoRA: y, and autograd dx / LoRA grads."""
    x = x.float().detach().requires_grad_()
    params = []

    def lin(m, z):
        y = z @ _w(m).t()
        if m.lora_A is not None:
            A = m.lora_A.float().detach().requires_grad_()
            B = m.lora_B.float().detach().requires_grad_()
            params.extend([A, B])
            y = y + m.scaling * (z @ A.t()) @ B.t()
        return y

    y = lin(down, TF.silu(lin(gate, x)) * lin(up, x))
    return x, y, params


@pytest.mark.parametrize("T,H,I,r,dq", CASES)
def test_swiglu_forward_matches_unfused_kernels_bitwise(T, H, I, r, dq):
    gate, up, _ = _mlp(H, I, r, dq, seed=T)
    x = torch.randn(T, H, generator=torch.Generator(device=DEV).manual_seed(5), device=DEV).to(torch.bfloat16)
    xa = ops.mlp_lora_down(x, gate.lora_A, up.lora_A, gate.scaling, up.scaling) if r else None
    h, g_out, u_out = ops.nf4_swiglu_fwd(x, (gate.quantized, gate.quant_state), (up.quantized, up.quant_state), xa,
                                         gate.lora_B, up.lora_B)
    # bitwise: the same (one-SM) kernel family sums in the same order
    ops.set_gemm_kernel("single")
    try:
        with torch.no_grad():
            g_ref = ops.nf4_gemm_fwd(x, gate.quantized, gate.quant_state, lora_A=gate.lora_A, lora_B=gate.lora_B,
                                     scaling=gate.scaling)
            u_ref = ops.nf4_gemm_fwd(x, up.quantized, up.quant_state, lora_A=up.lora_A, lora_B=up.lora_B,
                                     scaling=up.scaling)
            h_ref = FZ.swiglu(g_ref, u_ref)
    finally:
        ops.set_gemm_kernel("auto")
    torch.cuda.synchronize()
    from stratum_b200 import _lib

    assert _lib.device_status() == 0
    assert torch.equal(g_out, g_ref)
    assert torch.equal(u_out, u_ref)
    assert torch.equal(h, h_ref)


def test_swiglu_backward_rows_match_the_separate_kernel_bitwise():
    """[dgate | dup] rows (the stacked input gradient's dY) equal the two-output kernel's."""
    T, I = 1000, 1536
    gen = torch.Generator(device=DEV).manual_seed(6)
    g = (torch.randn(T, I, generator=gen, device=DEV) * 2).to(torch.bfloat16)
    u = torch.randn(T, I, generator=gen, device=DEV).to(torch.bfloat16)
    dh = torch.randn(T, I, generator=gen, device=DEV).to(torch.bfloat16)
    dgu = FZ.swiglu_backward_cat(g, u, dh)
    gg, uu = g.clone().requires_grad_(), u.clone().requires_grad_()
    FZ.swiglu(gg, uu).backward(dh)
    torch.cuda.synchronize()
    assert torch.equal(dgu[:, :I], gg.grad)
    assert torch.equal(dgu[:, I:], uu.grad)


@pytest.mark.parametrize("fuse_forward", [True, False], ids=["fused-forward", "split-forward"])
@pytest.mark.parametrize("T,H,I,r,dq", CASES)
def test_fused_mlp_matches_fp32_reference(T, H, I, r, dq, fuse_forward):
    gate, up, down = _mlp(H, I, r, dq, seed=T + 2)
    mlp = FZ.FusedMLP(gate, up, down, fuse_forward=fuse_forward)
    gen = torch.Generator(device=DEV).manual_seed(7)
    x = torch.randn(1, T, H, generator=gen, device=DEV).to(torch.bfloat16).requires_grad_()
    assert FZ._fusable(gate, up, down, x)
    y = mlp(x)
    dy = torch.randn(y.shape, generator=gen, device=DEV).to(torch.bfloat16)
    y.backward(dy)
    xr, yr, params = _ref_fp32(x.detach()[0], gate, up, down)
    yr.backward(dy[0].float())
    assert relative_error(y.detach()[0].float(), yr.detach()) < 1e-2
    assert relative_error(x.grad[0].float(), xr.grad) < 1e-2
    if r:
        got = [p.grad.float() for m in (gate, up, down) for p in (m.lora_A, m.lora_B)]
        # reference order: gate (A, B), up (A, B), down (A, B) -- the order lin() ran
        for a, b in zip(got, params):
            assert relative_error(a, b.grad) < 1e-2


@pytest.mark.parametrize("T,H,I,r,dq", CASES[:2])
def test_fused_mlp_matches_hf_llama_mlp(T, H, I, r, dq):
    """Against transformers' LlamaMLP holding the dequantized weights, with each
    adapter added around its projection as PEFT's lora.Linear does."""
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaMLP

    gate, up, down = _mlp(H, I, r, dq, seed=T + 3)
    cfg = LlamaConfig(hidden_size=H, intermediate_size=I, hidden_act="silu", mlp_bias=False)
    hf = LlamaMLP(cfg).to(DEV, torch.bfloat16)

    class _Peft(torch.nn.Module):
        def __init__(self, m):
            super().__init__()
            self.weight = torch.nn.Parameter(F.dequantize_4bit(m.quantized, m.quant_state,
                                                               out_dtype=torch.bfloat16), requires_grad=False)
            self.A = None if m.lora_A is None else torch.nn.Parameter(m.lora_A.detach().clone())
            self.B = None if m.lora_B is None else torch.nn.Parameter(m.lora_B.detach().clone())
            self.s = m.scaling

        def forward(self, z):
            y = TF.linear(z, self.weight)
            return y if self.A is None else y + self.s * TF.linear(TF.linear(z, self.A), self.B)

    hf.gate_proj, hf.up_proj, hf.down_proj = _Peft(gate), _Peft(up), _Peft(down)
    gen = torch.Generator(device=DEV).manual_seed(8)
    x = torch.randn(1, T, H, generator=gen, device=DEV).to(torch.bfloat16)
    dy = torch.randn(1, T, H, generator=gen, device=DEV).to(torch.bfloat16)
    xi = x.clone().requires_grad_()
    y_ref = hf(xi)
    y_ref.backward(dy)
    ref = (y_ref.detach().float(), xi.grad.float())
    for fuse_forward in (False, True):
        for m in (gate, up, down):
            for p in (m.lora_A, m.lora_B):
                if p is not None:
                    p.grad = None
        xi = x.clone().requires_grad_()
        y = FZ.FusedMLP(gate, up, down, fuse_forward=fuse_forward)(xi)
        y.backward(dy)
        assert relative_error(y.detach().float(), ref[0]) < 1e-2
        assert relative_error(xi.grad.float(), ref[1]) < 1e-2
        if r:
            for name, m in (("gate_proj", gate), ("up_proj", up), ("down_proj", down)):
                p = getattr(hf, name)
                assert relative_error(m.lora_A.grad.float(), p.A.grad.float()) < 1e-2, name
                assert relative_error(m.lora_B.grad.float(), p.B.grad.float()) < 1e-2, name


@pytest.mark.parametrize("kernel,dq", [("single", False), ("pair", False), ("pair", True)])
def test_fused_mlp_pair_input_gradient_matches_two_passes(kernel, dq):
    """The stacked gate/up input gradient equals the sum of the two plain passes
    within one bf16 rounding of the sum, on both kernels."""
    T, H, I = 640, 512, 1024
    gate, up, _ = _mlp(H, I, 0, dq, seed=9)
    gen = torch.Generator(device=DEV).manual_seed(10)
    dgu = torch.randn(T, 2 * I, generator=gen, device=DEV).to(torch.bfloat16)
    ops.set_gemm_kernel(kernel)
    try:
        dx = ops.nf4_gemm_dx_pair(dgu, (gate.quantized, gate.quant_state), (up.quantized, up.quant_state))
    finally:
        ops.set_gemm_kernel("auto")
    ref = (dgu[:, :I].float() @ _w(gate)) + (dgu[:, I:].float() @ _w(up))
    assert relative_error(dx.float(), ref) < 1e-2
