"""The C-ABI entry points can be captured into CUDA graphs (the bench and the
pipeline replay captured steps): a captured call must not query anything the
driver forbids during capture, and its replay must reproduce the eager result
bit for bit (same kernels, same inputs)."""

import pytest
import torch

from stratum_b200 import _lib, ops
from stratum_b200 import functional as F
from stratum_b200.experts import NF4Experts

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _capture(fn):
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = fn()
    return g, out


def test_codec_and_gemm_calls_replay_from_a_graph():
    g0 = torch.Generator(device=DEV).manual_seed(0)
    w = (torch.randn(512, 256, generator=g0, device=DEV) * 0.02).half()
    x = torch.randn(300, 256, generator=g0, device=DEV).to(torch.bfloat16)
    dy = torch.randn(300, 512, generator=g0, device=DEV).to(torch.bfloat16)

    def step():
        packed, qs = F.quantize_4bit(w, compress_statistics=True)
        wd = F.dequantize_4bit(packed, qs, out_dtype=torch.bfloat16)
        y = ops.nf4_gemm_fwd(x, packed, qs)
        dx = ops.nf4_gemm_dx(dy, packed, qs)
        return packed, wd, y, dx

    eager = step()
    torch.cuda.synchronize()
    g, captured = _capture(step)
    g.replay()
    torch.cuda.synchronize()
    for a, b in zip(eager, captured):
        assert torch.equal(a, b)
    assert _lib.device_status() == 0


def test_experts_forward_backward_replays_from_a_graph():
    E, H, I, T, k = 16, 512, 256, 500, 4
    g0 = torch.Generator(device=DEV).manual_seed(1)
    holder = torch.nn.Module()
    holder.gate_up_proj = torch.nn.Parameter((torch.randn(E, 2 * I, H, generator=g0, device=DEV) * 0.02).half(),
                                             requires_grad=False)
    holder.down_proj = torch.nn.Parameter((torch.randn(E, H, I, generator=g0, device=DEV) * 0.02).half(),
                                          requires_grad=False)
    mod = NF4Experts.from_experts(holder)
    x = torch.randn(T, H, generator=g0, device=DEV).to(torch.bfloat16).requires_grad_()
    probs = torch.softmax(torch.randn(T, E, generator=g0, device=DEV), -1)
    wts, idx = torch.topk(probs, k, -1)
    wts = wts.requires_grad_()
    dout = torch.randn(T, H, generator=g0, device=DEV).to(torch.bfloat16)

    def step():
        x.grad = None
        wts.grad = None
        out = mod(x, idx, wts)
        out.backward(dout)
        return out

    out_e = step().detach().clone()
    gx_e, gw_e = x.grad.clone(), wts.grad.clone()
    g, out_c = _capture(step)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out_c, out_e)
    assert torch.equal(x.grad, gx_e)
    assert torch.equal(wts.grad, gw_e)
