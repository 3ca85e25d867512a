"""GPU parity of the fused decoder-layer kernels against HF's own modules.

RMSNorm, rotary embedding and SwiGLU reproduce HF's forward arithmetic (the
same bf16 roundings), so their outputs match to the last bit except where a
reduction order differs (RMSNorm's mean: at most one bf16 ulp); backwards are
compared with torch autograd of the HF forward within 1e-2 relative.  A whole
decoder layer with the fused modules is compared with the HF layer holding the
same NF4 weights and LoRA adapters."""

import pytest
import torch
import torch.nn.functional as TF

from oracle.nf4_oracle import relative_error
from stratum_b200 import decoder as D
from stratum_b200 import fused as FZ

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _ulps_bf16(a, b):
    ai = a.view(torch.int16).int()
    bi = b.view(torch.int16).int()
    return (ai - bi).abs().max().item()


@pytest.mark.parametrize("n", [1024, 4096, 128])
def test_rmsnorm_matches_hf(n):
    from transformers.models.llama.modeling_llama import LlamaRMSNorm

    g = torch.Generator(device=DEV).manual_seed(n)
    x = (torch.randn(777, n, generator=g, device=DEV) * 3).to(torch.bfloat16).requires_grad_()
    hf = LlamaRMSNorm(n, eps=1e-6).to(DEV, torch.bfloat16)
    with torch.no_grad():
        hf.weight.copy_(torch.rand(n, generator=g, device=DEV) + 0.5)
    hf.weight.requires_grad_(False)
    ref = hf(x)
    dy = torch.randn_like(ref)
    ref.backward(dy)
    ref_dx = x.grad.clone()
    x.grad = None
    mod = FZ.FusedRMSNorm.from_hf(hf)
    y = mod(x)
    y.backward(dy)
    assert _ulps_bf16(y.detach(), ref.detach()) <= 1
    assert relative_error(x.grad.float(), ref_dx.float()) < 1e-2


def test_swiglu_matches_hf():
    g0 = torch.Generator(device=DEV).manual_seed(1)
    g = (torch.randn(513, 3072, generator=g0, device=DEV) * 3).to(torch.bfloat16).requires_grad_()
    u = torch.randn(513, 3072, generator=g0, device=DEV).to(torch.bfloat16).requires_grad_()
    ref = TF.silu(g) * u
    dh = torch.randn_like(ref)
    ref.backward(dh)
    rg, ru = g.grad.clone(), u.grad.clone()
    g.grad = u.grad = None
    h = FZ.swiglu(g, u)
    h.backward(dh)
    assert torch.equal(h.detach(), ref.detach())
    assert relative_error(u.grad.float(), ru.float()) < 1e-2
    assert relative_error(g.grad.float(), rg.float()) < 1e-2


@pytest.mark.parametrize("H", [32, 8])
def test_rope_to_heads_matches_hf(H):
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding, apply_rotary_pos_emb

    S, Dh = 1000, 128
    cfg = LlamaConfig(hidden_size=H * Dh, num_attention_heads=H, head_dim=Dh, rope_theta=5e5)
    rot = LlamaRotaryEmbedding(cfg, device=DEV)
    g0 = torch.Generator(device=DEV).manual_seed(2)
    x = torch.randn(S, H * Dh, generator=g0, device=DEV).to(torch.bfloat16).requires_grad_()
    cos, sin = rot(x, torch.arange(S, device=DEV)[None])
    xh = x.view(1, S, H, Dh).transpose(1, 2)
    ref, _ = apply_rotary_pos_emb(xh, xh, cos, sin)
    dy = torch.randn_like(ref)
    ref.backward(dy)
    rdx = x.grad.clone()
    x.grad = None
    y = FZ.to_heads(x, H, Dh, cos[0], sin[0])
    y.backward(dy)
    assert torch.equal(y.detach(), ref.detach().contiguous())
    assert relative_error(x.grad.float(), rdx.float()) < 1e-2
    t = FZ.to_tokens(y.detach())
    assert torch.equal(t, y.detach().transpose(1, 2).reshape(S, H * Dh))


@pytest.mark.parametrize("family", ["llama", "qwen3"])
def test_fused_layer_matches_hf_layer(family):
    spec = D.DecoderSpec("t", family, 1, 512, 1024, 8, 4, 64, 1000, 5e5, lora_r=8)
    hf = D.build_layer(spec, 0, DEV, seed=3, fused=False)
    fz = D.build_layer(spec, 0, DEV, seed=3, fused=True)
    with torch.no_grad():  # same non-zero LoRA B in both
        g = torch.Generator(device=DEV).manual_seed(9)
        bs = {}
        for n, p in hf.named_parameters():
            if n.endswith("lora_B"):
                bs[n.split(".")[-2]] = torch.randn(p.shape, generator=g, device=DEV).to(p.dtype) * 0.02
                p.copy_(bs[n.split(".")[-2]])
        for n, p in fz.named_parameters():
            if n.endswith("lora_B"):
                p.copy_(bs[n.split(".")[-2]])
    prefix = D.Prefix(spec, DEV, seed=3)
    ids = torch.randint(0, spec.vocab, (1, 256), device=DEV)
    tup = prefix(input_ids=ids)
    x = (tup[0].detach() * 50).requires_grad_()
    outs, grads = [], []
    for layer in (hf, fz):
        x.grad = None
        w = D.WrappedLayer(layer, 0)
        y = w((x,) + tup[1:])[0]
        y.backward(torch.ones_like(y) * 0.01)
        outs.append(y.detach())
        grads.append((x.grad.clone(), {n.split(".")[-2]: p.grad.clone() for n, p in layer.named_parameters()
                                       if p.requires_grad}))
    assert relative_error(outs[1].float(), outs[0].float()) < 1e-2
    assert relative_error(grads[1][0].float(), grads[0][0].float()) < 1e-2
    assert set(grads[1][1]) == set(grads[0][1])
    for k in grads[0][1]:
        assert relative_error(grads[1][1][k].float(), grads[0][1][k].float()) < 1e-2, k


def test_lm_head_cross_entropy_matches_torch():
    """Postfix's fused lm_head + CE against F.cross_entropy over the same bf16 logits."""
    spec = D.DecoderSpec("t", "llama", 1, 256, 512, 4, 2, 64, 1000, 5e5)
    post = D.Postfix(spec, DEV, seed=1)
    g0 = torch.Generator(device=DEV).manual_seed(4)
    hidden = torch.randn(1, 300, 256, generator=g0, device=DEV).to(torch.bfloat16).requires_grad_()
    labels = torch.randint(0, 1000, (1, 300), generator=g0, device=DEV)
    labels[0, 10:20] = -100
    loss = post.loss(hidden, labels)
    loss.backward()
    gh = hidden.grad.clone()
    hidden.grad = None
    w = post.lm_head.weight_dequantized.to(torch.bfloat16)
    h = post.norm(hidden)[:, :-1].reshape(-1, 256)
    logits = (h @ w.t()).float()
    ref = TF.cross_entropy(logits, labels[:, 1:].reshape(-1), ignore_index=-100)
    ref.backward()
    assert abs(float(loss.detach()) - float(ref.detach())) < 1e-2 * abs(float(ref.detach()))
    assert relative_error(gh.float(), hidden.grad.float()) < 1e-2


def test_lm_head_chunked_equals_unchunked_and_bounds_logits_memory():
    """token_chunk changes only how many logits are live: loss and dh are the same
    bits (every row is computed alone), and 256-row chunks hold a fraction of the
    full [rows, vocab] logits."""
    spec = D.DecoderSpec("t", "llama", 1, 256, 512, 4, 2, 64, 32000, 5e5)
    post = D.Postfix(spec, DEV, seed=2)
    g0 = torch.Generator(device=DEV).manual_seed(5)
    hidden = torch.randn(1, 2048, 256, generator=g0, device=DEV).to(torch.bfloat16).requires_grad_()
    labels = torch.randint(0, 32000, (1, 2048), generator=g0, device=DEV)
    labels[0, 100:400] = -100
    out = {}
    for chunk in (0, 256, 700):
        post.token_chunk = chunk
        hidden.grad = None
        torch.cuda.synchronize()
        base = torch.cuda.memory_allocated()
        torch.cuda.reset_peak_memory_stats()
        loss = post.loss(hidden, labels)
        torch.cuda.synchronize()
        peak = torch.cuda.max_memory_allocated() - base
        loss.backward()
        out[chunk] = (loss.detach().clone(), hidden.grad.clone(), peak)
    for chunk in (256, 700):
        assert torch.equal(out[chunk][0], out[0][0]), chunk
        assert torch.equal(out[chunk][1], out[0][1]), chunk
    logits_bytes = 2047 * 32000 * 2
    assert out[0][2] >= logits_bytes
    assert out[256][2] < logits_bytes // 4
