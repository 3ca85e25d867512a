"""Decoder models around the NF4 path: prefix, wrapped layers, postfix.

The reference builds its models from HF modules and splits them into a
prefix (embedding + rotary), wrapped decoder layers and a postfix (final norm,
lm_head, chunked cross entropy), all passing the 7-tuple
``(hidden, causal_mask, position_ids, position_embeddings, kwargs, labels,
logits_to_keep)`` (stratum/model/llama.py:164-400; stratum/model/qwen3.py;
stratum/model/qwen3_moe.py).  This module does the same for the synthetic
benchmark models (random init, no checkpoint): HF decoder layers whose frozen
linears become fused-mode :class:`~stratum_b200.nf4_linear.NF4Linear`\\ s with a
LoRA adapter, and whose routed experts become
:class:`~stratum_b200.experts.NF4Experts`.

Attention is torch's ``scaled_dot_product_attention`` through HF's ``sdpa``
path (causal, no materialised mask: the reference's flash mode,
stratum/model/llama.py:229-231); it is library code, outside the NF4 path.
"""

from __future__ import annotations

from dataclasses import dataclass, replace
from typing import Optional

import torch
import torch.nn as nn

from . import upload
from .experts import NF4Experts
from .nf4_linear import NF4Linear


@dataclass(frozen=True)
class DecoderSpec:
    """Shape of a decoder-only LM (the fields the benchmark configs name)."""

    name: str
    family: str  # "llama" | "qwen3" | "qwen3_moe"
    layers: int
    hidden: int
    intermediate: int
    heads: int
    kv_heads: int
    head_dim: int
    vocab: int
    rope_theta: float
    experts: int = 0
    top_k: int = 0
    expert_intermediate: int = 0
    lora_r: int = 0
    lora_alpha: float = 16.0
    double_quant: bool = False
    router_aux_coef: float = 0.0
    rms_eps: float = 1e-6

    def scaled(self, **kw) -> "DecoderSpec":
        return replace(self, **kw)

    @property
    def linear_params_per_layer(self) -> int:
        attn = self.hidden * self.head_dim * (self.heads * 2 + self.kv_heads * 2)
        if self.experts:
            return attn + self.experts * 3 * self.hidden * self.expert_intermediate
        return attn + 3 * self.hidden * self.intermediate


# The benchmark configs (random init).  LoRA alpha: the reference hard-codes 16
# (scripts/train.py:569); the value does not change the work.
SPECS = {
    # config 5: Llama-3-8B-shaped, layer-parallel over 1/2/4/8 GPUs
    "llama3-8b": DecoderSpec("llama3-8b", "llama", 32, 4096, 14336, 32, 8, 128, 128256, 5e5,
                             lora_r=64, lora_alpha=16.0, double_quant=True),
    # config 3: Qwen3-0.6B-shaped, 1 GPU
    "qwen3-0.6b": DecoderSpec("qwen3-0.6b", "qwen3", 28, 1024, 3072, 16, 8, 128, 151936, 1e6,
                              lora_r=16, lora_alpha=16.0),
    # config 4: Qwen3-30B-A3B-shaped MoE, layer-parallel over 2/4/8 GPUs
    "qwen3-30b-a3b": DecoderSpec("qwen3-30b-a3b", "qwen3_moe", 48, 2048, 6144, 32, 4, 128, 151936, 1e6,
                                 experts=128, top_k=8, expert_intermediate=768, lora_r=16, lora_alpha=16.0,
                                 router_aux_coef=0.001),
}


def hf_config(spec: DecoderSpec):
    """The transformers config of ``spec`` (``sdpa`` attention)."""
    common = dict(vocab_size=spec.vocab, hidden_size=spec.hidden, num_hidden_layers=spec.layers,
                  num_attention_heads=spec.heads, num_key_value_heads=spec.kv_heads, head_dim=spec.head_dim,
                  rope_theta=spec.rope_theta, rms_norm_eps=spec.rms_eps, max_position_embeddings=131072,
                  tie_word_embeddings=False)
    if spec.family == "llama":
        from transformers import LlamaConfig

        cfg = LlamaConfig(intermediate_size=spec.intermediate, **common)
    elif spec.family == "qwen3":
        from transformers import Qwen3Config

        cfg = Qwen3Config(intermediate_size=spec.intermediate, **common)
    elif spec.family == "qwen3_moe":
        from transformers import Qwen3MoeConfig

        cfg = Qwen3MoeConfig(intermediate_size=spec.intermediate, moe_intermediate_size=spec.expert_intermediate,
                             num_experts=spec.experts, num_experts_per_tok=spec.top_k, norm_topk_prob=True,
                             router_aux_loss_coef=spec.router_aux_coef, decoder_sparse_step=1, **common)
    else:
        raise ValueError(f"unknown decoder family {spec.family!r}")
    cfg._attn_implementation = "sdpa"
    return cfg


def _layer_classes(spec: DecoderSpec):
    if spec.family == "llama":
        from transformers.models.llama import modeling_llama as m

        return m.LlamaDecoderLayer, m.LlamaRotaryEmbedding, m.LlamaRMSNorm
    if spec.family == "qwen3":
        from transformers.models.qwen3 import modeling_qwen3 as m

        return m.Qwen3DecoderLayer, m.Qwen3RotaryEmbedding, m.Qwen3RMSNorm
    from transformers.models.qwen3_moe import modeling_qwen3_moe as m

    return m.Qwen3MoeDecoderLayer, m.Qwen3MoeRotaryEmbedding, m.Qwen3MoeRMSNorm


def _device(device) -> torch.device:
    """``device`` with its index filled in (``"cuda"`` -> the current CUDA device)."""
    dev = torch.device(device) if not isinstance(device, int) else torch.device("cuda", device)
    if dev.type == "cuda" and dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    return dev


# --------------------------------------------------------------------------------
# router side channel (router aux loss)
# --------------------------------------------------------------------------------

class RouterLogitsSink:
    """Collects the router probabilities of MoE layers during a forward (the
    reference's router-logit side channel, stratum/moe.py:83-159)."""

    def __init__(self):
        self.active = False
        self.probs: list[torch.Tensor] = []
        self.indices: list[torch.Tensor] = []

    def clear(self) -> None:
        self.probs.clear()
        self.indices.clear()


class _RouterTap(nn.Module):
    """Wraps an HF top-k router; records (probs, top-k indices) when the sink is active."""

    def __init__(self, router: nn.Module, sink: RouterLogitsSink):
        super().__init__()
        self.router = router
        self.sink = sink

    def forward(self, hidden_states):
        probs, scores, indices = self.router(hidden_states)
        if self.sink.active:
            self.sink.probs.append(probs)
            self.sink.indices.append(indices)
        return probs, scores, indices


def load_balancing_terms(probs: torch.Tensor, indices: torch.Tensor, n_experts: int):
    """Per-expert sums behind the router aux loss of one layer's tokens.

    The reference's ``load_balancing_loss_func`` (stratum/moe.py:162-223, a copy
    of HF's) takes each layer's router output -- in transformers 5.x already a
    softmax -- applies softmax again, takes the top-k, and returns
    ``E * sum_e (count_e / N) * (psum_e / N)`` over all N (layer, token) rows,
    where ``count_e`` counts the top-k slots routed to expert e and ``psum_e``
    sums the re-softmaxed probabilities.  The top-k of the re-softmaxed row is
    the router's own top-k (softmax is monotonic), so ``indices`` are reused.
    Returns ``(count, psum)`` for these rows; sums over layers, microbatches and
    pipeline ranks combine exactly."""
    counts = torch.zeros(n_experts, dtype=torch.float32, device=probs.device)
    counts.index_add_(0, indices.reshape(-1), torch.ones(indices.numel(), dtype=torch.float32, device=probs.device))
    return counts, torch.softmax(probs.float(), dim=-1).sum(0)


# --------------------------------------------------------------------------------
# building layers
# --------------------------------------------------------------------------------

@torch.no_grad()
def _random_init_(module: nn.Module, std: float, gen: torch.Generator) -> None:
    for p in module.parameters():
        if p.ndim >= 2:
            p.normal_(0.0, std, generator=gen)


def build_layer(spec: DecoderSpec, idx: int, device, *, stream: bool = False, seed: int = 0,
                sink: Optional[RouterLogitsSink] = None, fused: bool = True) -> nn.Module:
    """One random-init decoder layer on ``device`` with NF4 frozen weights.

    Frozen linears are quantized on the GPU (``upload.prepare_nf4``), replaced by
    fused-mode ``NF4Linear``\\ s with a LoRA adapter of rank ``spec.lora_r``
    (``upload.to_nf4_linear``), and uploaded once (``stream=False``) or left as
    pinned host payloads for per-step streaming (``stream=True``).  Routed experts
    become a resident ``NF4Experts``; the router stays bf16 and frozen.  With
    ``fused`` the layer's RMSNorms, attention and (dense) MLP become the
    single-kernel modules of :mod:`stratum_b200.fused` around the same NF4Linears.
    """
    dev = _device(device)
    cls, _, _ = _layer_classes(spec)
    cfg = hf_config(spec)
    gen = torch.Generator(device=dev).manual_seed(seed * 1000003 + idx)
    with torch.device(dev):
        layer = cls(cfg, idx).to(torch.bfloat16)
    _random_init_(layer, 0.02, gen)
    layer.requires_grad_(False)
    targets: list[nn.Module] = [layer]
    if spec.experts:
        moe = layer.mlp
        moe.experts = NF4Experts.from_experts(moe.experts, device=dev, compress_statistics=spec.double_quant)
        if sink is not None:
            moe.gate = _RouterTap(moe.gate, sink)
        targets = [layer.self_attn]
    for t in targets:
        upload.prepare_nf4(t, verbose=False, compress_statistics=spec.double_quant, device=dev)
        upload.to_nf4_linear(t, lora_r=spec.lora_r, lora_alpha=spec.lora_alpha, lora_dtype=torch.bfloat16,
                             lora_device=dev)
    if fused:
        from .fused import FusedAttention, FusedMLP, FusedRMSNorm

        layer.input_layernorm = FusedRMSNorm.from_hf(layer.input_layernorm)
        layer.post_attention_layernorm = FusedRMSNorm.from_hf(layer.post_attention_layernorm)
        layer.self_attn = FusedAttention.from_hf(layer.self_attn, spec.heads, spec.kv_heads, spec.head_dim)
        if not spec.experts:
            mlp = layer.mlp
            layer.mlp = FusedMLP(mlp.gate_proj, mlp.up_proj, mlp.down_proj)
    with torch.no_grad():  # adapters drawn from the layer's own generator: builds are reproducible
        for m in layer.modules():
            if isinstance(m, NF4Linear) and m.lora_A is not None:
                bound = 1.0 / (m.in_features ** 0.5)  # kaiming-uniform(a=sqrt 5), PEFT's default for A
                m.lora_A.uniform_(-bound, bound, generator=gen)
    if stream:
        upload.build_layer_arena(layer)
    else:
        upload.ensure_weights(layer, dev)
    for name, p in layer.named_parameters():
        p.requires_grad_("lora_" in name)
    return layer


class Prefix(nn.Module):
    """Embedding + rotary embedding -> the 7-tuple (stratum/model/llama.py:164-249).

    The embedding is frozen bf16; no mask is materialised (the attention kernel
    is causal)."""

    def __init__(self, spec: DecoderSpec, device, *, seed: int = 0, with_embedding: bool = True):
        super().__init__()
        _, rot_cls, _ = _layer_classes(spec)
        dev = _device(device)
        self.spec = spec
        self.embed_tokens = None
        if with_embedding:
            self.embed_tokens = nn.Embedding(spec.vocab, spec.hidden, device=dev, dtype=torch.bfloat16)
            gen = torch.Generator(device=dev).manual_seed(seed * 1000003 + 999983)
            with torch.no_grad():
                self.embed_tokens.weight.normal_(0.0, 0.02, generator=gen)
            self.embed_tokens.requires_grad_(False)
        with torch.device(dev):
            self.rotary_emb = rot_cls(hf_config(spec))

    def context(self, hidden: torch.Tensor, labels=None, position_ids=None, **kwargs):
        """The 7-tuple around ``hidden`` (used by pipeline ranks that receive hidden)."""
        if position_ids is None:
            position_ids = torch.arange(hidden.shape[1], device=hidden.device).unsqueeze(0)
        pos_emb = self.rotary_emb(hidden, position_ids)
        return (hidden, None, position_ids, pos_emb, kwargs, labels, 0)

    def forward(self, input_ids=None, attention_mask=None, position_ids=None, labels=None, **kwargs):
        if self.embed_tokens is None:
            raise RuntimeError("Prefix built without an embedding")
        if attention_mask is not None and not bool(attention_mask.all()):
            raise ValueError("Prefix: padded batches need a materialised mask, which this prefix does not build")
        hidden = self.embed_tokens(input_ids)
        return self.context(hidden, labels=labels, position_ids=position_ids, **kwargs)


class WrappedLayer(nn.Module):
    """One decoder layer on the 7-tuple (stratum/model/llama.py:252-331)."""

    def __init__(self, layer: nn.Module, idx: int):
        super().__init__()
        self.layer = layer
        self.idx = idx

    def forward(self, input_data):
        hidden, causal_mask, pos_ids, pos_emb, kwargs, labels, lk = input_data
        out = self.layer(hidden, attention_mask=causal_mask, position_ids=pos_ids, past_key_values=None,
                         use_cache=False, position_embeddings=pos_emb)
        if isinstance(out, tuple):
            out = out[0]
        return (out, causal_mask, pos_ids, pos_emb, kwargs, labels, lk)


class _LMHeadCE(torch.autograd.Function):
    """Mean next-token cross entropy of ``h . W_lm^T`` with the gradient formed in
    the forward: the NF4 GEMM writes bf16 logits, one kernel turns each row into
    its loss and (softmax - onehot) in place, and one fused NF4 input-gradient
    GEMM takes those rows to dh.  The 1/N mean is applied as a tensor, so nothing
    waits on the host.

    ``chunk`` rows at a time (0: all rows in one pass): a chunk's logits are
    freed as soon as its dh rows are formed, so at most ``chunk x vocab`` 16-bit
    logits are live, and what the backward keeps is dh ([rows, H]).  Every row
    is computed independently, so the loss and dh do not depend on ``chunk``.
    Unchunked, the logits themselves are kept and dh is formed in the backward."""

    @staticmethod
    def forward(ctx, h, labels, lm_head, chunk):
        from . import _lib, ops

        qs = lm_head.quant_state
        rows = h.shape[0]
        lab = labels.to(torch.int64).contiguous()
        loss_rows = torch.empty(rows, dtype=torch.float32, device=h.device)
        n = (lab != -100).sum().clamp_min(1).to(torch.float32)
        chunk = rows if chunk <= 0 else min(chunk, rows)
        need_grad = ctx.needs_input_grad[0]
        dh = torch.empty_like(h) if (need_grad and chunk < rows) else None
        logits = None
        for r0 in range(0, rows, chunk):
            r1 = min(r0 + chunk, rows)
            logits = ops.nf4_gemm_fwd(h[r0:r1], lm_head.quantized, qs)
            vocab = logits.shape[1]
            with torch.cuda.device(h.device):
                _lib.check(_lib.lib().stratum_ce_fwd_grad(_lib.ptr(logits), _lib.DTYPE_CODE[logits.dtype],
                                                          _lib.ptr(lab[r0:r1]), r1 - r0, vocab, -100, 1.0,
                                                          _lib.ptr(loss_rows[r0:r1]), _lib.stream_of(h.device)),
                           "ce_fwd_grad")
            if dh is not None:
                ops.nf4_gemm_dx(logits, lm_head.quantized, qs, out=dh[r0:r1])
                logits = None
        ctx.lm_head = lm_head
        if dh is not None:
            ctx.save_for_backward(dh, n)
            ctx.formed = True
        else:
            ctx.save_for_backward(logits if need_grad else None, n)
            ctx.formed = False
        return loss_rows.sum() / n

    @staticmethod
    def backward(ctx, g):
        from . import ops

        saved, n = ctx.saved_tensors
        if ctx.formed:
            dh = saved
        else:
            m = ctx.lm_head
            dh = ops.nf4_gemm_dx(saved, m.quantized, m.quant_state)
        return dh * (g / n).to(dh.dtype), None, None, None


class Postfix(nn.Module):
    """Final norm + lm_head + next-token cross entropy (stratum/model/llama.py:334-399).

    The lm_head is a frozen NF4Linear.  The reference chunks the loss over tokens
    and recomputes each chunk's logits in the backward
    (stratum/model/chunked_loss.py:66-192); here each chunk's bf16 logits are
    formed once, overwritten with their own gradient by the cross-entropy kernel
    and taken to dh by one NF4 input-gradient GEMM, with no recompute and no
    dequantized lm_head.  ``token_chunk`` bounds the live logits to
    ``token_chunk x vocab``; 0 (the default) forms a microbatch's logits in one
    pass and keeps them until its backward, which fills the GPU best when that
    memory is available.  Returns the mean loss over non-ignored tokens."""

    def __init__(self, spec: DecoderSpec, device, *, seed: int = 0, token_chunk: int = 0):
        super().__init__()
        _, _, norm_cls = _layer_classes(spec)
        dev = _device(device)
        self.spec = spec
        self.token_chunk = token_chunk
        with torch.device(dev):
            self.norm = norm_cls(spec.hidden, eps=spec.rms_eps).to(torch.bfloat16)
            head = nn.Linear(spec.hidden, spec.vocab, bias=False, dtype=torch.bfloat16)
        gen = torch.Generator(device=dev).manual_seed(seed * 1000003 + 999979)
        with torch.no_grad():
            head.weight.normal_(0.0, 0.02, generator=gen)
        head.requires_grad_(False)
        holder = nn.Module()
        holder.lm_head = head
        upload.prepare_nf4(holder, verbose=False, compress_statistics=spec.double_quant, device=dev)
        upload.to_nf4_linear(holder)
        upload.ensure_weights(holder, dev)
        self.lm_head: NF4Linear = holder.lm_head
        self.norm.requires_grad_(False)

    def loss(self, hidden: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        h = self.norm(hidden)[:, :-1, :].reshape(-1, self.spec.hidden)
        y = labels[:, 1:].reshape(-1)
        return _LMHeadCE.apply(h, y, self.lm_head, int(self.token_chunk))

    def forward(self, input_data):
        hidden, _, _, _, _, labels, _ = input_data
        if labels is None:
            return None
        return self.loss(hidden, labels)


def reference_flops_per_token(spec: DecoderSpec, seq: int) -> float:
    """Algorithmic FLOPs per token of a training step (fwd + dX + LoRA grads,
    attention fwd + bwd causal, lm_head fwd + dX; recompute not counted)."""
    linear = 2.0 * spec.layers * spec.linear_params_per_layer
    if spec.experts:  # only top_k of the experts see a token
        attn = spec.hidden * spec.head_dim * (spec.heads * 2 + spec.kv_heads * 2)
        linear = 2.0 * spec.layers * (attn + spec.top_k * 3 * spec.hidden * spec.expert_intermediate)
    fwd_bwd_linear = 2.0 * linear  # forward + input gradient (weights frozen)
    lora = 0.0
    if spec.lora_r:
        dims = [(spec.hidden, spec.heads * spec.head_dim), (spec.hidden, spec.kv_heads * spec.head_dim),
                (spec.hidden, spec.kv_heads * spec.head_dim), (spec.heads * spec.head_dim, spec.hidden)]
        if not spec.experts:
            dims += [(spec.hidden, spec.intermediate)] * 2 + [(spec.intermediate, spec.hidden)]
        lora = spec.layers * sum(2.0 * spec.lora_r * (k + n) * 3 for k, n in dims)
    # causal attention: QK^T and PV, half the square, fwd (1x) + bwd (2x)
    attn_flops = spec.layers * 4.0 * seq * spec.heads * spec.head_dim * 0.5 * 3
    head = 2.0 * spec.hidden * spec.vocab * 2
    return fwd_bwd_linear + lora + attn_flops + head


__all__ = ["DecoderSpec", "SPECS", "hf_config", "build_layer", "Prefix", "WrappedLayer", "Postfix",
           "RouterLogitsSink", "load_balancing_terms", "reference_flops_per_token"]
