"""GPU: the NF4 decoder through the pipelines against plain autograd.

Small Llama / Qwen3-MoE-shaped decoders (HF layers with fused NF4Linear + LoRA
and NF4Experts) run (a) as one plain autograd graph and (b) through
``StratumPipeline`` (per-layer recompute anchors, two stages, resident or
per-step streamed NF4 weights) or ``RankPipeline`` (one rank, several
microbatches).  Loss and LoRA gradients must agree within the GEMM tolerance
(||a - b|| / ||b|| <= 1e-2; attention backward is not bit-deterministic)."""

import os
import socket
import tempfile

import pytest
import torch
import torch.multiprocessing as mp

from oracle.nf4_oracle import relative_error
from stratum_b200 import decoder as D
from stratum_b200.pipeline import RankPipeline, StratumPipeline
from stratum_b200.stage import DeviceStage

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
TOL = 1e-2

TINY_LLAMA = D.DecoderSpec("tiny-llama", "llama", 4, 256, 512, 4, 2, 64, 1000, 5e5, lora_r=8, lora_alpha=16.0,
                           double_quant=True)
TINY_MOE = D.DecoderSpec("tiny-moe", "qwen3_moe", 3, 256, 512, 4, 2, 64, 1000, 1e6, experts=16, top_k=4,
                         expert_intermediate=128, lora_r=8, lora_alpha=16.0, router_aux_coef=0.01)


def _build(spec, stream=False, seed=0):
    sink = D.RouterLogitsSink() if spec.experts else None
    layers = [D.WrappedLayer(D.build_layer(spec, i, DEV, stream=stream, seed=seed, sink=sink), i)
              for i in range(spec.layers)]
    prefix = D.Prefix(spec, DEV, seed=seed)
    postfix = D.Postfix(spec, DEV, seed=seed, token_chunk=96)
    with torch.no_grad():  # LoRA B starts at zero; give it values so dA is not trivially zero
        g = torch.Generator(device=DEV).manual_seed(5)
        for l in layers:
            for n, p in l.named_parameters():
                if n.endswith("lora_B"):
                    p.normal_(0.0, 0.02, generator=g)
    return prefix, layers, postfix, sink


def _lora_grads(layers):
    return {f"{i}.{n}": p.grad.detach().clone() for i, l in enumerate(layers) for n, p in l.named_parameters()
            if p.requires_grad}


def _zero(layers):
    for l in layers:
        for p in l.parameters():
            p.grad = None


def _plain(prefix, layers, postfix, sink, spec, ids, labels):
    """One autograd graph over the whole model (the reference's layer semantics)."""
    if sink is not None:
        sink.clear()
        sink.active = True
    tup = prefix(input_ids=ids, labels=labels)
    for l in layers:
        tup = l(tup)
    if sink is not None:
        sink.active = False
    loss = postfix(tup)
    if sink is not None:
        cat = torch.cat(list(sink.probs), 0)
        rw = torch.softmax(cat.float(), -1)
        _, sel = torch.topk(rw, spec.top_k, -1)
        mask = torch.nn.functional.one_hot(sel, spec.experts).float()
        aux = torch.sum(mask.mean(0) * rw.mean(0).unsqueeze(0)) * spec.experts
        loss = loss + spec.router_aux_coef * aux
        sink.clear()
    loss.backward()
    return loss.detach()


def _data(spec, m=1, seq=192):
    g = torch.Generator(device=DEV).manual_seed(3)
    ids = torch.randint(0, spec.vocab, (m, seq), generator=g, device=DEV)
    return ids, ids.clone()


def _compare(loss_a, grads_a, loss_b, grads_b):
    assert relative_error(loss_a.float().reshape(1), loss_b.float().reshape(1)) < 1e-3
    assert set(grads_a) == set(grads_b)
    for k in grads_b:
        err = relative_error(grads_a[k].float(), grads_b[k].float())
        assert err < TOL, f"{k}: rel err {err}"


@pytest.mark.parametrize("spec", [TINY_LLAMA, TINY_MOE], ids=["llama", "qwen3-moe"])
def test_stratum_pipeline_matches_plain_autograd(spec):
    prefix, layers, postfix, sink = _build(spec)
    ids, labels = _data(spec)
    ref_loss = _plain(prefix, layers, postfix, sink, spec, ids, labels)
    ref = _lora_grads(layers)
    _zero(layers)
    stages = [DeviceStage(layers[:2], 0), DeviceStage(layers[2:], 0)]
    pipe = StratumPipeline(prefix, stages, postfix, router_sink=sink, router_aux_coef=spec.router_aux_coef,
                           n_experts=spec.experts)
    loss = pipe(ids, labels=labels)
    loss.backward()
    torch.cuda.synchronize()
    _compare(loss.detach(), _lora_grads(layers), ref_loss, ref)


def test_streamed_weights_match_resident_weights():
    spec = TINY_LLAMA
    prefix, layers, postfix, _ = _build(spec, stream=False)
    ids, labels = _data(spec)
    ref_loss = _plain(prefix, layers, postfix, None, spec, ids, labels)
    ref = _lora_grads(layers)
    prefix2, layers2, postfix2, _ = _build(spec, stream=True)
    pipe = StratumPipeline(prefix2, [DeviceStage(layers2, 0)], postfix2, prefetch_nf4=True)
    for _ in range(2):  # the second step re-uploads what the first freed
        _zero(layers2)
        loss = pipe(ids, labels=labels)
        loss.backward()
        torch.cuda.synchronize()
        _compare(loss.detach(), _lora_grads(layers2), ref_loss, ref)
    # every streamed layer's device copy was freed after its backward
    assert not any(m.quantized is not None for l in layers2 for m in l.modules()
                   if type(m).__name__ == "NF4Linear" and m.streamed)


def test_rank_pipeline_single_rank_microbatches():
    spec = TINY_LLAMA
    prefix, layers, postfix, _ = _build(spec, stream=True)
    ids, labels = _data(spec, m=3)
    pipe = RankPipeline(DeviceStage(layers, 0), prefix=prefix, postfix=postfix, rank=0, world=1,
                        hidden_size=spec.hidden)
    loss = pipe.train_step(ids, labels, microbatches=3)
    got = _lora_grads(layers)
    _zero(layers)
    plain = StratumPipeline(prefix, [DeviceStage(layers, 0)], postfix)
    total = 0.0
    for m in range(3):
        l = plain(ids[m:m + 1], labels=labels[m:m + 1]) / 3
        l.backward()
        total = total + l.detach()
    torch.cuda.synchronize()
    _compare(loss, got, total, _lora_grads(layers))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_rank(rank, world, port, out_dir, M):
    import torch.distributed as dist
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from stratum_b200.assign import assign_layers_to_devices, strata

        spec = TINY_LLAMA
        dev = f"cuda:{rank}"
        mine = strata(assign_layers_to_devices(spec.layers, n_devices=world))[rank][1]
        layers = [D.WrappedLayer(D.build_layer(spec, i, dev, stream=True, seed=0), i) for i in mine]
        with torch.no_grad():
            for l in layers:
                idx = l.idx
                g = torch.Generator(device=dev).manual_seed(1000 + idx)
                for n, p in l.named_parameters():
                    if n.endswith("lora_B"):
                        p.normal_(0.0, 0.02, generator=g)
        prefix = D.Prefix(spec, dev, seed=0, with_embedding=rank == 0)
        postfix = D.Postfix(spec, dev, seed=0, token_chunk=96) if rank == world - 1 else None
        pipe = RankPipeline(DeviceStage(layers, rank), prefix=prefix, postfix=postfix, rank=rank, world=world,
                            hidden_size=spec.hidden)
        g = torch.Generator(device=dev).manual_seed(3)
        ids = torch.randint(0, spec.vocab, (M, 192), generator=g, device=dev)
        loss = pipe.train_step(ids if rank == 0 else None, ids if rank == world - 1 else None, microbatches=M,
                               seq_len=192)
        torch.cuda.synchronize()
        grads = {f"{l.idx}.{n}": p.grad.cpu() for l in layers for n, p in l.named_parameters() if p.requires_grad}
        torch.save({"loss": None if loss is None else loss.cpu(), "grads": grads},
                   os.path.join(out_dir, f"rank{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_nccl_pipeline_matches_one_gpu():
    spec, M = TINY_LLAMA, 3
    prefix, layers, postfix, _ = _build(spec, seed=0)
    with torch.no_grad():  # the same LoRA B values the ranks draw
        for l in layers:
            g = torch.Generator(device=DEV).manual_seed(1000 + l.idx)
            for n, p in l.named_parameters():
                if n.endswith("lora_B"):
                    p.normal_(0.0, 0.02, generator=g)
    g = torch.Generator(device=DEV).manual_seed(3)
    ids = torch.randint(0, spec.vocab, (M, 192), generator=g, device=DEV)
    one = RankPipeline(DeviceStage(layers, 0), prefix=prefix, postfix=postfix, rank=0, world=1,
                       hidden_size=spec.hidden)
    ref_loss = one.train_step(ids, ids, microbatches=M)
    ref = {k: v.cpu() for k, v in _lora_grads(layers).items()}
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_nccl_rank, args=(2, _free_port(), d, M), nprocs=2, start_method="spawn", join=True)
        outs = [torch.load(os.path.join(d, f"rank{r}.pt")) for r in range(2)]
    got = {}
    for o in outs:
        got.update(o["grads"])
    _compare(outs[1]["loss"], got, ref_loss.cpu(), ref)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_stratum_pipeline_across_two_devices_matches_one_device():
    """Two stages on two GPUs (NVLink boundary copies, gradient copied back the same
    way) against the same layers on one GPU."""
    spec = TINY_LLAMA
    ids, labels = _data(spec)
    prefix, layers, postfix, _ = _build(spec, stream=True)
    one = StratumPipeline(prefix, [DeviceStage(layers, 0)], postfix, prefetch_nf4=True)
    loss1 = one(ids, labels=labels)
    loss1.backward()
    ref = _lora_grads(layers)
    # the same model with layers 2.. and the postfix on cuda:1
    prefix2 = D.Prefix(spec, "cuda:0", seed=0)
    l0 = [D.WrappedLayer(D.build_layer(spec, i, "cuda:0", stream=True, seed=0), i) for i in range(2)]
    l1 = [D.WrappedLayer(D.build_layer(spec, i, "cuda:1", stream=True, seed=0), i) for i in range(2, spec.layers)]
    post2 = D.Postfix(spec, "cuda:1", seed=0, token_chunk=96)
    with torch.no_grad():
        g = torch.Generator(device=DEV).manual_seed(5)
        for l in l0 + l1:
            for n, p in l.named_parameters():
                if n.endswith("lora_B"):
                    p.copy_(torch.empty(p.shape, dtype=p.dtype, device=DEV).normal_(0.0, 0.02, generator=g))
    two = StratumPipeline(prefix2, [DeviceStage(l0, 0), DeviceStage(l1, 1)], post2, prefetch_nf4=True)
    loss2 = two(ids, labels=labels)
    loss2.backward()
    torch.cuda.synchronize(0)
    torch.cuda.synchronize(1)
    got = {k: v.to(DEV) for k, v in _lora_grads(l0 + l1).items()}
    _compare(loss2.detach().to(DEV), got, loss1.detach(), ref)


def test_rank_pipeline_cuda_graph_matches_eager():
    """One rank, resident weights: microbatches replayed from a captured CUDA graph give the
    eager path's loss and LoRA gradients (twice, so the second step reuses the graph), and
    a new microbatch count rebuilds it."""
    spec = TINY_LLAMA
    prefix, layers, postfix, _ = _build(spec)
    ids, labels = _data(spec, m=3)

    def run(graph, m=3, steps=1):
        _zero(layers)
        pipe = RankPipeline(DeviceStage(layers, 0), prefix=prefix, postfix=postfix, rank=0, world=1,
                            hidden_size=spec.hidden, schedule="1f1b", recompute=False, cuda_graph=graph)
        loss = None
        for _ in range(steps):
            _zero(layers)
            loss = pipe.train_step(ids[:m], labels[:m], microbatches=m)
        torch.cuda.synchronize()
        return pipe, loss, _lora_grads(layers)

    _, loss_e, grads_e = run(False)
    pipe, loss_g, grads_g = run(True, steps=2)
    _compare(loss_g, grads_g, loss_e, grads_e)
    # a different microbatch count rebuilds the graph
    _, loss_e2, grads_e2 = run(False, m=2)
    _zero(layers)
    loss_g2 = pipe.train_step(ids[:2], labels[:2], microbatches=2)
    torch.cuda.synchronize()
    _compare(loss_g2, _lora_grads(layers), loss_e2, grads_e2)
    # a parameter replaced (not updated in place) is seen: the graph is captured again
    with torch.no_grad():
        lb = next(p for n, p in layers[0].named_parameters() if n.endswith("lora_B"))
        lb.data = lb.data * 1.5
    _, loss_e3, grads_e3 = run(False, m=2)
    _zero(layers)
    loss_g3 = pipe.train_step(ids[:2], labels[:2], microbatches=2)
    torch.cuda.synchronize()
    _compare(loss_g3, _lora_grads(layers), loss_e3, grads_e3)
    # gradients accumulate into existing .grad as the eager path's do
    before = _lora_grads(layers)
    pipe.train_step(ids[:2], labels[:2], microbatches=2)
    torch.cuda.synchronize()
    after = _lora_grads(layers)
    for k in before:
        assert relative_error(after[k].float(), 2 * before[k].float()) < TOL, k
