"""Pipeline schedule and boundary logic on the CPU (no GPU, gloo ranks).

A toy model with the reference's 7-tuple layer interface (frozen weights, a
trainable low-rank term per layer, and optionally a top-k router whose outputs
feed the router aux loss) runs through ``StratumPipeline`` (one process) and
``RankPipeline`` (two gloo ranks, NCCL's role played by gloo send/recv).  Loss
and every trainable gradient must match plain autograd over the same model:
the recompute anchors, the boundary gradients and the aux-loss injection are
exact up to float reassociation."""

import os
import socket
import tempfile

import pytest
import torch
import torch.multiprocessing as mp
import torch.nn as nn
import torch.nn.functional as TF

from stratum_b200.decoder import RouterLogitsSink, _RouterTap
from stratum_b200.pipeline import RankPipeline, StratumPipeline
from stratum_b200.stage import DeviceStage

H, V, S, E, K = 32, 50, 12, 6, 2
COEF = 0.05


class ToyRouter(nn.Module):
    def __init__(self, g):
        super().__init__()
        self.weight = nn.Parameter(torch.randn(E, H, generator=g) * 0.3, requires_grad=False)

    def forward(self, h):
        probs = torch.softmax(TF.linear(h, self.weight), dim=-1, dtype=torch.float)
        top, idx = torch.topk(probs, K, dim=-1)
        return probs, top, idx


class ToyLayer(nn.Module):
    def __init__(self, i, sink=None):
        super().__init__()
        g = torch.Generator().manual_seed(100 + i)
        self.W = nn.Parameter(torch.randn(H, H, generator=g) / H**0.5, requires_grad=False)
        self.A = nn.Parameter(torch.randn(4, H, generator=g) * 0.1)
        self.B = nn.Parameter(torch.randn(H, 4, generator=g) * 0.1)
        self.gate = _RouterTap(ToyRouter(g), sink) if sink is not None else None

    def forward(self, tup):
        h = tup[0]
        y = h + torch.tanh(h @ self.W.t()) + (h @ self.A.t()) @ self.B.t()
        if self.gate is not None:
            _, top, _ = self.gate(h.reshape(-1, H))
            y = y + 0.1 * top.sum(-1).reshape(h.shape[:-1]).unsqueeze(-1).to(y.dtype) * h
        return (y,) + tuple(tup[1:])


class ToyPrefix(nn.Module):
    def __init__(self):
        super().__init__()
        g = torch.Generator().manual_seed(7)
        self.table = nn.Parameter(torch.randn(V, H, generator=g), requires_grad=False)

    def context(self, hidden, labels=None, **kw):
        pos = torch.arange(hidden.shape[1]).unsqueeze(0)
        return (hidden, None, pos, None, kw, labels, 0)

    def forward(self, input_ids=None, attention_mask=None, labels=None, **kw):
        return self.context(self.table[input_ids], labels=labels)


class ToyPostfix(nn.Module):
    def __init__(self):
        super().__init__()
        g = torch.Generator().manual_seed(8)
        self.head = nn.Parameter(torch.randn(V, H, generator=g) / H**0.5, requires_grad=False)

    def forward(self, tup):
        h, labels = tup[0], tup[5]
        logits = h[:, :-1] @ self.head.t()
        return TF.cross_entropy(logits.reshape(-1, V), labels[:, 1:].reshape(-1))


def _model(n_layers, moe, sink=None):
    return [ToyLayer(i, sink if moe else None) for i in range(n_layers)]


def _data(m):
    g = torch.Generator().manual_seed(11)
    ids = torch.randint(0, V, (m, S), generator=g)
    return ids, ids.clone()


def _hf_aux(probs):
    """The reference's load_balancing_loss_func (stratum/moe.py:162-223) restated."""
    cat = torch.cat(probs, 0)
    rw = torch.softmax(cat, dim=-1)
    _, sel = torch.topk(rw, K, dim=-1)
    mask = TF.one_hot(sel, E).float()
    return torch.sum(mask.mean(0) * rw.mean(0).unsqueeze(0)) * E


def _reference(n_layers, moe, ids, labels):
    """Plain autograd, microbatch by microbatch; returns (mean loss, grads)."""
    prefix, postfix = ToyPrefix(), ToyPostfix()
    sink = RouterLogitsSink()
    layers = _model(n_layers, moe, sink)
    total = 0.0
    M = ids.shape[0]
    for m in range(M):
        sink.clear()
        sink.active = moe
        tup = prefix(input_ids=ids[m:m + 1], labels=labels[m:m + 1])
        for l in layers:
            tup = l(tup)
        sink.active = False
        loss = postfix(tup)
        if moe:
            loss = loss + COEF * _hf_aux(list(sink.probs))
        (loss / M).backward()
        total += float(loss.detach()) / M
    grads = {f"{i}.{n}": p.grad.clone() for i, l in enumerate(layers) for n, p in l.named_parameters()
             if p.requires_grad}
    return total, grads


@pytest.mark.parametrize("moe", [False, True])
def test_single_process_pipeline_matches_autograd(moe):
    ids, labels = _data(1)
    ref_loss, ref_grads = _reference(6, moe, ids, labels)
    sink = RouterLogitsSink()
    layers = _model(6, moe, sink)
    stages = [DeviceStage(layers[:2], "cpu"), DeviceStage(layers[2:5], "cpu"), DeviceStage(layers[5:], "cpu")]
    pipe = StratumPipeline(ToyPrefix(), stages, ToyPostfix(), router_sink=sink if moe else None,
                           router_aux_coef=COEF if moe else 0.0, n_experts=E)
    loss = pipe(ids, labels=labels)
    loss.backward()
    assert abs(float(loss) - ref_loss) < 1e-5
    got = {f"{i}.{n}": p.grad for i, l in enumerate(layers) for n, p in l.named_parameters() if p.requires_grad}
    for k, g in ref_grads.items():
        torch.testing.assert_close(got[k], g, rtol=1e-4, atol=1e-6, msg=k)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir, moe, M, n_layers, schedule="gpipe", recompute=True):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from stratum_b200.assign import assign_layers_to_devices, strata

        sink = RouterLogitsSink()
        layers = _model(n_layers, moe, sink)
        parts = strata(assign_layers_to_devices(n_layers, n_devices=world))
        mine = parts[rank][1]
        stage = DeviceStage([layers[i] for i in mine], "cpu")
        pipe = RankPipeline(stage, prefix=ToyPrefix(), postfix=ToyPostfix() if rank == world - 1 else None,
                            rank=rank, world=world, hidden_size=H, hidden_dtype=torch.float32,
                            router_sink=sink if moe else None, router_aux_coef=COEF if moe else 0.0,
                            n_experts=E if moe else 0, schedule=schedule, recompute=recompute)
        ids, labels = _data(M)
        loss = pipe.train_step(ids if rank == 0 else None, labels if rank == world - 1 else None,
                               microbatches=M, seq_len=S)
        grads = {f"{i}.{n}": p.grad for i in mine for n, p in layers[i].named_parameters() if p.requires_grad}
        torch.save({"loss": None if loss is None else float(loss), "grads": grads},
                   os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("moe,world,schedule,recompute", [
    (False, 2, "gpipe", True), (True, 2, "gpipe", True),
    (False, 3, "1f1b", False), (False, 2, "1f1b", True),
    (True, 2, "1f1b", True), (True, 3, "1f1b", False),
], ids=["gpipe", "gpipe-moe-aux", "1f1b-3rank-no-recompute", "1f1b-recompute", "1f1b-moe-aux-recompute",
        "1f1b-3rank-moe-aux-no-recompute"])
def test_rank_pipeline_matches_autograd(moe, world, schedule, recompute):
    M, n_layers = 4, 5
    ids, labels = _data(M)
    ref_loss, ref_grads = _reference(n_layers, moe, ids, labels)
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_rank_main, args=(world, _free_port(), d, moe, M, n_layers, schedule, recompute),
                           nprocs=world, start_method="spawn", join=True)
        outs = [torch.load(os.path.join(d, f"rank{r}.pt")) for r in range(world)]
    assert all(o["loss"] is None for o in outs[:-1])
    assert abs(outs[-1]["loss"] - ref_loss) < 1e-5
    got = {}
    for o in outs:
        got.update(o["grads"])
    assert set(got) == set(ref_grads)
    for k, g in ref_grads.items():
        torch.testing.assert_close(got[k], g, rtol=1e-4, atol=1e-6, msg=k)


def test_stratum_pipeline_keeps_the_reference_hooks():
    """The reference's recorder / timer setters and the bookkeeping names its tests inspect."""
    layers = _model(4, False)
    stages = [DeviceStage(layers[:2], "cpu"), DeviceStage(layers[2:], "cpu")]
    pipe = StratumPipeline(ToyPrefix(), stages, ToyPostfix())

    class Rec:
        def span(self, name, **kw):
            import contextlib

            return contextlib.nullcontext()

    rec = Rec()
    pipe.set_timing_recorder(rec)
    assert stages[1].timing_recorder is rec and stages[1].layer_start == 2
    pipe.set_layer_timer(None, adapt_every_n=0)
    # one recompute group per layer by default: each group's module holds that layer
    assert [[id(x) for x in m] for m in pipe._fwd_group_modules] == [[id(l)] for l in layers]
    pipe._pending_bwd_fences[99] = object()
    ids, labels = _data(1)
    pipe(ids, labels=labels).backward()
    assert 99 not in pipe._pending_bwd_fences
    assert pipe._param_upload_stream(0) is None


def test_rank_pipeline_cuda_graph_is_refused_where_it_cannot_apply():
    """CUDA-graph microbatches need one rank and no router aux loss (host-side checks only)."""
    sink = RouterLogitsSink()
    layers = _model(2, True, sink)
    stage = DeviceStage(layers, "cpu")
    with pytest.raises(ValueError, match="single rank"):
        RankPipeline(stage, prefix=ToyPrefix(), postfix=None, rank=0, world=2, hidden_size=H,
                     hidden_dtype=torch.float32, schedule="1f1b", recompute=False, cuda_graph=True)
    with pytest.raises(ValueError, match="aux loss"):
        RankPipeline(stage, prefix=ToyPrefix(), postfix=ToyPostfix(), rank=0, world=1, hidden_size=H,
                     hidden_dtype=torch.float32, router_sink=sink, router_aux_coef=COEF, n_experts=E,
                     schedule="1f1b", recompute=False, cuda_graph=True)


def test_cuda_graph_address_signature_tracks_storage_not_values():
    """What a captured graph has baked in: in-place updates keep the signature,
    replaced storage (a new ``param.data``, a re-uploaded NF4 payload) changes it."""
    from stratum_b200.pipeline import _address_signature

    layers = _model(2, False, None)
    model = nn.ModuleList(layers)
    sig = _address_signature(model)
    assert sig == _address_signature(model)
    p = next(q for q in model.parameters() if q.requires_grad)
    with torch.no_grad():
        p.mul_(1.5)  # an optimizer step: same storage
    assert _address_signature(model) == sig
    p.data = p.data.clone()  # new storage
    assert _address_signature(model) != sig
    sig = _address_signature(model)
    p.requires_grad_(False)  # a frozen adapter: the captured backward's gradient set changed
    assert _address_signature(model) != sig
    p.requires_grad_(True)
    assert _address_signature(model) == sig

    holder = nn.Module()  # uploaded NF4Experts-style weights are covered too

    class _QS:
        def __init__(self):
            self.absmax, self.code, self.offset, self.state2 = torch.ones(4), torch.ones(16), None, None

    holder.gate_up, holder.gate_up_state = torch.zeros(8, dtype=torch.uint8), _QS()
    holder.down, holder.down_state = None, None
    s1 = _address_signature(holder)
    holder.gate_up = torch.zeros(8, dtype=torch.uint8)
    assert _address_signature(holder) != s1


def _channel_main(rank, world, port, out_dir):
    import torch.distributed as dist

    from stratum_b200.boundary import P2PChannel

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ch = P2PChannel(rank, world)
        got = []
        if rank == 0:
            for i in range(3):  # send-only groups: not waited on, kept alive until they complete
                ch.send_forward([torch.full((5,), float(i))])
            in_flight = ch.sends_in_flight
            g = ch.recv_backward([((5,), torch.float32, "cpu")])[0]  # a receiving group is waited on
            got.append(g)
            ch.flush()
            torch.save({"in_flight": in_flight, "after_flush": ch.sends_in_flight, "got": got},
                       os.path.join(out_dir, "rank0.pt"))
        else:
            for _ in range(3):
                got.append(ch.recv_forward([((5,), torch.float32, "cpu")])[0])
            ch.send_backward([torch.full((5,), 7.0)])
            ch.flush()
            torch.save({"got": got, "after_flush": ch.sends_in_flight}, os.path.join(out_dir, "rank1.pt"))
    finally:
        dist.destroy_process_group()


def test_p2p_channel_send_only_groups_do_not_block_and_flush_retires_them():
    """Send-only boundary groups return without waiting (the sender's stream runs on),
    arrive in order, and ``flush`` retires every send still held."""
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_channel_main, args=(2, _free_port(), d), nprocs=2, start_method="spawn", join=True)
        r0 = torch.load(os.path.join(d, "rank0.pt"))
        r1 = torch.load(os.path.join(d, "rank1.pt"))
    assert 0 <= r0["in_flight"] <= 3
    assert r0["after_flush"] == 0 and r1["after_flush"] == 0
    assert [float(t[0]) for t in r1["got"]] == [0.0, 1.0, 2.0]
    assert torch.equal(r0["got"][0], torch.full((5,), 7.0))


def _retry_main(rank, world, port, out_dir, fail_rank, fail_times, retries):
    """RankPipeline.train_step with the status check of ``fail_rank`` raising, on the host,
    for its first ``fail_times`` calls (no GPU: the failure is injected, nothing faults)."""
    import torch.distributed as dist

    from stratum_b200 import _lib
    from stratum_b200 import pipeline as P

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from stratum_b200.assign import assign_layers_to_devices, strata

        calls = {"n": 0}

        def fake_check(devices, what):
            calls["n"] += 1
            if rank == fail_rank and calls["n"] <= fail_times:
                raise _lib.StratumError(f"{what}: injected device-side wait timeout")

        P._check_status = fake_check
        M, n_layers = 3, 4
        layers = _model(n_layers, False)
        parts = strata(assign_layers_to_devices(n_layers, n_devices=world))
        mine = parts[rank][1]
        stage = DeviceStage([layers[i] for i in mine], "cpu")
        pipe = RankPipeline(stage, prefix=ToyPrefix(), postfix=ToyPostfix() if rank == world - 1 else None,
                            rank=rank, world=world, hidden_size=H, hidden_dtype=torch.float32,
                            schedule="1f1b", recompute=False, step_retries=retries)
        ids, labels = _data(M)
        # gradients already present before the step must survive a retried step unchanged
        for i in mine:
            for p in layers[i].parameters():
                if p.requires_grad:
                    p.grad = torch.full_like(p, 0.5)
        result = {}
        try:
            loss = pipe.train_step(ids if rank == 0 else None, labels if rank == world - 1 else None,
                                   microbatches=M, seq_len=S)
            result["loss"] = None if loss is None else float(loss)
        except _lib.StratumError as exc:
            result["error"] = str(exc)
        result["retries"] = pipe.status_retries
        result["grads"] = {f"{i}.{n}": p.grad for i in mine for n, p in layers[i].named_parameters()
                           if p.requires_grad}
        torch.save(result, os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


def _run_retry(fail_rank, fail_times, retries):
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_retry_main, args=(world, _free_port(), d, fail_rank, fail_times, retries),
                           nprocs=world, start_method="spawn", join=True)
        return [torch.load(os.path.join(d, f"rank{r}.pt")) for r in range(world)]


def test_rank_pipeline_retries_a_step_whose_kernels_gave_up():
    """A status error on one rank makes every rank run the step again, from the gradients
    held before it: the result equals a clean step's."""
    clean = _run_retry(fail_rank=-1, fail_times=0, retries=1)
    retried = _run_retry(fail_rank=1, fail_times=1, retries=1)
    assert [o["retries"] for o in clean] == [0, 0]
    assert [o["retries"] for o in retried] == [1, 1]
    assert retried[-1]["loss"] == pytest.approx(clean[-1]["loss"], rel=1e-6)
    for a, b in zip(clean, retried):
        for k in a["grads"]:
            torch.testing.assert_close(b["grads"][k], a["grads"][k], rtol=0, atol=0, msg=k)


def test_rank_pipeline_raises_once_retries_are_spent():
    outs = _run_retry(fail_rank=0, fail_times=5, retries=1)
    assert "injected" in outs[0]["error"]
    assert "another rank" in outs[1]["error"]
    assert [o["retries"] for o in outs] == [1, 1]
