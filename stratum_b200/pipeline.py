"""Layer-parallel pipeline over the NF4 decoder layers.

Two drivers over the same pieces:

* :class:`StratumPipeline` -- the reference's class (stratum/pipeline.py:81-1115):
  one process drives every GPU; ``forward(input_ids, attention_mask, labels)``
  returns the loss and the caller runs ``loss.backward()``.  Stage boundaries
  are direct NVLink copies (``boundary.transfer``) instead of host staging.
* :class:`RankPipeline` -- one process per GPU (``torch.distributed``, NCCL):
  each rank holds one stratum of layers (``assign.strata``); ``train_step``
  runs a GPipe schedule over microbatches, boundary activations and gradients
  move by NCCL send/recv (``boundary.P2PChannel``).  This is how the path
  scales over the GPUs of one box.

Both keep the reference's memory model (stratum/runtime.py:195-290,
``anchor_explicit_group_backward``): a group of layers runs forward without an
autograd graph and saves only its input; its backward recomputes the group and
backpropagates through it.  Groups are single layers here.  With streamed NF4
weights (fused-mode ``NF4Linear`` fed by ``upload.ensure_weights``), layer i+1
uploads on a side stream while layer i computes (stratum/stage.py:51-137);
``StratumPipeline`` frees a layer after its forward and uploads it again for
its backward (as the reference does), ``RankPipeline`` uploads its stratum once
per step, overlapped with the first microbatch, and frees it at the end.

MoE layers: the router aux loss (HF ``load_balancing_loss_func``, the
reference's stratum/moe.py:162-223) is a function of per-expert counts and
summed router probabilities over every layer; the forward accumulates those
sums (all-reduced across ranks), and each layer's recompute adds the aux
term's gradient to its backward.
"""

from __future__ import annotations

from contextlib import nullcontext
from dataclasses import dataclass, field
from typing import Any, Optional

import torch
import torch.distributed as dist
import torch.nn as nn

from .boundary import P2PChannel, transfer
from .nf4_linear import NF4Linear
from .runtime import anchor_explicit_group_backward
from .scheduler import ModelExecutePlan
from .stage import DeviceStage
from .upload import (ensure_prefetched_weights, ensure_weights, free_weights, prefetch_weights, restore_module_buffers,
                     snapshot_module_buffers)


def _dev(d) -> torch.device:
    """A stage's device: ``torch.device`` / string as given; an integer id names a
    CUDA device (or the CPU on a machine without one, as the reference's tests run)."""
    if isinstance(d, torch.device):
        return d
    if isinstance(d, str):
        return torch.device(d)
    return torch.device("cuda", int(d)) if torch.cuda.is_available() else torch.device("cpu")


def _on(device: torch.device):
    """``torch.cuda.device`` for a CUDA device, nothing for the CPU (gloo tests)."""
    return torch.cuda.device(device) if device.type == "cuda" else nullcontext()


def _move_tree(value: Any, device: torch.device) -> Any:
    if torch.is_tensor(value):
        return value.to(device, non_blocking=True)
    if isinstance(value, tuple):
        return tuple(_move_tree(v, device) for v in value)
    if isinstance(value, list):
        return [_move_tree(v, device) for v in value]
    if isinstance(value, dict):
        return {k: _move_tree(v, device) for k, v in value.items()}
    return value


def _device_tensors(module: nn.Module) -> list[torch.Tensor]:
    out = []
    for m in module.modules():
        if isinstance(m, NF4Linear) and m.quantized is not None:
            out.append(m.quantized)
            qs = m.quant_state
            for t in (qs.absmax, qs.code, qs.offset):
                if torch.is_tensor(t):
                    out.append(t)
            if qs.state2 is not None:
                out += [t for t in (qs.state2.absmax, qs.state2.code) if torch.is_tensor(t)]
    return out


def _address_signature(module: nn.Module) -> tuple:
    """Data addresses of everything the module's forward reads from device memory:
    parameters, buffers, NF4Linear payloads and uploaded NF4Experts weights -- the
    addresses a captured CUDA graph has baked in -- plus which parameters are
    trainable (a captured backward writes the gradients of the set it was captured
    with, so freezing or unfreezing a parameter needs a new graph)."""
    params = list(module.parameters())
    ptrs = [t.data_ptr() for t in params] + [t.data_ptr() for t in module.buffers()]
    ptrs += [bool(p.requires_grad) for p in params]
    ptrs += [t.data_ptr() for t in _device_tensors(module)]
    for m in module.modules():
        for w, qs in ((getattr(m, "gate_up", None), getattr(m, "gate_up_state", None)),
                      (getattr(m, "down", None), getattr(m, "down_state", None))):
            if qs is None or not torch.is_tensor(w):
                continue
            ptrs.append(w.data_ptr())
            ptrs += [t.data_ptr() for t in (qs.absmax, qs.code, qs.offset) if torch.is_tensor(t)]
            if qs.state2 is not None:
                ptrs += [t.data_ptr() for t in (qs.state2.absmax, qs.state2.code) if torch.is_tensor(t)]
    return tuple(ptrs)


def _check_status(devices, what: str) -> None:
    """Raise if a GEMM kernel on any of ``devices`` gave up a bounded wait since the last
    check.  Reading the status word clears it, so a caller that catches the error can
    retry.  One host synchronisation per device; skipped for CPU devices (gloo tests)
    and while a stream captures a CUDA graph."""
    devs = {d for d in devices if d.type == "cuda"}
    if not devs or torch.cuda.is_current_stream_capturing():
        return
    from . import _lib

    for d in sorted(devs, key=lambda x: x.index or 0):
        _lib.check_device_status(what, d)


def _needs_streaming(module: nn.Module, device: torch.device) -> bool:
    return any(isinstance(m, NF4Linear) and m.streamed and not m.device_state_on(device) for m in module.modules())


# --------------------------------------------------------------------------------
# weight streaming
# --------------------------------------------------------------------------------

class _Streamer:
    """Per-layer NF4 upload on a side stream with event fences.

    ``acquire(i)`` makes the compute stream wait for layer i's upload (issuing it
    if nobody did); ``prefetch(i)`` issues it early; ``release(i)`` drops the
    device copy once the compute stream is done with it (the blocks are marked
    as used by that stream, so the allocator does not hand them to the next
    upload early)."""

    def __init__(self, layers: list[nn.Module], device: torch.device, enabled: bool):
        self.layers, self.device = layers, device
        self.enabled = bool(enabled) and device.type == "cuda"
        self.stream = torch.cuda.Stream(device) if self.enabled else None
        self.pending: dict[int, torch.cuda.Event] = {}
        self.resident: set[int] = set()

    def prefetch(self, i: int) -> None:
        if not self.enabled or not (0 <= i < len(self.layers)) or i in self.pending or i in self.resident:
            return
        with torch.cuda.device(self.device), torch.cuda.stream(self.stream):
            ensure_weights(self.layers[i], self.device)
            ev = torch.cuda.Event()
            ev.record(self.stream)
        self.pending[i] = ev

    def acquire(self, i: int) -> None:
        if not self.enabled or i in self.resident:
            return
        self.prefetch(i)
        torch.cuda.current_stream(self.device).wait_event(self.pending.pop(i))
        self.resident.add(i)

    def release(self, i: int) -> None:
        if not self.enabled or i not in self.resident:
            return
        cur = torch.cuda.current_stream(self.device)
        for t in _device_tensors(self.layers[i]):
            t.record_stream(cur)
        free_weights(self.layers[i])
        self.resident.discard(i)

    def release_all(self) -> None:
        for i in list(self.resident):
            self.release(i)
        self.pending.clear()


# --------------------------------------------------------------------------------
# router aux loss bookkeeping
# --------------------------------------------------------------------------------

@dataclass
class _AuxState:
    """Per-expert sums of one microbatch's router outputs over the layers seen so
    far; ``finalize`` turns global sums into the aux term's gradient weights."""

    n_experts: int
    coef: float
    counts: Optional[torch.Tensor] = None
    psum: Optional[torch.Tensor] = None
    rows: float = 0.0
    weight: Optional[torch.Tensor] = None
    value: Optional[torch.Tensor] = None
    extra: list = field(default_factory=list)

    def add(self, probs: torch.Tensor, indices: torch.Tensor) -> None:
        from .decoder import load_balancing_terms

        c, p = load_balancing_terms(probs.detach(), indices, self.n_experts)
        self.counts = c if self.counts is None else self.counts + c
        self.psum = p if self.psum is None else self.psum + p
        self.rows += float(probs.shape[0])

    def finalize(self, counts: torch.Tensor, psum: torch.Tensor, rows, grad_scale: float = 1.0) -> None:
        # loss = E / N^2 * sum_e count_e * psum_e, psum_e = sum over rows of softmax(router output)_e,
        # so d loss / d softmax(router output)[row, e] = E / N^2 * count_e (times the weight of this
        # microbatch's loss in the step's loss)
        n2 = torch.as_tensor(rows, dtype=torch.float32, device=counts.device).clamp_min(1.0) ** 2
        self.value = self.coef * self.n_experts * (counts * psum).sum() / n2
        self.weight = (self.coef * self.n_experts * grad_scale) * counts / n2


class _Runner:
    """Runs layers [i0, i1) of a stage on the pipeline tuple: forward without an
    autograd graph, and again with one for the backward (the recompute anchor of
    ``runtime.anchor_explicit_group_backward``), with per-layer weight streaming,
    the group's buffer snapshot and the router taps of MoE layers."""

    def __init__(self, stage, i0: int, i1: int, streamer: _Streamer, policy: str, sink=None,
                 aux: Optional[_AuxState] = None, group_module: Optional[nn.Module] = None,
                 buffers: Optional[dict] = None, reload=None, unload=None):
        self.stage, self.layers = stage, list(stage.layers)
        self.i0, self.i1 = i0, i1
        self.streamer, self.policy, self.sink, self.aux = streamer, policy, sink, aux
        self.group_module, self.buffers = group_module, buffers
        # groups made resident as a whole (not streamed): weights again for the
        # recomputation, dropped after the group's backward
        self.reload, self.unload = reload, unload
        self.extra: list = []

    def _run(self, tup: tuple, collect_grad_probs: Optional[list]) -> tuple:
        if self.sink is None:  # the stage's own range runner (timing spans), or the whole stage module
            if hasattr(self.stage, "forward_range"):
                return self.stage.forward_range(tup, local_start=self.i0, local_stop=self.i1)
            if self.i0 == 0 and self.i1 == len(self.layers):
                return self.stage(tup)
        t = tup
        for i in range(self.i0, self.i1):
            if self.sink is not None:
                self.sink.clear()
                self.sink.active = True
            try:
                t = self.layers[i](t)
            finally:
                if self.sink is not None:
                    self.sink.active = False
            if self.sink is not None:
                for probs, idx in zip(self.sink.probs, self.sink.indices):
                    if collect_grad_probs is None:
                        self.aux.add(probs, idx)
                    else:
                        collect_grad_probs.append(probs)
                self.sink.clear()
        return t

    def forward(self, tup: tuple) -> tuple:
        s = self.streamer
        for i in range(self.i0, self.i1):
            s.acquire(i)
        s.prefetch(self.i1)
        with torch.no_grad():
            out = self._run(tup, None)
        if self.policy == "group":  # reference behaviour: free after forward, upload again for backward
            last = len(self.layers) - 1
            for i in range(self.i0, self.i1):
                if i != last:
                    s.release(i)
        return out

    def recompute(self, tup: tuple) -> tuple:
        """The group again with autograd on (called by the anchor's backward); the
        router aux loss's gradient term, if any, is left in ``self.extra``."""
        s = self.streamer
        for i in range(self.i0, self.i1):
            s.acquire(i)
        s.prefetch(self.i0 - 1)
        if self.reload is not None:
            self.reload()
        if self.buffers is not None and self.group_module is not None:
            # the recomputation starts from the buffers the forward saw
            restore_module_buffers(self.group_module, self.buffers)
        probs: Optional[list] = [] if self.sink is not None else None
        out = self._run(tup, probs)
        self.extra = []
        if probs and self.aux is not None and self.aux.weight is not None:
            term = sum((torch.softmax(p.float(), dim=-1) * self.aux.weight.to(p.device)).sum() for p in probs)
            if term.requires_grad:  # else the term reaches no trainable parameter
                self.extra.append(term)
        return out

    def extra_terms(self) -> list:
        out, self.extra = self.extra, []
        return out

    def after_backward(self) -> None:
        if self.policy == "group":
            for i in range(self.i0, self.i1):
                self.streamer.release(i)
        if self.unload is not None:
            self.unload()


def _anchor_group(runner: _Runner, tup: tuple, offload: bool, look_ahead=None) -> tuple:
    """Forward of one layer group without a graph, anchored so its backward recomputes it."""
    out = runner.forward(tup)
    return anchor_explicit_group_backward(run_group=runner.recompute, group_input=tup, group_output=out,
                                          offload_input_to_cpu=offload, look_ahead_upload=look_ahead,
                                          on_backward_complete=runner.after_backward,
                                          extra_terms=runner.extra_terms)


def _trainable(modules: list[nn.Module]) -> list[torch.Tensor]:
    return [p for m in modules for p in m.parameters() if p.requires_grad]


def _stage_layers(stage) -> list[nn.Module]:
    return list(stage.layers)


def _run_stage(stage, hidden: torch.Tensor, rest: tuple, streamer: _Streamer, policy: str, sink, aux,
               offload: bool) -> torch.Tensor:
    """Every layer of ``stage`` as its own recompute group (the per-rank pipeline)."""
    tup = (hidden,) + tuple(rest)
    for i in range(len(stage.layers)):
        runner = _Runner(stage, i, i + 1, streamer, policy, sink, aux)
        tup = _anchor_group(runner, tup, offload)
    return tup[0]


# --------------------------------------------------------------------------------
# one process, several GPUs (the reference's class)
# --------------------------------------------------------------------------------

def _move_tensor_tree(value: Any, device) -> Any:
    """Tensors of a nested tuple / list / dict moved to ``device`` (other leaves kept):
    the non-hidden parts of the pipeline tuple crossing a stage boundary."""
    return _move_tree(value, device)


class StratumPipeline(nn.Module):
    """A multi-GPU pipeline of DeviceStages driven by one process.

    Same constructor and calls as the reference (stratum/pipeline.py:90-99,
    646-1071).  ``prefix`` runs on the first stage's device, each stage on its own
    device, ``postfix`` on the last stage's device; boundaries are NVLink device
    copies.  Layers run in recompute groups: ``execute_plan`` (a
    ``scheduler.ModelExecutePlan``; groups may not cross stages) or, by default,
    one group per layer.  Each group's forward runs without a graph after its
    buffers are snapshotted; its weights are freed right after (the reference's
    memory model) and its backward recomputes it (``runtime``), starting the
    previous group's upload first (the look-ahead).

    Weights: a stage of fused-mode NF4Linear layers streams them per layer on a
    side stream (``_param_upload_stream``).  Otherwise each group's module is
    made resident with ``ensure_weights`` -- with ``prefetch_nf4``, through
    ``prefetch_weights`` / ``ensure_prefetched_weights``, the next group's (or the
    postfix's) copies started before the current group runs -- as the reference
    does on its group-level path; the prefix and postfix always are.
    ``offload_stage_inputs`` keeps each group's saved input in host memory.  For
    MoE models pass the ``router_sink`` the layers were built with and the
    aux-loss coefficient.
    """

    def __init__(self, prefix: nn.Module, stages: list, postfix: nn.Module, *, prefetch_nf4: bool = False,
                 offload_stage_inputs: bool = False, execute_plan: Any = None, router_sink=None,
                 router_aux_coef: float = 0.0, n_experts: int = 0):
        super().__init__()
        self.prefix = prefix
        self.stages = nn.ModuleList(stages)
        self.postfix = postfix
        self.prefetch_nf4 = prefetch_nf4
        self.offload_stage_inputs = offload_stage_inputs
        self.router_sink = router_sink
        self.router_aux_coef = float(router_aux_coef)
        self.n_experts = int(n_experts)
        self._stage_ranges = []
        start = 0
        for st in stages:
            self._stage_ranges.append(range(start, start + len(st.layers)))
            start += len(st.layers)
        total = start
        plan = execute_plan if execute_plan is not None else ModelExecutePlan.per_layer(total)
        plan.check_valid(total, "train")
        if {(r.start, r.stop) for r in plan.fwd_plan} != {(r.start, r.stop) for r in plan.bwd_plan}:
            raise ValueError("StratumPipeline: backward groups must be the forward groups (each forward group "
                             "is recomputed as one backward group)")
        self.execute_plan = plan
        # (stage index, first layer in the stage, end layer in the stage, global layer range) per group
        self._groups: list[tuple[int, int, int, range]] = []
        for r in plan.fwd_plan:
            owner = next((si for si, sr in enumerate(self._stage_ranges) if sr.start <= r.start and r.stop <= sr.stop),
                         None)
            if owner is None:
                raise ValueError(f"StratumPipeline: layer group {r.start}:{r.stop} must lie inside one stage")
            sr = self._stage_ranges[owner]
            self._groups.append((owner, r.start - sr.start, r.stop - sr.start, r))
        # the module that holds each group's layers (the stage itself when the group is the whole stage)
        self._fwd_group_modules: list[nn.Module] = [
            stages[si] if (a == 0 and b == len(stages[si].layers)) else nn.ModuleList(list(stages[si].layers)[a:b])
            for si, a, b, _ in self._groups]
        self._streamers = [
            _Streamer(_stage_layers(s), _dev(s.device_id), any(_needs_streaming(l, _dev(s.device_id))
                                                               for l in s.layers))
            for s in stages]
        self.last_aux: Optional[torch.Tensor] = None
        self.timing_recorder = None
        self._layer_timer = None
        self._plan_adapt_after_n = 0
        # backward look-ahead fences of the current step, by group (streamed groups carry their
        # upload events in their streamer, so this stays empty on that path)
        self._pending_bwd_fences: dict = {}

    @property
    def n_devices(self) -> int:
        return len({str(_dev(s.device_id)) for s in self.stages})

    # ---------------------------------------------------------- weights

    def _param_upload_stream(self, device_id) -> Optional["torch.cuda.Stream"]:
        """The side stream streamed layers of ``device_id`` upload on (None when the
        stage's weights are made resident group by group instead)."""
        for stage, st in zip(self.stages, self._streamers):
            if _dev(stage.device_id) == _dev(device_id) and st.enabled:
                return st.stream
        return None

    def _prefetch_module(self, module: nn.Module, device_id):
        if not self.prefetch_nf4:
            return None
        return prefetch_weights(module, device_id)

    def _ensure_module(self, module: nn.Module, device_id, prefetch=None) -> int:
        if self.prefetch_nf4:
            return ensure_prefetched_weights(module, device_id, prefetch)
        return ensure_weights(module, device_id)

    def _start_bwd_look_ahead(self, gid: int) -> None:
        """Backward of group ``gid + 1`` is starting: make group ``gid`` resident early
        (streamed stages: its first layer's upload on the side stream)."""
        si, a, _, _ = self._groups[gid]
        st = self._streamers[si]
        if st.enabled:
            with _on(st.device):
                st.prefetch(a)

    # ---------------------------------------------------------- forward

    def forward(self, input_ids: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
                labels: Optional[torch.Tensor] = None, **kwargs):
        """Run forward through all stages; returns the postfix's output (the loss when
        labels are given)."""
        self._pending_bwd_fences = {}
        # the previous step's backward ran after the last check: report a kernel that gave up
        _check_status([_dev(s.device_id) for s in self.stages], "StratumPipeline.forward")
        if self._layer_timer is not None and hasattr(self._layer_timer, "update_times"):
            self._layer_timer.update_times()
        dev0 = _dev(self.stages[0].device_id) if len(self.stages) else _dev(0)
        last = _dev(self.stages[-1].device_id) if len(self.stages) else dev0
        if input_ids.device != dev0:
            input_ids = input_ids.to(dev0, non_blocking=True)
        if labels is not None and labels.device != dev0:
            labels = labels.to(dev0, non_blocking=True)
        if attention_mask is not None and attention_mask.device != dev0:
            attention_mask = attention_mask.to(dev0, non_blocking=True)
        n = len(self._groups)
        grouped = [self._param_upload_stream(self.stages[si].device_id) is None for si, *_ in self._groups]
        with _on(dev0):
            self._ensure_module(self.prefix, dev0)
            pending = self._prefetch_module(self._fwd_group_modules[0], dev0) if n and grouped[0] else None
            tup = self.prefix(input_ids=input_ids, attention_mask=attention_mask, labels=labels, **kwargs)
        if not isinstance(tup, tuple):
            raise TypeError(f"StratumPipeline: the prefix must return the pipeline tuple, got {type(tup).__name__}")
        aux = _AuxState(self.n_experts, self.router_aux_coef) if (self.router_sink is not None and
                                                                  self.router_aux_coef) else None
        sink = self.router_sink if aux is not None else None
        pending_postfix = None
        for gid, (si, a, b, _) in enumerate(self._groups):
            stage = self.stages[si]
            dev = _dev(stage.device_id)
            if tup[0].device != dev:  # stage boundary: NVLink copy of the hidden state
                tup = (transfer(tup[0], dev),) + tuple(_move_tree(tuple(tup[1:]), dev))
            module = self._fwd_group_modules[gid]
            with _on(dev):
                if grouped[gid]:
                    self._ensure_module(module, dev, pending)
                    pending = None
                # start the next group's (or the postfix's) copies before this group runs
                if gid + 1 < n:
                    if grouped[gid + 1]:
                        pending = self._prefetch_module(self._fwd_group_modules[gid + 1],
                                                        _dev(self.stages[self._groups[gid + 1][0]].device_id))
                else:
                    pending_postfix = self._prefetch_module(self.postfix, last)
                snapshot = snapshot_module_buffers(module)
                runner = _Runner(stage, a, b, self._streamers[si], "group", sink, aux, group_module=module,
                                 buffers=snapshot,
                                 reload=(lambda m=module, d=dev: self._ensure_module(m, d)) if grouped[gid] else None,
                                 unload=(lambda m=module: free_weights(m)) if grouped[gid] else None)
                out = runner.forward(tup)
                if grouped[gid]:
                    free_weights(module)  # at most one group's weights resident at a time
                look = None if gid == 0 else (lambda g=gid - 1: self._start_bwd_look_ahead(g))
                tup = anchor_explicit_group_backward(run_group=runner.recompute, group_input=tup,
                                                     group_output=out,
                                                     offload_input_to_cpu=self.offload_stage_inputs,
                                                     look_ahead_upload=look,
                                                     on_backward_complete=runner.after_backward,
                                                     extra_terms=runner.extra_terms)
        if tup[0].device != last:
            tup = (transfer(tup[0], last),) + tuple(_move_tree(tuple(tup[1:]), last))
        with _on(last):
            self._ensure_module(self.postfix, last, pending_postfix)
            loss = self.postfix(tup)
        if aux is not None and aux.counts is not None:
            aux.finalize(aux.counts, aux.psum, aux.rows)
            self.last_aux = aux.value.detach()
            if loss is not None:
                loss = loss + aux.value.detach().to(loss.device)
        return loss

    def set_timing_recorder(self, recorder) -> None:
        """Attach a timing recorder to every stage's layer spans (stratum/pipeline.py:231-245)."""
        self.timing_recorder = recorder
        start = 0
        for stage in self.stages:
            stage.set_timing_recorder(recorder, layer_start=start)
            start += len(stage.layers)

    def set_layer_timer(self, timer, *, adapt_every_n: int = 0) -> None:
        """Attach a per-layer timer (stratum/pipeline.py:247-268).  Plans are not
        adapted from its timings here (the reference's timing-driven plan search is
        not part of this build), so ``adapt_every_n`` is kept for the call's shape."""
        self._layer_timer = timer
        self._plan_adapt_after_n = adapt_every_n

    def free_all_weights(self) -> None:
        """Drop every streamed layer's device copy (reference: call after backward)."""
        for s in self._streamers:
            s.release_all()
        for stage in self.stages:
            free_weights(stage)
        _check_status([_dev(s.device_id) for s in self.stages], "StratumPipeline.free_all_weights")

    def forward_batch(self, batch: Any, *, ignore_index: int = -100):
        """Forward on a dict-like batch with ``input_ids`` / ``attention_mask`` / ``labels``."""
        get = (lambda k: batch[k]) if isinstance(batch, dict) else (lambda k: getattr(batch, k))
        return self(get("input_ids"), attention_mask=get("attention_mask"), labels=get("labels"))


# --------------------------------------------------------------------------------
# one process per GPU
# --------------------------------------------------------------------------------

class RankPipeline(nn.Module):
    """This rank's stratum of a layer-parallel pipeline (one process per GPU).

    Every rank holds a ``prefix`` for its rotary context (rank 0's also embeds
    tokens); the last rank holds the ``postfix``.  ``train_step`` runs forward
    and backward over ``microbatches`` sequences.  Input ids are read on rank 0,
    labels on the last rank.  Returns the mean loss on the last rank, ``None``
    elsewhere.

    Schedules: ``"gpipe"`` -- all forwards (each rank sends its stratum's output
    on as soon as it is computed), then all backwards in reverse order;
    ``"1f1b"`` -- after ``world - rank - 1`` warm-up forwards each rank
    alternates one forward and one backward, so at most ``world - rank``
    microbatches are in flight on it.  ``recompute=False`` keeps every layer's
    autograd graph instead of recomputing it in the backward (the 1F1B bound on
    microbatches in flight is what makes that fit).  The router aux loss needs
    each microbatch's global per-expert sums before its backward: GPipe
    all-reduces them after the forwards; 1F1B carries them on the boundary
    messages (partial sums forward, global sums back).

    ``cuda_graph=True`` (one rank, weights resident on the device, no router aux
    loss): one microbatch's forward and backward are captured once into a CUDA
    graph -- together with adding its LoRA gradients and loss into static
    accumulators -- and every microbatch is a replay of it, so a model whose
    kernels are small no longer waits on the host's per-op dispatch.  The graph
    is built once per (microbatch count, sequence length); gradients are added
    into the parameters' ``.grad`` as the eager path does.  Replays read the
    parameters and NF4 weights at the addresses they had when the graph was
    captured; each step compares those addresses with the current ones and
    captures again if any moved (a replaced ``param.data``, a re-upload), so
    in-place updates (as torch optimizers make) keep the graph.
    ``graph_launches`` counts the library kernels the replays ran (they bypass
    the host-side launch counter).

    ``step_retries`` (default 2): a step whose kernels report that a bounded
    device-side wait gave up (the status word read at the end of every step) has
    invalid gradients; every rank learns of it through one all-reduce of a flag,
    the trainable parameters' ``.grad`` are put back as they were before the step,
    and the step runs again, at most ``step_retries`` times before
    ``StratumError`` is raised.  ``status_retries`` counts the retried steps.
    """

    def __init__(self, stage: DeviceStage, *, prefix: nn.Module, postfix: Optional[nn.Module], rank: int,
                 world: int, group=None, hidden_size: int, offload_stage_inputs: bool = False, router_sink=None,
                 router_aux_coef: float = 0.0, n_experts: int = 0, hidden_dtype=torch.bfloat16,
                 schedule: str = "gpipe", recompute: bool = True, cuda_graph: bool = False,
                 step_retries: int = 2):
        super().__init__()
        if (postfix is None) != (rank + 1 < world):
            raise ValueError("RankPipeline: the postfix lives on the last rank only")
        if schedule not in ("gpipe", "1f1b"):
            raise ValueError(f"RankPipeline: unknown schedule {schedule!r}")
        if not recompute and schedule != "1f1b":
            raise ValueError("RankPipeline: recompute=False needs the 1f1b schedule (bounded microbatches in flight)")
        self.schedule, self.recompute = schedule, recompute
        self.stage, self.prefix, self.postfix = stage, prefix, postfix
        self.rank, self.world, self.group = rank, world, group
        if world > 1 and torch.cuda.is_available():
            from . import ops

            ops.multirank_gemm_default()  # one-SM GEMM kernels beside NCCL traffic
        self.device = _dev(stage.device_id)
        self.hidden_size, self.hidden_dtype = hidden_size, hidden_dtype
        self.offload = offload_stage_inputs
        self.router_sink = router_sink
        self.router_aux_coef = float(router_aux_coef)
        self.n_experts = int(n_experts)
        self.chan = P2PChannel(rank, world, group)
        self.streamer = _Streamer(_stage_layers(stage), self.device,
                                  any(_needs_streaming(l, self.device) for l in stage.layers))
        self.last_aux: Optional[torch.Tensor] = None
        self.cuda_graph = bool(cuda_graph)
        if self.cuda_graph:
            if world != 1:
                raise ValueError("RankPipeline: cuda_graph needs a single rank (boundaries are NCCL calls)")
            if self.streamer.enabled:
                raise ValueError("RankPipeline: cuda_graph needs the stratum's weights resident on the device")
            if router_sink is not None and self.router_aux_coef != 0.0 and self.n_experts > 0:
                raise ValueError("RankPipeline: cuda_graph does not cover the router aux loss")
        self._graphs: dict = {}
        self.graph_launches = 0
        self.step_retries = max(0, int(step_retries))
        self.status_retries = 0

    def _aux_reduce(self, states: list[_AuxState]) -> None:
        E = self.n_experts
        M = len(states)
        buf = torch.zeros(M, 2 * E + 1, dtype=torch.float32, device=self.device)
        for m, a in enumerate(states):
            if a.counts is not None:
                buf[m, :E] = a.counts
                buf[m, E:2 * E] = a.psum
                buf[m, 2 * E] = a.rows
        if self.world > 1 and dist.is_initialized():
            dist.all_reduce(buf, group=self.group)
        for m, a in enumerate(states):  # the step's loss is the mean over its M microbatches
            a.finalize(buf[m, :E], buf[m, E:2 * E], buf[m, 2 * E], grad_scale=1.0 / M)

    def _stats(self, aux: Optional[_AuxState]) -> torch.Tensor:
        """This rank's router sums of one microbatch as [counts | psum | rows] (zeros if none)."""
        E = self.n_experts
        buf = torch.zeros(2 * E + 1, dtype=torch.float32, device=self.device)
        if aux is not None and aux.counts is not None:
            buf[:E] = aux.counts
            buf[E:2 * E] = aux.psum
            buf[2 * E] = aux.rows
        return buf

    def _forward_mb(self, m: int, ids, labs, shape, x_recv: Optional[torch.Tensor], sink, aux):
        """Forward of microbatch m on this stratum: (stage input, stage output, loss or None, router
        probabilities kept for the aux-loss backward when layers keep their graph)."""
        first, last = self.rank == 0, self.rank + 1 == self.world
        if first:
            tup = self.prefix(input_ids=ids[m])
            h_in = tup[0]
        else:
            h_in = x_recv.requires_grad_(True)
            tup = self.prefix.context(h_in)
        rest = tup[1:]
        probs: list = []
        if self.recompute:
            out = _run_stage(self.stage, h_in, rest, self.streamer, "step", sink, aux, self.offload)
        else:
            t = (h_in,) + rest
            for i, layer in enumerate(self.stage.layers):
                self.streamer.acquire(i)
                if sink is not None:
                    sink.clear()
                    sink.active = True
                try:
                    t = layer(t)
                finally:
                    if sink is not None:
                        sink.active = False
                if sink is not None:
                    for p, idx in zip(sink.probs, sink.indices):
                        aux.add(p, idx)
                        probs.append(p)
                    sink.clear()
            out = t[0]
        loss = self.postfix((out,) + rest[:4] + (labs[m],) + rest[5:]) if last else None
        return h_in, out, loss, probs

    def _backward_mb(self, out, loss, g, M: int, aux: Optional[_AuxState] = None, probs=()):
        outs, grads = [], []
        if loss is not None:
            outs.append(loss / M)
            grads.append(torch.ones((), dtype=loss.dtype, device=loss.device))
        else:
            outs.append(out)
            grads.append(g)
        if probs and aux is not None and aux.weight is not None:  # graph kept: the aux term's gradient here
            term = sum((torch.softmax(p.float(), dim=-1) * aux.weight).sum() for p in probs)
            if term.requires_grad:
                outs.append(term)
                grads.append(torch.ones((), dtype=term.dtype, device=term.device))
        torch.autograd.backward(outs, grads)

    def _train_1f1b(self, ids, labs, M: int, shape, use_aux: bool):
        """1F1B.  With the router aux loss, every boundary message carries the
        microbatch's router sums: forward, the sums of the ranks so far; backward,
        the global sums, from which each rank forms the aux gradient before
        running that microbatch's backward."""
        first, last = self.rank == 0, self.rank + 1 == self.world
        dev, dt, ch = self.device, self.hidden_dtype, self.chan
        sink = self.router_sink if use_aux else None
        E = self.n_experts
        act = [(shape, dt, dev)] + ([((2 * E + 1,), torch.float32, dev)] if use_aux else [])
        warm = min(self.world - self.rank - 1, M)
        rem = M - warm
        inflight = []
        losses = []
        aux_values = []
        mf = 0

        def fwd(msg):
            nonlocal mf
            x = None if msg is None else msg[0]
            aux = _AuxState(E, self.router_aux_coef) if use_aux else None
            h_in, out, loss, probs = self._forward_mb(mf, ids, labs, shape, x, sink, aux)
            mf += 1
            stats = None
            if use_aux:
                stats = self._stats(aux) + (msg[1] if msg is not None else 0.0)
                if last:  # global sums of this microbatch: finalize here, send them back with the gradient
                    aux.finalize(stats[:E], stats[E:2 * E], stats[2 * E], grad_scale=1.0 / M)
                    aux_values.append(aux.value.detach())
            if loss is not None:
                losses.append(loss.detach())
            inflight.append((h_in, out, loss, aux, probs, stats))
            return [out.detach()] + ([stats] if use_aux else [])

        def bwd(msg):
            h_in, out, loss, aux, probs, stats = inflight.pop(0)
            g = None if msg is None else msg[0]
            if use_aux and not last:
                gs = msg[1]
                aux.finalize(gs[:E], gs[E:2 * E], gs[2 * E], grad_scale=1.0 / M)
                stats = gs
            self._backward_mb(out, loss, g, M, aux, probs)
            if first:
                return None
            return [h_in.grad] + ([stats] if use_aux else [])

        for _ in range(warm):
            msg = None if first else ch.recv_forward(act)
            y = fwd(msg)
            if not last:
                ch.send_forward(y)
        msg = None if (first or rem == 0) else ch.recv_forward(act)
        for i in range(rem):
            y = fwd(msg)
            gmsg = None if last else ch.send_forward_recv_backward(y, act)
            gx = bwd(gmsg)
            if i == rem - 1:
                if not first:
                    ch.send_backward(gx)
            elif first:
                msg = None
            else:
                msg = ch.send_backward_recv_forward(gx, act)
        for _ in range(warm):
            gmsg = None if last else ch.recv_backward(act)
            gx = bwd(gmsg)
            if not first:
                ch.send_backward(gx)
        if use_aux and last:
            self.last_aux = torch.stack(aux_values).mean()
        return losses

    # ------------------------------------------------------------ CUDA graph

    def _one_microbatch(self, ids, labs, M: int) -> torch.Tensor:
        """Forward and backward of the microbatch in ``ids`` / ``labs`` ([1, 1, S]), loss scaled by 1/M."""
        _, out, loss, _ = self._forward_mb(0, ids, labs, None, None, None, None)
        self._backward_mb(out, loss, None, M)
        return loss.detach()

    def _graph_build(self, M: int, S: int):
        from . import _lib

        dev = self.device
        trainable = [p for p in self.parameters() if p.requires_grad]
        saved = [p.grad for p in trainable]
        ids = torch.zeros((1, 1, S), dtype=torch.int64, device=dev)
        labs = torch.zeros((1, 1, S), dtype=torch.int64, device=dev)
        # warm-up off the capture (library handles, workspaces, kernel attributes), on a
        # side stream as capture requires; its gradients are discarded
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):
                for p in trainable:
                    p.grad = None
                self._one_microbatch(ids, labs, M)
        torch.cuda.current_stream(dev).wait_stream(side)
        params = [p for p in trainable if p.grad is not None]  # the ones this stratum's loss reaches
        accs = [torch.zeros_like(p) for p in params]
        loss_acc = torch.zeros((), dtype=torch.float32, device=dev)
        for p in trainable:
            p.grad = None  # the captured backward creates them in the graph's pool; every replay rewrites them
        graph = torch.cuda.CUDAGraph()
        n0 = _lib.launch_count()
        with torch.cuda.graph(graph):
            loss = self._one_microbatch(ids, labs, M)
            loss_acc.add_(loss.float())
            torch._foreach_add_(accs, [p.grad for p in params])
        launches = _lib.launch_count() - n0
        pool_grads = [p.grad for p in params]  # owned by the graph's pool: kept alive with the graph
        for p, g in zip(trainable, saved):
            p.grad = g
        return graph, ids, labs, params, accs, loss_acc, pool_grads, launches, _address_signature(self)

    def _graph_train(self, ids, labs, M: int) -> torch.Tensor:
        key = (M, int(ids.shape[-1]))
        if key in self._graphs and self._graphs[key][-1] != _address_signature(self):
            self._graphs.clear()  # a parameter or weight moved: every graph reads stale addresses
        if key not in self._graphs:
            self._graphs[key] = self._graph_build(*key)
        graph, sids, slabs, params, accs, loss_acc, _, launches, _ = self._graphs[key]
        torch._foreach_zero_(accs)
        loss_acc.zero_()
        for m in range(M):
            sids.copy_(ids[m:m + 1])
            slabs.copy_(labs[m:m + 1])
            graph.replay()
        self.graph_launches += M * launches
        for p, a in zip(params, accs):
            if p.grad is None:
                p.grad = a.clone()
            else:
                p.grad.add_(a)
        _check_status([self.device], "RankPipeline.train_step")
        return loss_acc / M

    def _grads_before(self) -> list:
        return [(p, None if p.grad is None else p.grad.detach().clone()) for p in self.parameters()
                if p.requires_grad]

    @staticmethod
    def _grads_restore(saved: list) -> None:
        for p, g in saved:
            p.grad = None if g is None else g.clone()  # a copy: the next attempt accumulates into it

    def _failed_anywhere(self, failed: bool) -> bool:
        """Whether this rank or any other saw its step fail (one all-reduce when world > 1)."""
        if self.world == 1 or not dist.is_initialized():
            return failed
        flag = torch.tensor([1.0 if failed else 0.0], dtype=torch.float32, device=self.device)
        dist.all_reduce(flag, op=dist.ReduceOp.MAX, group=self.group)
        return bool(flag.item() > 0)

    def train_step(self, input_ids: Optional[torch.Tensor] = None, labels: Optional[torch.Tensor] = None, *,
                   microbatches: int = 1, seq_len: Optional[int] = None):
        M = int(microbatches)
        if self.cuda_graph:
            dev = self.device
            with _on(dev):
                ids = input_ids.reshape(M, 1, -1).to(dev, non_blocking=True)
                labs = labels.reshape(M, 1, -1).to(dev, non_blocking=True)
                return self._graph_train(ids, labs, M)
        if self.step_retries == 0:
            return self._train_step_once(input_ids, labels, M, seq_len)
        from ._lib import StratumError

        saved = self._grads_before()
        for attempt in range(self.step_retries + 1):
            err, out = None, None
            try:
                out = self._train_step_once(input_ids, labels, M, seq_len)
            except StratumError as exc:
                err = exc
            if not self._failed_anywhere(err is not None):
                return out
            if attempt == self.step_retries:
                raise err if err is not None else StratumError(
                    "RankPipeline.train_step: a device-side wait gave up on another rank in every attempt")
            self.status_retries += 1
            self._grads_restore(saved)

    def _train_step_once(self, input_ids, labels, M: int, seq_len: Optional[int]):
        first, last = self.rank == 0, self.rank + 1 == self.world
        dev = self.device
        if first:
            ids = input_ids.reshape(M, 1, -1).to(dev, non_blocking=True)
            seq_len = ids.shape[-1]
        if last:
            labs = labels.reshape(M, 1, -1).to(dev, non_blocking=True)
            seq_len = labs.shape[-1]
        if seq_len is None:
            raise ValueError("RankPipeline.train_step: seq_len is needed on middle ranks")
        shape = (1, seq_len, self.hidden_size)
        use_aux = self.router_sink is not None and self.router_aux_coef != 0.0 and self.n_experts > 0
        if self.schedule == "1f1b":
            with _on(dev):
                for i in range(len(self.stage.layers)):  # the stratum's upload, overlapped with microbatch 0
                    self.streamer.prefetch(i)
                losses = self._train_1f1b(ids if first else None, labs if last else None, M, shape, use_aux)
                self.chan.flush()
                self.streamer.release_all()
            _check_status([dev], "RankPipeline.train_step")
            if not last:
                return None
            loss = torch.stack(losses).mean()
            return loss + self.last_aux.to(loss.device) if use_aux else loss
        sink = self.router_sink if use_aux else None
        records = []
        losses = []
        with _on(dev):
            for i in range(len(self.stage.layers)):  # the stratum's upload, overlapped with microbatch 0
                self.streamer.prefetch(i)
            for m in range(M):
                if first:
                    tup = self.prefix(input_ids=ids[m])
                    h_in = tup[0]
                else:
                    h_in = self.chan.recv_forward([(shape, self.hidden_dtype, dev)])[0].requires_grad_(True)
                    tup = self.prefix.context(h_in)
                aux = _AuxState(self.n_experts, self.router_aux_coef) if use_aux else None
                rest = tup[1:]
                out = _run_stage(self.stage, h_in, rest, self.streamer, "step", sink, aux, self.offload)
                if last:
                    losses.append(self.postfix((out,) + rest[:4] + (labs[m],) + rest[5:]))
                else:
                    self.chan.send_forward(out.detach())
                records.append((h_in, out, aux))
            aux_states = [r[2] for r in records]
            if use_aux:
                self._aux_reduce(aux_states)
            for m in reversed(range(M)):
                h_in, out, aux = records[m]
                if last:
                    (losses[m] / M).backward()
                else:
                    g = self.chan.recv_backward([(shape, self.hidden_dtype, dev)])[0]
                    torch.autograd.backward(out, g)
                if not first:
                    self.chan.send_backward(h_in.grad)
                records[m] = None
            self.chan.flush()
            self.streamer.release_all()
        _check_status([dev], "RankPipeline.train_step")
        if use_aux:
            self.last_aux = torch.stack([r.value for r in aux_states]).mean()
        if not last:
            return None
        loss = torch.stack([l.detach() for l in losses]).mean()
        if use_aux:
            loss = loss + self.last_aux.to(loss.device)
        return loss


__all__ = ["StratumPipeline", "RankPipeline"]
