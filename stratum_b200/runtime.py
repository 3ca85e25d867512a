"""Recompute anchors: a layer group's backward re-runs its forward.

The reference's memory model (stratum/runtime.py:74-290,
``capture_backward_input`` / ``anchor_explicit_group_backward``): a group of
layers runs forward without an autograd graph and keeps only its input; when
the gradient of the group's output arrives, the group runs again with autograd
on from the saved input and backpropagates through the recomputation.  This
module provides that API (same function names and keyword arguments) on its
own implementation; the pipelines in ``stratum_b200.pipeline`` build every
layer group on it.

``anchor_explicit_group_backward(run_group=..., group_input=..., group_output=...)``
returns ``group_output`` with its floating-point tensors replaced by tensors
whose backward (one custom autograd node for the whole group):

1. calls ``look_ahead_upload()`` -- the caller starts the next group's weight
   upload so it overlaps this recomputation;
2. recomputes ``run_group(saved input)`` with autograd and backpropagates the
   incoming gradients (plus any ``extra_terms()`` scalars, e.g. a router aux
   loss, with gradient 1);
3. calls ``on_backward_complete()``, then returns the input gradients.
"""

from __future__ import annotations

import copy
from dataclasses import dataclass, field
from typing import Any, Callable, Optional

import torch
from torch.utils._pytree import tree_flatten, tree_unflatten


@dataclass
class CapturedInput:
    """A group input saved for its recomputation: the flattened pytree with tensor
    leaves detached (optionally moved to host memory) and where they came from."""

    flat: list
    spec: Any
    tensor_devices: list
    tensor_requires_grad: list

    def restore(self) -> Any:
        """The input again, tensors back on their devices as fresh autograd leaves."""
        out = []
        for item, dev, rg in zip(self.flat, self.tensor_devices, self.tensor_requires_grad):
            if torch.is_tensor(item):
                t = item if item.device == dev else item.to(dev, non_blocking=True)
                out.append(t.detach().requires_grad_(bool(rg)))
            else:
                out.append(item)
        return tree_unflatten(out, self.spec)


def capture_backward_input(value: Any, *, offload_to_cpu: bool = False) -> CapturedInput:
    """Save ``value`` (a pytree) for a later recomputation: tensors detached (to host
    memory with ``offload_to_cpu``), other leaves copied so later mutation by the
    caller cannot change the recomputation."""
    flat, spec = tree_flatten(value)
    saved, devices, grads = [], [], []
    for item in flat:
        if torch.is_tensor(item):
            devices.append(item.device)
            grads.append(item.requires_grad)
            t = item.detach()
            if offload_to_cpu and t.device.type != "cpu":
                t = t.to("cpu")
            saved.append(t)
        else:
            devices.append(None)
            grads.append(None)
            saved.append(copy.copy(item))
    return CapturedInput(saved, spec, devices, grads)


@dataclass
class _AnchorMeta:
    """What one group's backward needs: how to rerun it, its saved input, which
    flattened input / output leaves carry gradients, and the caller's hooks."""

    run_group: Callable[[Any], Any]
    captured_input: CapturedInput
    input_indices: list
    output_indices: list
    output_leaf_count: int
    output_spec: Any
    recompute_data: Any = None
    timing_recorder: Any = None
    timing_fields: dict = field(default_factory=dict)
    compute_stream: Any = None
    on_backward_complete: Optional[Callable[[], None]] = None
    look_ahead_upload: Optional[Callable[[], None]] = None
    extra_terms: Optional[Callable[[], list]] = None
    done: bool = False


class _GroupAnchor(torch.autograd.Function):
    @staticmethod
    def forward(ctx, meta: _AnchorMeta, anchor: torch.Tensor, *tensors):
        ctx.meta = meta
        n_in = len(meta.input_indices)
        # the already computed outputs, handed on as this node's outputs
        return tuple(t.view_as(t) for t in tensors[n_in:])

    @staticmethod
    def backward(ctx, *grads):
        meta: _AnchorMeta = ctx.meta
        if meta.done:
            raise RuntimeError("a layer group's recompute backward can run only once (no double backward)")
        meta.done = True
        if meta.look_ahead_upload is not None:
            meta.look_ahead_upload()
        inp = meta.captured_input.restore()
        flat_in, _ = tree_flatten(inp)
        stream = meta.compute_stream
        ctx_stream = torch.cuda.stream(stream) if stream is not None else None
        if ctx_stream is not None:
            ctx_stream.__enter__()
        try:
            with torch.enable_grad():
                out = meta.run_group(inp)
                flat_out, _ = tree_flatten(out)
                roots, root_grads = [], []
                for idx, g in zip(meta.output_indices, grads):
                    t = flat_out[idx]
                    if g is not None and torch.is_tensor(t) and t.requires_grad:
                        roots.append(t)
                        root_grads.append(g)
                for term in (meta.extra_terms() if meta.extra_terms is not None else []):
                    if torch.is_tensor(term) and term.requires_grad:
                        roots.append(term)
                        root_grads.append(torch.ones_like(term))
                if roots:
                    torch.autograd.backward(roots, root_grads)
        finally:
            if ctx_stream is not None:
                ctx_stream.__exit__(None, None, None)
        in_grads = [flat_in[i].grad for i in meta.input_indices]
        if meta.on_backward_complete is not None:
            meta.on_backward_complete()
        ctx.meta = None
        return (None, None) + tuple(in_grads) + (None,) * len(meta.output_indices)


def anchor_explicit_group_backward(*, run_group: Callable[[Any], Any], group_input: Any, group_output: Any,
                                   captured_input: Optional[CapturedInput] = None, recompute_data: Any = None,
                                   timing_recorder: Any = None, timing_fields: Optional[dict] = None,
                                   compute_stream: Any = None, offload_input_to_cpu: bool = False,
                                   on_backward_complete: Optional[Callable[[], None]] = None, iter_timer: Any = None,
                                   layer_ids: Any = None, look_ahead_upload: Optional[Callable[[], None]] = None,
                                   extra_terms: Optional[Callable[[], list]] = None) -> Any:
    """``group_output`` whose gradient path recomputes ``run_group(group_input)``.

    Tensor leaves of ``group_input`` that require grad receive gradients; the
    floating-point tensor leaves of ``group_output`` are replaced (same values,
    same pytree).  ``extra_terms`` (this build's addition): called after the
    recomputation, returns scalar tensors that are backpropagated with gradient 1
    along with the output gradients."""
    flat_in, _ = tree_flatten(group_input)
    flat_out, out_spec = tree_flatten(group_output)
    in_idx = [i for i, t in enumerate(flat_in) if torch.is_tensor(t) and t.requires_grad]
    out_idx = [i for i, t in enumerate(flat_out) if torch.is_tensor(t) and t.is_floating_point()]
    if captured_input is None:
        captured_input = capture_backward_input(group_input, offload_to_cpu=offload_input_to_cpu)
    meta = _AnchorMeta(run_group=run_group, captured_input=captured_input, input_indices=in_idx,
                       output_indices=out_idx, output_leaf_count=len(flat_out), output_spec=out_spec,
                       recompute_data=recompute_data, timing_recorder=timing_recorder,
                       timing_fields=dict(timing_fields or {}), compute_stream=compute_stream,
                       on_backward_complete=on_backward_complete, look_ahead_upload=look_ahead_upload,
                       extra_terms=extra_terms)
    # a leaf that requires grad, so the outputs join the graph even when no input does
    # (the group's trainable parameters are reached through the recomputation)
    anchor = torch.empty(0, requires_grad=True)
    outs = _GroupAnchor.apply(meta, anchor, *[flat_in[i] for i in in_idx], *[flat_out[i].detach() for i in out_idx])
    new_flat = list(flat_out)
    for i, t in zip(out_idx, outs):
        new_flat[i] = t
    return tree_unflatten(new_flat, out_spec)


__all__ = ["CapturedInput", "capture_backward_input", "anchor_explicit_group_backward"]
