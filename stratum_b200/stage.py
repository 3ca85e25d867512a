"""DeviceStage: a contiguous slice of decoder layers on one GPU (one stratum).

Reference: stratum/stage.py:14-140.  Same constructor and ``forward_range``
signature.  With a ``param_stream`` the NF4 payload of layer i+1 is uploaded on
that stream (one coalesced copy per layer when the layer has an arena; in
fused mode no dequantization happens at all) while layer i computes, and the
compute stream waits on a per-layer event before running the layer.
"""

from __future__ import annotations

from contextlib import nullcontext
from typing import Any, Optional

import torch
import torch.nn as nn

from .upload import ensure_weights


class DeviceStage(nn.Module):
    """Holds a contiguous slice of decoder layers on one CUDA device.

    Layers take and return the pipeline tuple (reference layer interface).
    Parameters are not moved here; the streaming contract uploads them.
    """

    def __init__(self, layers: list[nn.Module], device_id: int):
        super().__init__()
        self.device_id = device_id
        self.layers = nn.ModuleList(layers)
        self.timing_recorder = None
        self.layer_start = 0

    def set_timing_recorder(self, recorder, *, layer_start: int = 0) -> None:
        self.timing_recorder = recorder
        self.layer_start = layer_start

    def _time(self, name: str, **fields: Any):
        if self.timing_recorder is None:
            return nullcontext()
        return self.timing_recorder.span(name, device_id=self.device_id, **fields)

    def _upload(self, index: int, param_stream) -> "torch.cuda.Event":
        with torch.cuda.stream(param_stream):
            ensure_weights(self.layers[index], self.device_id)
            ev = torch.cuda.Event()
            ev.record(param_stream)
        return ev

    def forward_range(
        self,
        input_data,
        *,
        local_start: int = 0,
        local_stop: Optional[int] = None,
        iter_timer=None,
        param_stream: Optional["torch.cuda.Stream"] = None,
        first_layer_fence: Optional["torch.cuda.Event"] = None,
    ):
        """Run layers ``[local_start, local_stop)`` with per-layer upload overlap."""
        if local_stop is None:
            local_stop = len(self.layers)
        if local_start < 0 or local_stop > len(self.layers) or local_start >= local_stop:
            raise ValueError(f"invalid stage layer range {local_start}:{local_stop} for {len(self.layers)} layers")
        use_stream = param_stream is not None and torch.cuda.is_available()
        n = local_stop - local_start
        fences: list[Optional[torch.cuda.Event]] = [None] * n if use_stream else []
        if use_stream:
            fences[0] = first_layer_fence if first_layer_fence is not None else self._upload(local_start, param_stream)
        for i, idx in enumerate(range(local_start, local_stop)):
            if use_stream:
                if i + 1 < n and fences[i + 1] is None:  # next layer's upload goes first
                    fences[i + 1] = self._upload(local_start + i + 1, param_stream)
                torch.cuda.current_stream(self.device_id).wait_event(fences[i])
            layer_index = self.layer_start + idx
            ctx = iter_timer.time_fwd("fwd", layer_index, torch.cuda.current_stream(self.device_id)) \
                if (iter_timer is not None and torch.cuda.is_available()) else nullcontext()
            with ctx, self._time("layer_forward", stage_device=self.device_id, layer_index=layer_index,
                                 stage_layer_index=idx):
                input_data = self.layers[idx](input_data)
        return input_data

    def forward(self, input_data):
        return self.forward_range(input_data)
