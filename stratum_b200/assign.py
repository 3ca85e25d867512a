"""Layer-to-device assignment (reference: stratum/assign.py:9-83).

Same rule as the reference (llama.cpp's LLAMA_SPLIT_MODE_LAYER): the devices
own consecutive fractions of the layer range given by the cumulative,
normalised ``tensor_split``; layer i goes to the first device whose cumulative
fraction is >= i / n_layers (a lower-bound search).  On an 8 x B200 box each
device holds one stratum of consecutive layers.
"""

from __future__ import annotations

from bisect import bisect_left
from typing import Optional


def assign_layers_to_devices(
    n_layers: int,
    tensor_split: Optional[list[float]] = None,
    device_ids: Optional[list[int]] = None,
    n_devices: Optional[int] = None,
) -> dict[int, int]:
    """Map each decoder layer index to a device id."""
    if tensor_split is not None:
        nd = len(tensor_split)
        if nd == 0:
            raise ValueError("tensor_split list is empty")
    elif n_devices is not None:
        nd = n_devices
        if nd <= 0:
            raise ValueError(f"n_devices must be >= 1, got {nd}")
    else:
        nd = 1
    if device_ids is None:
        device_ids = list(range(nd))
    elif len(device_ids) != nd:
        raise ValueError(f"device_ids length {len(device_ids)} != n_devices {nd}")
    if nd == 1:
        return {i: device_ids[0] for i in range(n_layers)}
    if tensor_split is not None:
        total = float(sum(tensor_split))
        if total <= 0:
            raise ValueError("tensor_split must sum to > 0")
        acc, bounds = 0.0, []
        for s in tensor_split:
            acc += s
            bounds.append(acc / total)
    else:
        bounds = [(i + 1) / nd for i in range(nd)]
    return {i: device_ids[min(bisect_left(bounds, i / n_layers), nd - 1)] for i in range(n_layers)}


def strata(assignment: dict[int, int]) -> list[tuple[int, list[int]]]:
    """Consecutive runs of layers per device: [(device_id, [layer indices]), ...]."""
    out: list[tuple[int, list[int]]] = []
    for layer in sorted(assignment):
        dev = assignment[layer]
        if out and out[-1][0] == dev:
            out[-1][1].append(layer)
        else:
            out.append((dev, [layer]))
    return out


def balanced_strata(n_layers: int, n_devices: int, *, tail_cost: float = 0.0,
                    head_cost: float = 0.0) -> list[list[int]]:
    """Contiguous layer strata, one per device, minimising the largest per-device
    load when the first device also runs the prefix (``head_cost``) and the last
    the postfix (``tail_cost``), both in units of one decoder layer.

    The reference splits by user weights with a cumulative rule
    (stratum/assign.py:9-83, :func:`assign_layers_to_devices`), which rounds a
    cost-aware split unevenly; this picks the integer layer counts directly."""
    if n_devices <= 0:
        raise ValueError("n_devices must be positive")
    extra = [0.0] * n_devices
    extra[0] += head_cost
    extra[-1] += tail_cost
    cands = sorted({k + e for e in extra for k in range(n_layers + 1)})
    counts = None
    for m in cands:  # smallest max load whose floor(m - extra) counts cover every layer
        c = [max(int(m - e + 1e-9), 0) for e in extra]
        if sum(c) >= n_layers:
            counts = c
            break
    surplus = sum(counts) - n_layers
    while surplus > 0:  # drop layers from the most loaded devices first
        r = max(range(n_devices), key=lambda i: (counts[i] + extra[i], counts[i]))
        counts[r] -= 1
        surplus -= 1
    out, start = [], 0
    for c in counts:
        out.append(list(range(start, start + c)))
        start += c
    return out
