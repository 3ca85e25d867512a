"""Layer-group execution plans for ``StratumPipeline``.

The reference's ``StratumPipeline(..., execute_plan=...)`` (stratum/pipeline.py:90-99)
takes a ``ModelExecutePlan`` (stratum/scheduler.py:36-113): contiguous layer
ranges that run forward as one recompute group each, listed in forward order
(``fwd_plan``) and in backward order (``bwd_plan``).  This module keeps that
type -- its constructors and its validity check -- so callers that build plans
keep working.  The timing-driven plan search and the tracker the reference
builds on top of it belong to its scheduler, not to the NF4 path, and are not
provided.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional, Sequence


def _ranges(items) -> list[range]:
    out = []
    for r in items:
        if not isinstance(r, range):
            r = range(int(r[0]), int(r[1]))
        if r.step != 1:
            raise ValueError(f"layer ranges must be contiguous, got {r}")
        out.append(range(r.start, r.stop))
    return out


@dataclass
class ModelExecutePlan:
    """Forward and backward layer groups (``range`` objects over global layer ids)."""

    fwd_plan: list[range] = field(default_factory=list)
    bwd_plan: list[range] = field(default_factory=list)

    @classmethod
    def from_stage_ranges(cls, fwd_plan: Sequence[range],
                          bwd_plan: Optional[Sequence[range]] = None) -> "ModelExecutePlan":
        """Explicit groups; the backward order defaults to the forward groups reversed."""
        fwd = _ranges(fwd_plan)
        bwd = _ranges(bwd_plan) if bwd_plan is not None else list(reversed(fwd))
        return cls(fwd, bwd)

    @classmethod
    def from_stage_lengths(cls, lengths: Sequence[int]) -> "ModelExecutePlan":
        """One group per stage, from the stages' layer counts."""
        groups, start = [], 0
        for n in lengths:
            if int(n) <= 0:
                raise ValueError(f"stage lengths must be positive, got {n}")
            groups.append(range(start, start + int(n)))
            start += int(n)
        return cls.from_stage_ranges(groups)

    @classmethod
    def per_layer(cls, n_layers: int) -> "ModelExecutePlan":
        """One group per layer (the finest recompute granularity)."""
        return cls.from_stage_ranges([range(i, i + 1) for i in range(int(n_layers))])

    def check_valid(self, num_layers: int, run_type: str = "train") -> None:
        """Raise ``ValueError`` unless the forward groups cover layers 0..num_layers-1 in
        order (``"infer"`` / ``"train"``), and for training the backward groups, read
        last to first, cover them too."""
        def walk(groups, what, start):
            nxt = start
            for r in groups:
                if len(r) == 0:
                    raise ValueError(f"empty layer range in {what} plan")
                if r.start != nxt:
                    raise ValueError(f"{what} plan: layer {r.start} follows layer {nxt - 1}")
                nxt = r.stop
            return nxt

        if run_type not in ("infer", "train", "fused"):
            raise ValueError(f"unknown run type {run_type!r}")
        end = walk(self.fwd_plan, "forward", 0)
        if run_type in ("infer", "train") and end != num_layers:
            raise ValueError(f"forward plan covers {end} of {num_layers} layers")
        if run_type == "infer":
            return
        # training: the backward groups cover every layer; fused: the layers after the forward groups
        bstart = 0 if run_type == "train" else end
        bend = walk(list(reversed(self.bwd_plan)), "backward", bstart)
        if bend != num_layers:
            raise ValueError(f"backward plan ends at layer {bend}, not {num_layers}")

    def __repr__(self) -> str:
        return f"Fwd Plan: {self.fwd_plan}, Bwd Plan: {self.bwd_plan}"


__all__ = ["ModelExecutePlan"]
