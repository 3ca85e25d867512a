"""Pipeline boundaries: activations forward, gradients backward, GPU to GPU.

Replaces the reference's host-staged boundary (stratum/host_staging.py:72-200,
``HostStagingPool.transfer`` / ``transfer_async``: peer copy when available,
else device -> pinned host -> device with a host sync) and its gradient hook
(stratum/grad_hooks.py:8-30, ``make_boundary_hook``).  On an NVSwitch box every
GPU reaches every other at full NVLink bandwidth, so no path goes through host
memory:

* one process driving several GPUs (``StratumPipeline``): a boundary is a
  device-to-device copy on the destination's current stream, ordered after the
  source's pending work by an event, and differentiable -- the gradient flows
  back through the same kind of copy;
* one process per GPU (``RankPipeline``): a boundary is an NCCL ``send`` /
  ``recv`` pair between adjacent ranks (:class:`P2PChannel`), activations
  forward and gradients backward, enqueued on the ranks' compute streams so the
  host never waits for them.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist


def _device(d) -> torch.device:
    if isinstance(d, torch.device):
        return d
    if isinstance(d, str):
        return torch.device(d)
    return torch.device("cuda", int(d))


class _DeviceCopy(torch.autograd.Function):
    """``x`` copied to ``dst`` after the source device's current work; the
    backward copies the gradient back the same way."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, dst: torch.device):
        ctx.src = x.device
        return _copy_after(x, dst)

    @staticmethod
    def backward(ctx, g: torch.Tensor):
        return _copy_after(g, ctx.src), None


def _copy_after(x: torch.Tensor, dst: torch.device) -> torch.Tensor:
    if x.device == dst:
        return x
    if x.is_cuda and dst.type == "cuda":
        # the destination stream waits for the source stream's pending writes of x
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(x.device))
        out_stream = torch.cuda.current_stream(dst)
        out_stream.wait_event(ev)
        with torch.cuda.device(dst), torch.cuda.stream(out_stream):
            out = torch.empty_like(x, device=dst)
            out.copy_(x, non_blocking=True)  # peer copy over NVLink
        # x must outlive the copy, which runs on the destination's stream
        x.record_stream(out_stream)
        return out
    return x.to(dst)


def _typed_buffer_view(buffer: torch.Tensor, dtype: torch.dtype, numel: int) -> torch.Tensor:
    """The first ``numel`` elements of ``dtype`` over a byte buffer (the staging
    buffer of a host-staged boundary copy)."""
    nbytes = numel * torch.empty((), dtype=dtype).element_size()
    return buffer.narrow(0, 0, nbytes).view(dtype)


def _peer_ok(a: torch.device, b: torch.device) -> bool:
    try:
        return torch.cuda.can_device_access_peer(a.index or 0, b.index or 0)
    except (RuntimeError, AssertionError):
        return False


def transfer(x: torch.Tensor, dst_device) -> torch.Tensor:
    """Move a boundary activation to ``dst_device`` (differentiable)."""
    dst = _device(dst_device)
    if x.device == dst:
        return x
    if x.requires_grad:
        return _DeviceCopy.apply(x, dst)
    return _copy_after(x, dst)


class DeviceTransferPool:
    """Drop-in for ``HostStagingPool`` (stratum/host_staging.py:47-200): same
    ``transfer`` / ``transfer_async`` calls, but a direct device-to-device copy
    (NVLink peer access, every GPU pair of an NVSwitch box) with no host
    synchronisation.  Only between GPUs without peer access does a copy go
    through a pinned host buffer, as the reference's always does."""

    def __init__(self):
        self._buf: Optional[torch.Tensor] = None

    def ensure(self, size_bytes: int) -> None:
        """Grow the pinned staging buffer (used only between GPUs without peer access)."""
        if self._buf is None or self._buf.numel() < size_bytes:
            self._buf = torch.empty(int(size_bytes), dtype=torch.uint8, pin_memory=torch.cuda.is_available())

    def _staged(self, x: torch.Tensor, dst: torch.device) -> torch.Tensor:
        flat = x.detach().reshape(-1)
        self.ensure(flat.numel() * flat.element_size())
        host = _typed_buffer_view(self._buf, flat.dtype, flat.numel())
        host.copy_(flat)  # synchronous D2H: the buffer is reused by the next transfer
        out = torch.empty(x.shape, dtype=x.dtype, device=dst)
        out.view(-1).copy_(host)
        torch.cuda.current_stream(dst).synchronize()
        return out

    def transfer(self, tensor: torch.Tensor, dst_device, src_device=None) -> torch.Tensor:
        dst = _device(dst_device)
        if (tensor.is_cuda and dst.type == "cuda" and tensor.device != dst and not tensor.requires_grad
                and not _peer_ok(tensor.device, dst)):
            return self._staged(tensor, dst)
        return transfer(tensor, dst_device)

    def transfer_async(self, tensor: torch.Tensor, dst_device, src_device=None):
        out = transfer(tensor, dst_device)
        ev = None
        if out.is_cuda:
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(out.device))
        return out, ev


def make_boundary_hook(prev_device, next_device, pool: Optional[DeviceTransferPool] = None):
    """Gradient hook moving a boundary gradient from ``next_device`` back to
    ``prev_device`` (stratum/grad_hooks.py:8-30), by a direct device copy."""
    prev = _device(prev_device)

    def hook(grad: torch.Tensor) -> torch.Tensor:
        return _copy_after(grad, prev)

    return hook


class P2PChannel:
    """NCCL point-to-point boundary between this rank and its pipeline neighbours.

    ``send_forward`` / ``recv_forward`` carry the stage output to the next rank;
    ``send_backward`` / ``recv_backward`` carry the gradient of the stage input
    to the previous rank.  Each takes or returns a list of tensors (the boundary
    activation, plus any small side tensors that travel with it); every call is
    one batched NCCL group.  Both ends issue their calls in the same order (the
    schedule guarantees it); NCCL runs the transfers on its own stream, ordered
    after the caller's current stream, and received tensors are ordered before
    the caller's next work, so the host does not block.
    """

    def __init__(self, rank: int, world: int, group=None):
        self.rank, self.world, self.group = rank, world, group
        self.prev = rank - 1 if rank > 0 else None
        self.next = rank + 1 if rank + 1 < world else None
        # send-only groups in flight: (works, tensors kept alive until the sends complete)
        self._pending: list = []
        # when a list: (start, end) CUDA event pairs around every wait of the caller's
        # stream for received tensors (the time this rank's compute sat idle on a neighbour)
        self.wait_events: Optional[list] = None

    def _peer(self, r: int) -> int:
        return dist.get_global_rank(self.group, r) if self.group is not None else r

    def _retire(self) -> None:
        self._pending = [(ws, ts) for ws, ts in self._pending if not all(w.is_completed() for w in ws)]

    def flush(self) -> None:
        """Order the caller's stream after every send still in flight and drop the
        references that kept their tensors alive (end of a step)."""
        for ws, _ in self._pending:
            for w in ws:
                w.wait()
        self._pending.clear()

    @property
    def sends_in_flight(self) -> int:
        return len(self._pending)

    def exchange(self, sends=(), recvs=()) -> list:
        """One NCCL group: ``sends`` = [(tensor, rank)], ``recvs`` = [(shape, dtype, device, rank)];
        returns the received tensors in order.

        A group that receives is waited on by the caller's stream (NCCL completes a
        group as a whole, so its sends are waited on with the receives they are paired
        with -- in 1F1B those pairs mirror the neighbour's and finish together).  A
        send-only group is not waited on: the caller's stream runs on while NCCL's
        stream transfers, and the sent tensors stay referenced until the host sees the
        group complete (or ``flush``), so the allocator cannot recycle them early."""
        self._retire()
        ops, out, held = [], [], []
        for t, r in sends:
            t = t.contiguous()
            held.append(t)
            ops.append(dist.P2POp(dist.isend, t, self._peer(r), self.group))
        for shape, dtype, device, r in recvs:
            buf = torch.empty(shape, dtype=dtype, device=device)
            out.append(buf)
            ops.append(dist.P2POp(dist.irecv, buf, self._peer(r), self.group))
        if not ops:
            return out
        works = dist.batch_isend_irecv(ops)
        if not recvs:
            self._pending.append((works, held))
            return out
        timed = self.wait_events is not None and out and out[0].is_cuda
        if timed:
            e0 = torch.cuda.Event(enable_timing=True)
            e0.record()
        for w in works:
            w.wait()
        if timed:
            e1 = torch.cuda.Event(enable_timing=True)
            e1.record()
            self.wait_events.append((e0, e1))
        return out

    def send_forward(self, xs) -> None:
        self.exchange(sends=[(x, self.next) for x in _as_list(xs)])

    def recv_forward(self, specs) -> list:
        return self.exchange(recvs=[(s, d, dev, self.prev) for s, d, dev in specs])

    def send_backward(self, gs) -> None:
        self.exchange(sends=[(g, self.prev) for g in _as_list(gs)])

    def recv_backward(self, specs) -> list:
        return self.exchange(recvs=[(s, d, dev, self.next) for s, d, dev in specs])

    def send_forward_recv_backward(self, ys, specs) -> list:
        """Send this stage's outputs to the next rank and receive the gradients of an
        earlier output from it, as one NCCL group (the two ranks issue the mirror
        pair at the same time in a 1F1B schedule; separate blocking calls would
        wait on each other)."""
        return self.exchange(sends=[(y, self.next) for y in _as_list(ys)],
                             recvs=[(s, d, dev, self.next) for s, d, dev in specs])

    def send_backward_recv_forward(self, gs, specs) -> list:
        """Send input gradients to the previous rank and receive its next outputs."""
        return self.exchange(sends=[(g, self.prev) for g in _as_list(gs)],
                             recvs=[(s, d, dev, self.prev) for s, d, dev in specs])


def _as_list(xs):
    return list(xs) if isinstance(xs, (list, tuple)) else [xs]
