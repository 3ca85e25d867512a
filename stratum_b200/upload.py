"""NF4 weight streaming: the reference's ``stratum/upload.py`` contract on B200 kernels.

Two phases, as in the reference (stratum/upload.py:1-12):

* :func:`prepare_nf4` quantizes each frozen >= 2-D parameter to NF4 (on the
  GPU, with the sm_100a quantizer), keeps the payload in pinned host memory on
  the parameter under :data:`NF4_ATTR`, and drops the original data.
* :func:`ensure_weights` / :func:`prefetch_weights` + :class:`NF4Prefetch`
  upload payloads host -> device, :func:`free_weights` drops the device copy.

Two ways a payload becomes usable on the device:

* compat mode (the reference's behaviour, stratum/upload.py:1021-1040): the
  payload is dequantized into ``param.data`` in ``payload.dtype`` so stock
  ``nn.Linear`` / HF modules run unchanged;
* fused mode: when the parameter belongs to an :class:`NF4Linear` built with
  :func:`to_nf4_linear`, only the packed bytes (and absmax) are uploaded and
  the fused GEMM consumes them directly -- the weight is never materialised.

A module can also carry a coalesced pinned arena (:func:`build_layer_arena`):
every NF4 payload of the module packed into one pinned buffer, uploaded with a
single copy per layer instead of one per tensor.

Cache files keep the reference's version-1 format (stratum/upload.py:287-302)
and add a version-2 format carrying the double-quant fields.
"""

from __future__ import annotations

import hashlib
import re
import time
from dataclasses import dataclass, field
from pathlib import Path
from typing import Optional, cast

import torch
import torch.nn as nn

from . import functional as F
from .functional import QuantState

NF4_ATTR = "roundpipe_nf4_payload"
FP16_ATTR = "stratum_fp16_staged"
ARENA_ATTR = "stratum_b200_nf4_arena"
CACHE_VERSION = 2


@dataclass
class NF4Stats:
    """NF4 preparation statistics (reference: stratum/upload.py:31-45)."""

    tensors: int = 0
    source_bytes: int = 0
    payload_bytes: int = 0
    cache_hits: int = 0
    cache_misses: int = 0
    cache_writes: int = 0

    @property
    def compression(self) -> float:
        if self.payload_bytes == 0:
            return 0.0
        return self.source_bytes / self.payload_bytes


def _pin_cpu(t: torch.Tensor) -> torch.Tensor:
    """Copy *t* into pinned host memory (reference: stratum/upload.py:48-55)."""
    t = t.detach().contiguous().cpu()
    if t.is_pinned() or not torch.cuda.is_available():
        return t
    pinned = torch.empty_like(t, device=torch.device("cpu"), pin_memory=True)
    pinned.copy_(t)
    return pinned


def _payload_bytes(*tensors: Optional[torch.Tensor]) -> int:
    return sum(t.numel() * t.element_size() for t in tensors if t is not None)


def _dtype_name(dtype: torch.dtype) -> str:
    return str(dtype).removeprefix("torch.")


def _dtype_from_name(name: str) -> torch.dtype:
    return cast(torch.dtype, getattr(torch, name.removeprefix("torch.")))


@dataclass
class NF4Payload:
    """NF4 payload of one frozen weight, kept in pinned host memory between steps.

    The first ten fields are the reference's (stratum/upload.py:70-95).  When
    ``nested`` is set the payload is double-quantized: ``absmax`` holds the
    uint8 codes and ``absmax2`` / ``code2`` / ``offset`` the second level.
    """

    quantized: torch.Tensor
    absmax: torch.Tensor
    code: torch.Tensor
    shape: tuple
    dtype: torch.dtype
    blocksize: int
    quant_type: str
    source_numel: int
    source_bytes: int
    payload_bytes: int
    nested: bool = False
    absmax2: Optional[torch.Tensor] = None
    code2: Optional[torch.Tensor] = None
    offset: Optional[torch.Tensor] = None
    blocksize2: int = 256

    def quant_state(self, device=None, absmax=None, absmax2=None, code=None, code2=None, offset=None) -> QuantState:
        """QuantState over this payload (or over device copies of its tensors)."""
        dev = lambda t: t if device is None else t.to(device, non_blocking=True)  # noqa: E731
        if self.nested:
            state2 = QuantState(absmax=absmax2 if absmax2 is not None else dev(self.absmax2),
                                code=code2 if code2 is not None else dev(self.code2), blocksize=self.blocksize2,
                                dtype=torch.float32)
            return QuantState(absmax if absmax is not None else dev(self.absmax), self.shape,
                              code if code is not None else dev(self.code), self.blocksize, self.quant_type,
                              self.dtype, offset=offset if offset is not None else dev(self.offset), state2=state2)
        return QuantState(absmax if absmax is not None else dev(self.absmax), self.shape,
                          code if code is not None else dev(self.code), self.blocksize, self.quant_type, self.dtype)

    def host_tensors(self) -> list[torch.Tensor]:
        ts = [self.quantized, self.absmax, self.code]
        if self.nested:
            ts += [self.absmax2, self.code2, self.offset.reshape(1)]
        return ts


@dataclass
class FP16StagedPayload:
    """Frozen 16-bit weight kept pinned on the host for per-step upload (stratum/upload.py:98-108)."""

    data: torch.Tensor
    shape: tuple
    dtype: torch.dtype
    source_bytes: int


# --------------------------------------------------------------------------------
# owner bookkeeping
# --------------------------------------------------------------------------------

def _replace_param_data(param: nn.Parameter, new_data: torch.Tensor, owner: Optional[nn.Module] = None,
                        pname: Optional[str] = None) -> None:
    """Set ``param.data``; re-register the parameter when a subclass rejects it
    (reference: stratum/upload.py:1286-1310)."""
    try:
        param.data = new_data
        return
    except (RuntimeError, TypeError):
        pass
    if owner is not None and pname is not None:
        new_param = nn.Parameter(new_data, requires_grad=param.requires_grad)
        for attr in (NF4_ATTR, FP16_ATTR):
            if hasattr(param, attr):
                setattr(new_param, attr, getattr(param, attr))
        owner.register_parameter(pname, new_param)


def _build_param_owner_map(module: nn.Module) -> dict[int, tuple[nn.Module, str]]:
    pmap: dict[int, tuple[nn.Module, str]] = {}
    for _, sub in module.named_modules():
        for pname, p in sub.named_parameters(recurse=False):
            pmap[id(p)] = (sub, pname)
    return pmap


class _ExpertsWeight:
    """One of a streamed NF4Experts' two weights, seen as a fused owner."""

    def __init__(self, owner, which: str):
        self.owner, self.which = owner, which

    def load_device_state(self, quantized, quant_state) -> None:
        self.owner.load_device_state(self.which, quantized, quant_state)

    def device_state_on(self, device) -> bool:
        return self.owner.device_state_on(self.which, device)

    def drop_device_state(self) -> bool:
        return self.owner.drop_device_state(self.which)


def _fused_owner(owner: Optional[nn.Module], pname: Optional[str]):
    """The fused module that consumes this parameter's payload directly, if any:
    a streamed NF4Linear (its ``weight``) or a streamed NF4Experts (its
    ``gate_up_weight`` / ``down_weight``)."""
    from .experts import NF4Experts
    from .nf4_linear import NF4Linear

    if isinstance(owner, NF4Linear) and pname == "weight" and owner.streamed:
        return owner
    if isinstance(owner, NF4Experts) and owner.streamed and pname in ("gate_up_weight", "down_weight"):
        return _ExpertsWeight(owner, pname)
    return None


# --------------------------------------------------------------------------------
# cache (reference format v1, plus v2 with double-quant fields)
# --------------------------------------------------------------------------------

def _canonical_param_name(name: str) -> str:
    return name.replace(".module.", ".")


def _cache_path(cache_dir: Path, name: str) -> Path:
    """``<sha1[:12]>-<sanitised name>.pt`` (reference naming, stratum/upload.py:236-240)."""
    name = _canonical_param_name(name)
    safe = re.sub(r"[^A-Za-z0-9_.-]+", "_", name)[-160:]
    digest = hashlib.sha1(name.encode("utf-8")).hexdigest()[:12]
    return cache_dir / f"{digest}-{safe}.pt"


def _load_payload_from_cache(path: Path, param: nn.Parameter, *, blocksize: int, quant_type: str,
                             compress_statistics: bool = False) -> Optional[NF4Payload]:
    """Load a cached payload; ``None`` on a missing file, an unreadable file or
    any metadata mismatch (reference: stratum/upload.py:243-284)."""
    if not path.exists():
        return None
    try:
        obj = torch.load(path, map_location="cpu", weights_only=False)
    except Exception:
        return None
    if not isinstance(obj, dict) or obj.get("version") not in (1, 2):
        return None
    expected = {
        "shape": tuple(param.shape),
        "dtype": _dtype_name(param.dtype),
        "blocksize": int(blocksize),
        "quant_type": str(quant_type),
        "source_numel": int(param.numel()),
        "source_bytes": int(param.numel() * param.element_size()),
    }
    for key, value in expected.items():
        got = obj.get(key)
        if key == "shape" and got is not None:
            got = tuple(got)
        if got != value:
            return None
    nested = bool(obj.get("nested", False))
    if nested != bool(compress_statistics):
        return None
    quantized = cast(torch.Tensor, obj["quantized"])
    absmax = cast(torch.Tensor, obj["absmax"])
    code = cast(torch.Tensor, obj["code"])
    extra = {}
    if nested:
        extra = dict(nested=True, absmax2=_pin_cpu(obj["absmax2"]), code2=_pin_cpu(obj["code2"]),
                     offset=_pin_cpu(obj["offset"].reshape(())), blocksize2=int(obj.get("blocksize2", 256)))
    return NF4Payload(
        quantized=_pin_cpu(quantized), absmax=_pin_cpu(absmax), code=_pin_cpu(code), shape=tuple(obj["shape"]),
        dtype=_dtype_from_name(str(obj["dtype"])), blocksize=int(obj["blocksize"]),
        quant_type=str(obj["quant_type"]), source_numel=int(obj["source_numel"]),
        source_bytes=int(obj["source_bytes"]),
        payload_bytes=_payload_bytes(quantized, absmax, code, obj.get("absmax2"), obj.get("code2")), **extra)


def _save_payload_to_cache(path: Path, payload: NF4Payload) -> None:
    """Atomic write (tmp file, then replace): version 1 unless the payload is nested."""
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_name(f"{path.name}.tmp")
    obj = {
        "version": 2 if payload.nested else 1,
        "shape": tuple(payload.shape),
        "dtype": _dtype_name(payload.dtype),
        "blocksize": int(payload.blocksize),
        "quant_type": str(payload.quant_type),
        "source_numel": int(payload.source_numel),
        "source_bytes": int(payload.source_bytes),
        "quantized": payload.quantized.detach().contiguous().cpu(),
        "absmax": payload.absmax.detach().contiguous().cpu(),
        "code": payload.code.detach().contiguous().cpu(),
    }
    if payload.nested:
        obj.update(nested=True, absmax2=payload.absmax2.detach().cpu(), code2=payload.code2.detach().cpu(),
                   offset=payload.offset.detach().cpu(), blocksize2=int(payload.blocksize2))
    torch.save(obj, tmp)
    tmp.replace(path)


# --------------------------------------------------------------------------------
# phase 1: quantize
# --------------------------------------------------------------------------------

def _quantize_param(weight: torch.Tensor, blocksize: int, quant_type: str, compress_statistics: bool,
                    orig_shape: tuple, source_bytes: int, device) -> NF4Payload:
    w = weight.detach().contiguous()
    if w.ndim > 2:  # stacked expert weights [E, A, B] -> [-1, last] (stratum/upload.py:361-366)
        w = w.reshape(-1, w.shape[-1])
    dev = torch.device(device) if device is not None else (
        w.device if w.device.type == "cuda" else torch.device("cuda", torch.cuda.current_device()))
    wd = w.to(dev, non_blocking=True)
    packed, qs = F.quantize_4bit(wd, blocksize=blocksize, compress_statistics=compress_statistics,
                                 quant_type=quant_type)
    torch.cuda.current_stream(dev).synchronize()
    kw = {}
    if qs.nested:
        kw = dict(nested=True, absmax2=_pin_cpu(qs.state2.absmax), code2=_pin_cpu(qs.state2.code),
                  offset=_pin_cpu(qs.offset.reshape(())), blocksize2=int(qs.state2.blocksize))
    pq, pa, pc = _pin_cpu(packed), _pin_cpu(qs.absmax), _pin_cpu(qs.code)
    return NF4Payload(
        quantized=pq, absmax=pa, code=pc, shape=tuple(orig_shape), dtype=qs.dtype, blocksize=int(qs.blocksize),
        quant_type=str(qs.quant_type), source_numel=int(weight.numel()), source_bytes=int(source_bytes),
        payload_bytes=_payload_bytes(pq, pa, pc, kw.get("absmax2"), kw.get("code2")), **kw)


@torch.no_grad()
def prepare_nf4(
    module: nn.Module,
    *,
    min_numel: int = 4096,
    cache_dir: Optional[Path | str] = None,
    verbose: bool = True,
    blocksize: int = 64,
    quant_type: str = "nf4",
    compress_statistics: bool = False,
    device=None,
) -> NF4Stats:
    """Quantize frozen >= 2-D parameters to NF4, attach payloads, drop the originals.

    Reference: stratum/upload.py:305-398 (same selection rules: frozen, ndim
    >= 2, numel >= ``min_numel``, fp16/bf16/fp32; 3-D stacked experts are
    quantized as ``[-1, last]`` and keep their original ``payload.shape``).
    Quantization runs on a CUDA device (``device`` or the current one); the
    reference quantizes on the CPU through bitsandbytes.
    ``compress_statistics=True`` adds 8-bit double quantization of the absmax.
    """
    stats = NF4Stats()
    for name, param in module.named_parameters():
        if param.requires_grad or param.ndim < 2 or param.numel() < min_numel:
            continue
        if param.dtype not in (torch.float16, torch.bfloat16, torch.float32):
            continue
        if hasattr(param, NF4_ATTR):
            payload = cast(NF4Payload, getattr(param, NF4_ATTR))
            stats.tensors += 1
            stats.source_bytes += payload.source_bytes
            stats.payload_bytes += payload.payload_bytes
            continue
        cache_path = _cache_path(Path(cache_dir), name) if cache_dir else None
        payload = (_load_payload_from_cache(cache_path, param, blocksize=blocksize, quant_type=quant_type,
                                            compress_statistics=compress_statistics)
                   if cache_path is not None else None)
        if payload is not None:
            stats.cache_hits += 1
        else:
            if cache_path is not None:
                stats.cache_misses += 1
            payload = _quantize_param(param.data, blocksize, quant_type, compress_statistics, tuple(param.shape),
                                      param.numel() * param.element_size(), device)
            if cache_path is not None:
                _save_payload_to_cache(cache_path, payload)
                stats.cache_writes += 1
        setattr(param, NF4_ATTR, payload)
        param.data = torch.empty(0, dtype=payload.dtype, device=param.device)
        stats.tensors += 1
        stats.source_bytes += payload.source_bytes
        stats.payload_bytes += payload.payload_bytes
    if verbose:
        print(f"  nf4 total: {stats.tensors} tensors, {stats.source_bytes / 1024**3:.2f} GiB -> "
              f"{stats.payload_bytes / 1024**3:.2f} GiB payload (compression {stats.compression:.2f}x, "
              f"cache hits={stats.cache_hits} misses={stats.cache_misses} writes={stats.cache_writes})", flush=True)
    return stats


@torch.no_grad()
def prepare_nf4_from_cache(module: nn.Module, cache_dir: Path | str, *, min_numel: int = 4096,
                           blocksize: int = 64, quant_type: str = "nf4", verbose: bool = True) -> NF4Stats:
    """Attach cached payloads only (no quantization); parameters without a valid
    cache entry are left untouched (reference: stratum/upload.py:1207-1283)."""
    stats = NF4Stats()
    for name, param in module.named_parameters():
        if param.requires_grad or param.ndim < 2 or param.numel() < min_numel or hasattr(param, NF4_ATTR):
            continue
        path = _cache_path(Path(cache_dir), name)
        payload = _load_payload_from_cache(path, param, blocksize=blocksize, quant_type=quant_type)
        if payload is None:
            payload = _load_payload_from_cache(path, param, blocksize=blocksize, quant_type=quant_type,
                                               compress_statistics=True)
        if payload is None:
            stats.cache_misses += 1
            continue
        stats.cache_hits += 1
        setattr(param, NF4_ATTR, payload)
        param.data = torch.empty(0, dtype=payload.dtype, device=param.device)
        stats.tensors += 1
        stats.source_bytes += payload.source_bytes
        stats.payload_bytes += payload.payload_bytes
    if verbose:
        print(f"  nf4 from cache: {stats.tensors} tensors (hits={stats.cache_hits} misses={stats.cache_misses})",
              flush=True)
    return stats


@torch.no_grad()
def prepare_fp16_staged(module: nn.Module, *, min_numel: int = 4096, verbose: bool = True) -> int:
    """Pin frozen params for per-step 16-bit upload (reference: stratum/upload.py:111-160)."""
    count = 0
    for _, param in module.named_parameters():
        if param.requires_grad or param.numel() < min_numel or param.ndim < 2:
            continue
        if hasattr(param, NF4_ATTR) or hasattr(param, FP16_ATTR):
            continue
        if param.dtype not in (torch.float16, torch.bfloat16, torch.float32):
            continue
        payload = FP16StagedPayload(data=_pin_cpu(param.data), shape=tuple(param.shape), dtype=param.dtype,
                                    source_bytes=param.numel() * param.element_size())
        setattr(param, FP16_ATTR, payload)
        param.data = torch.empty(0, dtype=param.dtype, device=param.device)
        count += 1
    if verbose:
        total = sum(getattr(p, FP16_ATTR).source_bytes for p in module.parameters() if hasattr(p, FP16_ATTR))
        print(f"  fp16 staged: {count} tensors, {total / 1024**3:.2f} GiB to upload per step", flush=True)
    return count


@torch.no_grad()
def estimate_module_upload_gib(module: nn.Module) -> float:
    """GB (1e9) a module occupies once materialised (reference: stratum/upload.py:401-422)."""
    total, seen = 0, set()
    for p in module.parameters():
        if id(p) in seen:
            continue
        seen.add(id(p))
        payload = getattr(p, NF4_ATTR, None)
        total += payload.source_bytes if payload is not None else p.numel() * p.element_size()
        if p.grad is not None:
            total += p.grad.numel() * p.grad.element_size()
    for b in module.buffers():
        total += b.numel() * b.element_size()
    return total / 10**9


# --------------------------------------------------------------------------------
# coalesced per-layer arena
# --------------------------------------------------------------------------------

_ALIGN = 256


@dataclass
class LayerArena:
    """All NF4 payload tensors of one module in one pinned buffer (one H2D copy per layer)."""

    host: torch.Tensor                                   # pinned uint8
    slots: dict = field(default_factory=dict)           # (param id, index) -> (offset, nbytes, dtype, shape)

    def views(self, dev_buf: torch.Tensor, pid: int, n: int) -> list[torch.Tensor]:
        out = []
        for i in range(n):
            off, nbytes, dtype, shape = self.slots[(pid, i)]
            out.append(dev_buf[off:off + nbytes].view(dtype).view(shape))
        return out


def build_layer_arena(module: nn.Module) -> Optional[LayerArena]:
    """Coalesce every NF4 payload under ``module`` into one pinned arena (256-B aligned slots)."""
    items = []
    for p in module.parameters():
        payload = getattr(p, NF4_ATTR, None)
        if payload is not None:
            items.append((p, payload.host_tensors()))
    if not items:
        return None
    offset = 0
    slots = {}
    for p, ts in items:
        for i, t in enumerate(ts):
            nbytes = t.numel() * t.element_size()
            slots[(id(p), i)] = (offset, nbytes, t.dtype, tuple(t.shape))
            offset += (nbytes + _ALIGN - 1) // _ALIGN * _ALIGN
    host = torch.empty(max(offset, _ALIGN), dtype=torch.uint8, pin_memory=torch.cuda.is_available())
    for p, ts in items:
        for i, t in enumerate(ts):
            off, nbytes, _, _ = slots[(id(p), i)]
            host[off:off + nbytes].copy_(t.contiguous().view(-1).view(torch.uint8))
    arena = LayerArena(host=host, slots=slots)
    setattr(module, ARENA_ATTR, arena)
    return arena


# --------------------------------------------------------------------------------
# phase 2: upload / free
# --------------------------------------------------------------------------------

def _device_state(payload: NF4Payload, dev_tensors: list[torch.Tensor]):
    a, c = dev_tensors[1], dev_tensors[2]
    if payload.nested:
        return payload.quant_state(absmax=a, code=c, absmax2=dev_tensors[3], code2=dev_tensors[4],
                                   offset=dev_tensors[5].reshape(()))
    return payload.quant_state(absmax=a, code=c)


def _materialize(param, payload: NF4Payload, dev_tensors: list[torch.Tensor], owner, pname, device,
                 pending: Optional[list] = None) -> None:
    """Make an uploaded payload usable: fused owner -> NF4 state, else dequantize into
    param.data -- right away, or (with ``pending``) queued for one batched launch
    per layer by :func:`_flush_dequant`."""
    q = dev_tensors[0]
    qs = _device_state(payload, dev_tensors)
    fused = _fused_owner(owner, pname)
    if fused is not None:
        fused.load_device_state(q, qs)
        return
    if pending is not None:
        pending.append((param, q, qs, owner, pname))
        return
    _replace_param_data(param, F.dequantize_4bit(q, qs).contiguous(), owner=owner, pname=pname)


def _flush_dequant(pending: list) -> None:
    """Dequantize queued payloads, one batched launch per (blocksize, dtype) group."""
    groups: dict = {}
    for item in pending:
        qs = item[2]
        groups.setdefault((int(qs.blocksize), qs.dtype), []).append(item)
    for (_, dtype), items in groups.items():
        outs = F.dequantize_4bit_many([(q, qs) for _, q, qs, _, _ in items], out_dtype=dtype)
        for (param, _, _, owner, pname), out in zip(items, outs):
            _replace_param_data(param, out, owner=owner, pname=pname)
    pending.clear()


def _device(device_id) -> torch.device:
    return device_id if isinstance(device_id, torch.device) else torch.device(f"cuda:{int(device_id)}")


def _is_resident(param, payload, owner, pname, device) -> bool:
    fused = _fused_owner(owner, pname)
    if fused is not None:
        return fused.device_state_on(device)
    return param.data.numel() > 0 and param.data.device == device


DEFAULT_CHUNK_UPLOAD_BYTES = 64 << 20


@torch.no_grad()
def copy_tensor_chunked(src: torch.Tensor, dst: torch.Tensor, *, chunk_bytes: int = DEFAULT_CHUNK_UPLOAD_BYTES,
                        non_blocking: bool = False) -> int:
    """Copy ``src`` into ``dst`` (same shape and dtype) in flat chunks of at most
    ``chunk_bytes``; returns the number of copies issued (the reference's
    stratum/layer_transfer.py:59-89 contract, used for FP16-staged weights)."""
    if src.shape != dst.shape:
        raise ValueError(f"shape mismatch: {tuple(src.shape)} != {tuple(dst.shape)}")
    if src.dtype != dst.dtype:
        raise ValueError(f"dtype mismatch: {src.dtype} != {dst.dtype}")
    n = src.numel()
    if n == 0:
        return 0
    if not dst.is_contiguous():
        dst.copy_(src, non_blocking=non_blocking)
        return 1
    a = src.detach().contiguous().view(-1)
    b = dst.view(-1)
    step = max(1, int(chunk_bytes) // max(1, src.element_size()))
    chunks = 0
    for lo in range(0, n, step):
        hi = min(n, lo + step)
        b[lo:hi].copy_(a[lo:hi], non_blocking=non_blocking)
        chunks += 1
    return chunks


@torch.no_grad()
def ensure_weights(module: nn.Module, device_id: int) -> int:
    """Upload NF4 payloads (and move other params/buffers) for *module* to ``cuda:device_id``.

    Reference: stratum/upload.py:969-1069.  Issues its copies and kernels on
    the current stream.  Returns the number of tensors made resident.
    """
    device = _device(device_id)
    owner_map = _build_param_owner_map(module)
    arena: Optional[LayerArena] = getattr(module, ARENA_ATTR, None)
    arena_dev = None
    tensors = 0
    pending: list = []  # compat-mode payloads, dequantized together after the loop
    for name, param in module.named_parameters():
        owner, pname = owner_map.get(id(param), (None, None))
        fp16 = getattr(param, FP16_ATTR, None)
        if fp16 is not None:
            if param.data.numel() > 0 and param.data.device == device:
                continue
            dst = torch.empty(fp16.shape, dtype=fp16.dtype, device=device)
            copy_tensor_chunked(fp16.data, dst, non_blocking=True)
            param.data = dst
            tensors += 1
            continue
        payload = getattr(param, NF4_ATTR, None)
        if payload is None:
            if param.data.numel() > 0 and param.data.device != device:
                if param.requires_grad:
                    raise RuntimeError(
                        f"trainable shared parameter {name!r} is on {param.data.device}, but module is running on "
                        f"{device}; Stratum cannot safely move trainable parameters between stages")
                param.data = param.data.to(device, non_blocking=True)
                tensors += 1
            continue
        if _is_resident(param, payload, owner, pname, device):
            continue
        if device.type != "cuda":
            raise RuntimeError(f"ensure_weights: NF4 payloads need a CUDA device, got {device}")
        if arena is not None:
            if arena_dev is None:
                arena_dev = torch.empty(arena.host.numel(), dtype=torch.uint8, device=device)
                arena_dev.copy_(arena.host, non_blocking=True)
            dev_tensors = arena.views(arena_dev, id(param), len(payload.host_tensors()))
        else:
            dev_tensors = [t.to(device, non_blocking=True) for t in payload.host_tensors()]
        _materialize(param, payload, dev_tensors, owner, pname, device, pending)
        tensors += 1
    if pending:
        _flush_dequant(pending)
    for buf in module.buffers():
        if buf.device != device and buf.device.type != "meta":
            buf.data = buf.data.to(device, non_blocking=True)
            tensors += 1
    return tensors


@dataclass
class _PrefetchEntry:
    param: nn.Parameter
    payload: NF4Payload
    tensors: list
    owner: Optional[nn.Module] = None
    pname: Optional[str] = None


@dataclass
class NF4Prefetch:
    """Pending asynchronous NF4 upload for one module (reference: stratum/upload.py:163-228).

    ``finalize()`` makes the current stream wait for the copy event and then
    materialises every entry (fused state or dequantized ``param.data``).
    """

    entries: list
    device: torch.device
    stream: Optional["torch.cuda.Stream"] = None
    event: Optional["torch.cuda.Event"] = None
    arena_buffer: Optional[torch.Tensor] = None

    def finalize(self) -> int:
        if not self.entries:
            return 0
        if self.device.type != "cuda" or not torch.cuda.is_available():
            raise RuntimeError(f"CUDA is not available for NF4 prefetch finalize on {self.device}")
        current = torch.cuda.current_stream(device=self.device)
        if self.event is not None:
            current.wait_event(self.event)
        n = 0
        with torch.cuda.device(self.device), torch.no_grad():
            if self.arena_buffer is not None:
                self.arena_buffer.record_stream(current)
            pending: list = []
            for e in self.entries:
                for t in e.tensors:
                    t.record_stream(current)
                if _is_resident(e.param, e.payload, e.owner, e.pname, self.device):
                    continue
                _materialize(e.param, e.payload, e.tensors, e.owner, e.pname, self.device, pending)
                n += 1
            if pending:
                _flush_dequant(pending)
        self.entries = []
        return n

    def wait(self) -> int:
        return self.finalize()


@torch.no_grad()
def prefetch_weights(module: nn.Module, device_id: int, stream: Optional["torch.cuda.Stream"] = None) -> NF4Prefetch:
    """Start the H2D copies of *module*'s NF4 payloads on a side stream (reference:
    stratum/upload.py:1072-1125).  Nothing is mutated until :meth:`NF4Prefetch.finalize`."""
    device = _device(device_id)
    owner_map = _build_param_owner_map(module)
    todo = []
    for _, param in module.named_parameters():
        payload = getattr(param, NF4_ATTR, None)
        if payload is None:
            continue
        owner, pname = owner_map.get(id(param), (None, None))
        if _is_resident(param, payload, owner, pname, device):
            continue
        todo.append((param, payload, owner, pname))
    if not todo:
        return NF4Prefetch([], device)
    if device.type != "cuda" or not torch.cuda.is_available():
        raise RuntimeError(f"CUDA is not available for NF4 prefetch to {device}")
    stream = stream or torch.cuda.Stream(device=device)
    arena: Optional[LayerArena] = getattr(module, ARENA_ATTR, None)
    entries = []
    buf = None
    with torch.cuda.device(device), torch.cuda.stream(stream):
        if arena is not None:
            buf = torch.empty(arena.host.numel(), dtype=torch.uint8, device=device)
            buf.copy_(arena.host, non_blocking=True)
        for param, payload, owner, pname in todo:
            n = len(payload.host_tensors())
            ts = (arena.views(buf, id(param), n) if arena is not None
                  else [t.to(device, non_blocking=True) for t in payload.host_tensors()])
            entries.append(_PrefetchEntry(param, payload, ts, owner, pname))
        event = torch.cuda.Event()
        stream.record_event(event)
    return NF4Prefetch(entries, device=device, stream=stream, event=event, arena_buffer=buf)


@torch.no_grad()
def ensure_prefetched_weights(module: nn.Module, device_id: int, prefetch: Optional[NF4Prefetch]) -> int:
    """Finalize a matching prefetch, then ensure the rest (reference: stratum/upload.py:1128-1141)."""
    if prefetch is None:
        return ensure_weights(module, device_id)
    if prefetch.device != _device(device_id):
        raise ValueError(f"prefetch device {prefetch.device} does not match cuda:{device_id}")
    return prefetch.finalize() + ensure_weights(module, device_id)


@torch.no_grad()
def free_weights(module: nn.Module) -> int:
    """Drop the device copies of NF4 / FP16-staged params (reference: stratum/upload.py:1144-1159)."""
    owner_map = _build_param_owner_map(module)
    tensors = 0
    for _, param in module.named_parameters():
        if not hasattr(param, NF4_ATTR) and not hasattr(param, FP16_ATTR):
            continue
        owner, pname = owner_map.get(id(param), (None, None))
        fused = _fused_owner(owner, pname) if hasattr(param, NF4_ATTR) else None
        if fused is not None:
            if fused.drop_device_state():
                tensors += 1
            continue
        if param.data.numel() == 0:
            continue
        param.data = torch.empty(0, dtype=param.dtype, device=param.device)
        tensors += 1
    return tensors


@torch.no_grad()
def upload_stream(module: nn.Module, device_id: int, *, verbose: bool = True) -> int:
    """Synchronous permanent upload of a whole module (reference: stratum/upload.py:907-966)."""
    t0 = time.time()
    n = ensure_weights(module, device_id)
    torch.cuda.current_stream(_device(device_id)).synchronize()
    if verbose:
        print(f"  device {device_id}: {n} tensors in {time.time() - t0:.1f}s", flush=True)
    return n


@torch.no_grad()
def snapshot_module_buffers(module: nn.Module) -> dict[str, torch.Tensor]:
    """Host copies of every non-empty buffer, taken before a group's forward so its
    recompute can start from the same buffer state (stratum/upload.py:1162-1180).
    Empty buffers (released weights, placeholders) are left out; the copies live in
    host memory whatever the buffer's device, so a snapshot costs no device memory."""
    snap: dict[str, torch.Tensor] = {}
    for name, b in module.named_buffers():
        if b.numel() > 0:
            snap[name] = b.detach().to("cpu").clone()
    return snap


@torch.no_grad()
def restore_module_buffers(module: nn.Module, snapshot: dict[str, torch.Tensor]) -> int:
    """Copy a snapshot back into the module's buffers on their current devices
    (stratum/upload.py:1183-1203); returns the number restored."""
    if not snapshot:
        return 0
    bufs = dict(module.named_buffers())
    n = 0
    for name, saved in snapshot.items():
        b = bufs.get(name)
        if b is None:
            continue
        b.data.copy_(saved.to(b.device))
        n += 1
    return n


# --------------------------------------------------------------------------------
# fused mode: nn.Linear -> NF4Linear
# --------------------------------------------------------------------------------

@torch.no_grad()
def to_nf4_linear(module: nn.Module, *, lora_r: int = 0, lora_alpha: float = 16.0,
                  lora_dtype: torch.dtype = torch.bfloat16, target: Optional[callable] = None,
                  lora_device=None) -> int:
    """Replace every ``nn.Linear`` child whose frozen weight carries an NF4 payload
    by a streamed :class:`NF4Linear` (fused mode).  With ``lora_r > 0`` each gets a
    PEFT-style adapter.  Returns the number of layers converted."""
    from .nf4_linear import NF4Linear

    count = 0
    for parent_name, parent in list(module.named_modules()):
        for cname, child in list(parent.named_children()):
            if not isinstance(child, nn.Linear):
                continue
            payload = getattr(child.weight, NF4_ATTR, None)
            if payload is None or len(payload.shape) != 2:
                continue
            full = f"{parent_name}.{cname}" if parent_name else cname
            if target is not None and not target(full):
                continue
            new = NF4Linear.streamed_from(child.weight, payload, bias=child.bias)
            if lora_r > 0:
                new.attach_lora(lora_r, lora_alpha, dtype=lora_dtype,
                                device=lora_device if lora_device is not None else torch.device("cpu"))
            setattr(parent, cname, new)
            count += 1
    return count


@torch.no_grad()
def to_nf4_experts(module: nn.Module) -> int:
    """Replace every routed-experts module whose 3-D ``gate_up_proj`` / ``down_proj``
    carry NF4 payloads (HF ``Qwen3MoeExperts`` after :func:`prepare_nf4`, staged as
    ``[-1, last]`` like stratum/upload.py:361-366) by a streamed
    :class:`~stratum_b200.experts.NF4Experts` fed by ``ensure_weights`` and consumed
    by the grouped NF4 kernels.  Returns the number of modules converted."""
    from .experts import NF4Experts

    count = 0
    for parent_name, parent in list(module.named_modules()):
        for cname, child in list(parent.named_children()):
            gu = getattr(child, "gate_up_proj", None)
            dn = getattr(child, "down_proj", None)
            if not isinstance(gu, nn.Parameter) or not isinstance(dn, nn.Parameter):
                continue
            gp, dp = getattr(gu, NF4_ATTR, None), getattr(dn, NF4_ATTR, None)
            if gp is None or dp is None or len(gp.shape) != 3:
                continue
            act = getattr(child, "act_fn", None)
            if act is not None and not isinstance(act, nn.SiLU) and type(act).__name__ not in ("SiLU", "SiLUActivation"):
                continue
            setattr(parent, cname, NF4Experts.streamed_from(gu, gp, dn, dp))
            count += 1
    return count


# --------------------------------------------------------------------------------
# streaming load + quantize (checkpoint -> NF4 payloads, one tensor at a time)
# --------------------------------------------------------------------------------

def _ckpt_key_fn(module: nn.Module):
    """``keys(param_name) -> [checkpoint key candidates]`` for a pipeline module:
    the name itself, with PEFT's ``.base_layer.`` and wrappers' ``.inner.`` /
    ``.layer.`` removed, with a ``model.`` prefix, and wrapped decoder layers
    (modules with ``idx`` and ``layer``) mapped to ``model.layers.{idx}.``
    (the reference's rule, stratum/upload.py:425-473)."""
    import re

    layer_prefixes = []
    for mname, sub in module.named_modules():
        idx = getattr(sub, "idx", None)
        if isinstance(idx, int) and hasattr(sub, "layer"):
            layer_prefixes.append((f"{mname}.layer." if mname else "layer.", f"model.layers.{idx}."))

    def no_base(n: str) -> str:
        return n.replace(".base_layer.", ".")

    def keys(pname: str) -> list[str]:
        out: list[str] = []
        pname = _canonical_param_name(pname)

        def add(name: str) -> None:
            variants = [name]
            if ".inner." in name:
                variants.append(name.replace(".inner.", "."))
            for v in variants:
                stripped = re.sub(r"\.layer\.(?!layer)", ".", v)
                for k in (v, no_base(v), stripped, no_base(stripped)):
                    out.append(k)
                for k in (v, no_base(v), stripped, no_base(stripped)):
                    out.append(f"model.{k}")

        add(pname)
        if pname == "lm_head.weight":  # tied embeddings
            add("model.embed_tokens.weight")
            add("embed_tokens.weight")
        for prefix, global_prefix in layer_prefixes:
            if pname.startswith(prefix):
                add(global_prefix + pname[len(prefix):])
        return list(dict.fromkeys(out))

    return keys


def _load_stacked_experts(handle, keys: set, pname: str, param, key_fn):
    """A 3-D expert parameter stacked from per-expert checkpoint tensors: the
    reference's LFM2 layout (``...feed_forward.experts.{e}.w1/w3/w2.weight``,
    stratum/upload.py:476-532) and, as an extension, HF Qwen3-MoE's
    (``...mlp.experts.{e}.gate_proj/up_proj/down_proj.weight``)."""
    if param.ndim != 3:
        return None
    E = int(param.shape[0])
    layouts = (
        (".feed_forward.experts.gate_up_proj", ".feed_forward.experts", ("w1", "w3")),
        (".feed_forward.experts.down_proj", ".feed_forward.experts", ("w2",)),
        (".mlp.experts.gate_up_proj", ".mlp.experts", ("gate_proj", "up_proj")),
        (".mlp.experts.down_proj", ".mlp.experts", ("down_proj",)),
    )
    for cand in key_fn(pname):
        for suffix, base_sfx, parts in layouts:
            if not cand.endswith(suffix):
                continue
            base = cand[: -len(suffix)] + base_sfx
            need = [f"{base}.{e}.{p}.weight" for e in range(E) for p in parts]
            if not all(k in keys for k in need):
                continue
            rows = []
            for e in range(E):
                ts = [handle.get_tensor(f"{base}.{e}.{p}.weight") for p in parts]
                rows.append(torch.cat(ts, dim=0) if len(ts) > 1 else ts[0])
            return torch.stack(rows, dim=0)
    return None


@torch.no_grad()
def stream_load_and_quantize_module(
    module: nn.Module,
    hf_model_name: str,
    *,
    min_numel: int = 4096,
    cache_dir: Optional[Path | str] = None,
    blocksize: int = 64,
    quant_type: str = "nf4",
    verbose: bool = False,
    compress_statistics: bool = False,
    device=None,
) -> Optional[NF4Stats]:
    """Load and NF4-quantize a meta-device module in one streaming pass
    (reference: stratum/upload.py:670-904).  For each frozen parameter still on
    the meta device (or empty): an NF4-eligible one is served from the payload
    cache if present, else its checkpoint tensor is read, quantized on the GPU
    and dropped before the next one; other parameters get their checkpoint
    tensor.  Peak host memory is the payloads so far plus one tensor.

    ``hf_model_name`` is a local checkpoint directory or a cached hub id
    (``model.safetensors`` or a sharded ``model.safetensors.index.json``).
    Returns ``NF4Stats``, or ``None`` when a parameter has no checkpoint key or
    a shard is missing (the reference's contract).
    """
    from safetensors import safe_open

    def locate(fname: str) -> Optional[Path]:
        local = Path(hf_model_name) / fname
        if local.exists():
            return local
        try:
            from transformers.utils.hub import cached_file

            p = cached_file(hf_model_name, fname, cache_dir=None)
            return Path(p) if p and Path(p).exists() else None
        except Exception:
            return None

    cache_root = Path(cache_dir) if cache_dir else None
    owner_map = _build_param_owner_map(module)
    key_fn = _ckpt_key_fn(module)

    def eligible(p) -> bool:
        return p.ndim >= 2 and p.numel() >= min_numel and p.dtype in (torch.float16, torch.bfloat16, torch.float32)

    stats = NF4Stats()
    needed = []
    for n, p in module.named_parameters():
        if hasattr(p, NF4_ATTR):
            pl = cast(NF4Payload, getattr(p, NF4_ATTR))
            stats.tensors += 1
            stats.source_bytes += pl.source_bytes
            stats.payload_bytes += pl.payload_bytes
            continue
        if p.requires_grad or (p.device.type != "meta" and p.data.numel() != 0):
            continue
        needed.append((n, p))

    def attach(name, param, payload) -> None:
        setattr(param, NF4_ATTR, payload)
        owner, pname = owner_map.get(id(param), (None, None))
        _replace_param_data(param, torch.empty(0, dtype=payload.dtype, device="cpu"), owner=owner, pname=pname)
        stats.tensors += 1
        stats.source_bytes += payload.source_bytes
        stats.payload_bytes += payload.payload_bytes

    def from_cache(name, param) -> bool:
        if cache_root is None:
            return False
        payload = _load_payload_from_cache(_cache_path(cache_root, name), param, blocksize=blocksize,
                                           quant_type=quant_type, compress_statistics=compress_statistics)
        if payload is None:
            return False
        attach(name, param, payload)
        stats.cache_hits += 1
        return True

    def consume(name, param, t) -> bool:
        t = t.to(device="cpu", dtype=param.dtype)
        if eligible(param):
            payload = _quantize_param(t, blocksize, quant_type, compress_statistics, tuple(param.shape),
                                      param.numel() * param.element_size(), device)
            if cache_root is not None:
                _save_payload_to_cache(_cache_path(cache_root, name), payload)
                stats.cache_writes += 1
                stats.cache_misses += 1
            attach(name, param, payload)
            return True
        owner, pname = owner_map.get(id(param), (None, None))
        try:
            _replace_param_data(param, t, owner=owner, pname=pname)
        except (RuntimeError, TypeError):
            return False
        return True

    if needed:
        index = locate("model.safetensors.index.json")
        if index is not None:
            import json

            weight_map = json.loads(index.read_text())["weight_map"]
            todo = []
            for n, p in needed:
                if eligible(p) and from_cache(n, p):
                    continue
                ck = next((k for k in key_fn(n) if k in weight_map), None)
                if ck is None:
                    if verbose:
                        print(f"  stream_nf4: no checkpoint key for {n}", flush=True)
                    return None
                todo.append((n, p, ck))
            by_shard: dict = {}
            for n, p, ck in todo:
                by_shard.setdefault(weight_map[ck], []).append((n, p, ck))
            for shard, items in by_shard.items():
                sp = index.parent / shard
                if not sp.exists():
                    return None
                with safe_open(str(sp), framework="pt") as f:
                    for n, p, ck in items:
                        if not consume(n, p, f.get_tensor(ck)):
                            return None
        else:
            single = locate("model.safetensors")
            if single is None:
                return None
            with safe_open(str(single), framework="pt") as f:
                all_keys = set(f.keys())
                for n, p in needed:
                    if eligible(p) and from_cache(n, p):
                        continue
                    ck = next((k for k in key_fn(n) if k in all_keys), None)
                    t = f.get_tensor(ck) if ck is not None else _load_stacked_experts(f, all_keys, n, p, key_fn)
                    if t is None:
                        if verbose:
                            print(f"  stream_nf4: no checkpoint key for {n}", flush=True)
                        return None
                    if not consume(n, p, t):
                        return None
    if verbose:
        print(f"  nf4 total: {stats.tensors} tensors, {stats.source_bytes / 1024**3:.2f} GiB -> "
              f"{stats.payload_bytes / 1024**3:.2f} GiB payload (cache hits={stats.cache_hits} "
              f"misses={stats.cache_misses} writes={stats.cache_writes})", flush=True)
    return stats
