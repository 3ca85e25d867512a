"""GPU tests of the streaming contract: the golden fixtures reproduced by the GPU
quantizer, compat mode (dequantize into param.data), fused mode (NF4Linear fed
by ensure_weights), prefetch, the coalesced per-layer arena, double quant, and
DeviceStage's per-layer upload overlap."""

import json
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.nn as nn

from oracle import nf4_oracle as O
from oracle.nf4_oracle import relative_error
from stratum_b200 import functional as F
from stratum_b200 import upload
from stratum_b200.nf4_linear import NF4Linear
from stratum_b200.stage import DeviceStage
from stratum_b200.upload import NF4_ATTR

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def test_golden_fixtures_reproduced_by_gpu_quantizer():
    manifest = json.loads((GOLDEN / "manifest.json").read_text())
    inputs = torch.load(GOLDEN / "nf4_inputs.pt")
    for name in manifest["quantized_params"]:
        t = inputs[name]
        param = nn.Parameter(t.clone(), requires_grad=False)
        fixture = upload._load_payload_from_cache(upload._cache_path(GOLDEN / "nf4_cache_v1", name), param,
                                                  blocksize=64, quant_type="nf4")
        w = t.reshape(-1, t.shape[-1]) if t.ndim > 2 else t
        packed, qs = F.quantize_4bit(w.cuda())
        assert torch.equal(packed.cpu().reshape(-1), fixture.quantized.reshape(-1)), name
        assert torch.equal(qs.absmax.cpu(), fixture.absmax), name


def _model(dtype=torch.float16, seed=0):
    g = torch.Generator().manual_seed(seed)
    m = nn.Sequential(nn.Linear(256, 512, bias=True), nn.Linear(512, 128, bias=False))
    with torch.no_grad():
        for lin in m:
            lin.weight.copy_(torch.randn(lin.weight.shape, generator=g) * 0.02)
            if lin.bias is not None:
                lin.bias.copy_(torch.randn(lin.bias.shape, generator=g) * 0.1)
    m = m.to(dtype)
    for p in m.parameters():
        p.requires_grad_(False)
    return m


def test_compat_mode_dequantizes_into_param_data():
    m = _model()
    originals = {n: p.data.clone() for n, p in m.named_parameters()}
    stats = upload.prepare_nf4(m, min_numel=4096, verbose=False)
    assert stats.tensors == 2 and stats.compression > 3.0
    for name, p in m.named_parameters():
        payload = getattr(p, NF4_ATTR, None)
        if payload is not None:
            assert p.data.numel() == 0 and payload.quantized.is_pinned()
    n = upload.ensure_weights(m, 0)
    torch.cuda.synchronize()
    assert n >= 2
    for name, p in m.named_parameters():
        if hasattr(p, NF4_ATTR):
            ref = O.dequantize_nf4(*O.quantize_nf4(originals[name], 64), originals[name].numel(), 64)
            assert p.data.device.type == "cuda" and p.data.shape == originals[name].shape
            assert np.array_equal(p.data.cpu().numpy().view(np.uint16).reshape(-1), ref.view(np.uint16))
    assert upload.ensure_weights(m, 0) == 0  # already resident
    assert upload.free_weights(m) == 2
    assert upload.ensure_weights(m, 0) == 2


@pytest.mark.parametrize("arena", [False, True])
@pytest.mark.parametrize("dq", [False, True])
def test_fused_mode_streamed_nf4linear(arena, dq):
    m = _model(torch.bfloat16, seed=1)
    ref_w = [lin.weight.data.clone() for lin in m]
    ref_b = m[0].bias.data.clone()
    upload.prepare_nf4(m, min_numel=4096, verbose=False, compress_statistics=dq)
    assert upload.to_nf4_linear(m, lora_r=8, lora_alpha=16, lora_device="cuda") == 2
    assert isinstance(m[0], NF4Linear) and m[0].streamed
    m[0].bias.data = m[0].bias.data.cuda()
    if arena:
        assert upload.build_layer_arena(m) is not None
    x = torch.randn(64, 256, device="cuda").to(torch.bfloat16)
    with pytest.raises(RuntimeError, match="not resident"):
        m(x)
    upload.ensure_weights(m, 0)
    y = m(x)
    # reference path: dequantized weights + F.linear (LoRA B starts at zero -> no contribution)
    h = torch.nn.functional.linear(x, m[0].weight_dequantized.to(torch.bfloat16), ref_b.cuda())
    y_ref = torch.nn.functional.linear(h, m[1].weight_dequantized.to(torch.bfloat16))
    assert relative_error(y.float(), y_ref.float()) < 1e-2
    assert upload.free_weights(m) == 2 and m[0].quantized is None
    pf = upload.prefetch_weights(m, 0)
    assert len(pf.entries) == 2 and pf.event is not None
    assert upload.ensure_prefetched_weights(m, 0, pf) >= 2
    y2 = m(x)
    assert torch.equal(y, y2)
    # gradients reach the adapters through the fused kernels
    y2.float().sum().backward()
    assert m[0].lora_A.grad is not None and m[1].lora_B.grad is not None
    del ref_w


class _Layer(nn.Module):
    def __init__(self, lin):
        super().__init__()
        self.lin = lin

    def forward(self, data):
        hidden, *rest = data
        return (torch.relu(self.lin(hidden)), *rest)


def test_device_stage_streams_layers_with_overlap():
    torch.manual_seed(0)
    layers = []
    for _ in range(4):
        lin = nn.Linear(256, 256, bias=False).to(torch.bfloat16)
        lin.weight.data.mul_(0.1)
        lin.weight.requires_grad_(False)
        layers.append(_Layer(lin))
    stage = DeviceStage(layers, device_id=0)
    upload.prepare_nf4(stage, min_numel=4096, verbose=False)
    upload.to_nf4_linear(stage)
    for layer in stage.layers:
        upload.build_layer_arena(layer)
    x = torch.randn(128, 256, device="cuda").to(torch.bfloat16)
    stream = torch.cuda.Stream()
    out = stage.forward_range((x, None), param_stream=stream)[0]
    eager = x
    for layer in stage.layers:
        eager = torch.relu(torch.nn.functional.linear(eager, layer.lin.weight_dequantized.to(torch.bfloat16)))
    torch.cuda.synchronize()
    assert relative_error(out.float(), eager.float()) < 1e-2
    upload.free_weights(stage)
    assert all(layer.lin.quantized is None for layer in stage.layers)


def test_stream_load_matches_prepare_nf4(tmp_path):
    """Checkpoint -> stream_load_and_quantize_module gives the same payload bytes as
    loading the tensor and running prepare_nf4 on it (both quantize on the GPU)."""
    from safetensors.torch import save_file

    g = torch.Generator().manual_seed(5)
    w = (torch.randn(512, 256, generator=g) * 0.02).half()
    save_file({"model.proj.weight": w}, str(tmp_path / "model.safetensors"))
    with torch.device("meta"):
        m = torch.nn.Module()
        m.proj = torch.nn.Linear(256, 512, bias=False, dtype=torch.float16)
    m.requires_grad_(False)
    stats = upload.stream_load_and_quantize_module(m, str(tmp_path))
    assert stats is not None and stats.tensors == 1
    ref = torch.nn.Module()
    ref.proj = torch.nn.Linear(256, 512, bias=False, dtype=torch.float16)
    ref.requires_grad_(False)
    ref.proj.weight.data.copy_(w)
    upload.prepare_nf4(ref, verbose=False)
    a, b = getattr(m.proj.weight, upload.NF4_ATTR), getattr(ref.proj.weight, upload.NF4_ATTR)
    assert torch.equal(a.quantized, b.quantized) and torch.equal(a.absmax, b.absmax)
