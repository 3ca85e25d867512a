"""Host-side tests of the streaming contract (CPU, no GPU): the reference's
test_upload.py / test_assign.py / stage semantics, plus the golden cache files
written by the reference's own prepare_nf4 (tests/golden/make_golden.py)."""

import json
from pathlib import Path
from unittest import mock

import numpy as np
import pytest
import torch
import torch.nn as nn

from oracle import nf4_oracle as O
from stratum_b200 import upload
from stratum_b200.assign import assign_layers_to_devices, strata
from stratum_b200.functional import QuantState
from stratum_b200.stage import DeviceStage
from stratum_b200.upload import NF4_ATTR, NF4Payload

GOLDEN = Path(__file__).resolve().parent / "golden"


# ------------------------------------------------------------------ golden --

def test_golden_cache_files_load_and_match_the_oracle():
    """Cache files written by the reference's prepare_nf4 load through our loader, keep
    the reference metadata, and hold exactly the oracle's codec output for the inputs."""
    manifest = json.loads((GOLDEN / "manifest.json").read_text())
    inputs = torch.load(GOLDEN / "nf4_inputs.pt")
    assert manifest["quantized_params"] == ["gate_up_proj", "o_proj.weight", "q_proj.weight"]
    for name in manifest["quantized_params"]:
        t = inputs[name]
        param = nn.Parameter(t.clone(), requires_grad=False)
        path = upload._cache_path(GOLDEN / "nf4_cache_v1", name)
        assert path.name in manifest["files"]
        payload = upload._load_payload_from_cache(path, param, blocksize=64, quant_type="nf4")
        assert payload is not None, name
        assert payload.shape == tuple(t.shape) and payload.dtype == torch.float16
        assert payload.source_numel == t.numel() and payload.source_bytes == t.numel() * 2
        packed, absmax = O.quantize_nf4(t, 64)  # 3-D reshape to [-1, last] does not change the flat order
        assert np.array_equal(payload.quantized.numpy().reshape(-1), packed)
        assert np.array_equal(payload.absmax.numpy(), absmax)
        assert np.array_equal(payload.code.numpy(), O.NF4_LEVELS)
    # mismatching metadata is rejected exactly like the reference (None, not an error)
    wrong = nn.Parameter(inputs["q_proj.weight"].float(), requires_grad=False)
    path = upload._cache_path(GOLDEN / "nf4_cache_v1", "q_proj.weight")
    assert upload._load_payload_from_cache(path, wrong, blocksize=64, quant_type="nf4") is None
    assert upload._load_payload_from_cache(path, nn.Parameter(inputs["q_proj.weight"], requires_grad=False),
                                           blocksize=128, quant_type="nf4") is None


# ------------------------------------------------------------ prepare_nf4 --

def _fake_quantizer():
    calls = []

    def fake(weight, blocksize, quant_type, compress_statistics, orig_shape, source_bytes, device):
        calls.append(tuple(weight.shape))
        w = weight.reshape(-1, weight.shape[-1]) if weight.ndim > 2 else weight
        packed, absmax = O.quantize_nf4(w, blocksize)
        pq, pa = torch.from_numpy(packed).reshape(-1, 1), torch.from_numpy(absmax)
        pc = torch.from_numpy(O.NF4_LEVELS.copy())
        return NF4Payload(pq, pa, pc, tuple(orig_shape), weight.dtype, blocksize, quant_type, weight.numel(),
                          source_bytes, upload._payload_bytes(pq, pa, pc))

    return fake, calls


def _run_prepare(module, **kw):
    fake, calls = _fake_quantizer()
    with mock.patch.object(upload, "_quantize_param", side_effect=fake):
        stats = upload.prepare_nf4(module, verbose=False, **kw)
    return stats, calls


def test_prepare_nf4_stages_2d_frozen_param():
    param = nn.Parameter(torch.randn(8, 8, dtype=torch.float16), requires_grad=False)
    module = nn.Module()
    module.register_parameter("weight", param)
    stats, calls = _run_prepare(module, min_numel=8)
    assert stats.tensors == 1 and hasattr(param, NF4_ATTR)
    assert getattr(param, NF4_ATTR).shape == (8, 8)
    assert param.data.numel() == 0
    assert (8, 8) in calls


def test_prepare_nf4_stages_3d_stacked_param_with_original_shape():
    param = nn.Parameter(torch.randn(4, 16, 8, dtype=torch.float16), requires_grad=False)
    module = nn.Module()
    module.register_parameter("gate_up_proj", param)
    stats, calls = _run_prepare(module, min_numel=8)
    assert stats.tensors == 1
    assert getattr(param, NF4_ATTR).shape == (4, 16, 8)


def test_prepare_nf4_skips_trainable_small_and_1d():
    module = nn.Module()
    module.register_parameter("trainable", nn.Parameter(torch.randn(64, 64, dtype=torch.float16)))
    module.register_parameter("small", nn.Parameter(torch.randn(8, 8, dtype=torch.float16), requires_grad=False))
    module.register_parameter("vec", nn.Parameter(torch.randn(8192, dtype=torch.float16), requires_grad=False))
    module.register_parameter("ints", nn.Parameter(torch.ones(64, 64, dtype=torch.int32), requires_grad=False))
    stats, calls = _run_prepare(module, min_numel=4096)
    assert stats.tensors == 0 and calls == []


def test_prepare_nf4_cache_roundtrip(tmp_path):
    module = nn.Module()
    module.register_parameter("w", nn.Parameter(torch.randn(64, 128, dtype=torch.float16), requires_grad=False))
    ref = module.w.data.clone()
    s1, c1 = _run_prepare(module, min_numel=8, cache_dir=tmp_path)
    assert (s1.cache_misses, s1.cache_writes, s1.cache_hits) == (1, 1, 0)
    m2 = nn.Module()
    m2.register_parameter("w", nn.Parameter(ref.clone(), requires_grad=False))
    s2, c2 = _run_prepare(m2, min_numel=8, cache_dir=tmp_path)
    assert (s2.cache_hits, s2.cache_misses) == (1, 0) and c2 == []
    p1, p2 = getattr(module.w, NF4_ATTR), getattr(m2.w, NF4_ATTR)
    assert torch.equal(p1.quantized, p2.quantized) and torch.equal(p1.absmax, p2.absmax)


def test_cache_v2_double_quant_roundtrip_and_rejections(tmp_path):
    w = torch.randn(64, 256, dtype=torch.float16)
    packed, aq, a2, c2, off = O.quantize_nf4_dq(w, 64)
    t = torch.from_numpy
    payload = NF4Payload(t(packed).reshape(-1, 1), t(aq), t(O.NF4_LEVELS.copy()), (64, 256), torch.float16, 64, "nf4",
                         w.numel(), w.numel() * 2, 0, nested=True, absmax2=t(a2), code2=t(c2),
                         offset=torch.tensor(off))
    path = tmp_path / "w.pt"
    upload._save_payload_to_cache(path, payload)
    param = nn.Parameter(w, requires_grad=False)
    got = upload._load_payload_from_cache(path, param, blocksize=64, quant_type="nf4", compress_statistics=True)
    assert got is not None and got.nested and torch.equal(got.absmax2, payload.absmax2)
    assert float(got.offset) == float(off)
    # a double-quant file does not satisfy a plain request (and vice versa)
    assert upload._load_payload_from_cache(path, param, blocksize=64, quant_type="nf4") is None
    path.write_bytes(b"not a torch file")
    assert upload._load_payload_from_cache(path, param, blocksize=64, quant_type="nf4",
                                           compress_statistics=True) is None


# ------------------------------------------------------------- lifecycle --

def _staged_module():
    module = nn.Module()
    p = nn.Parameter(torch.zeros(0, dtype=torch.float16), requires_grad=False)
    payload = NF4Payload(torch.zeros(2, dtype=torch.uint8), torch.ones(1), torch.zeros(16), (2, 2), torch.float16, 64,
                         "nf4", 4, 8, 19)
    setattr(p, NF4_ATTR, payload)
    module.register_parameter("weight", p)
    return module, p


def test_free_weights_releases_materialised_data_only():
    module, p = _staged_module()
    assert upload.free_weights(module) == 0  # nothing materialised yet
    p.data = torch.ones(2, 2, dtype=torch.float16)
    assert upload.free_weights(module) == 1
    assert p.data.numel() == 0 and hasattr(p, NF4_ATTR)


def test_ensure_weights_rejects_trainable_param_on_another_device():
    module = nn.Module()
    module.register_parameter("lora", nn.Parameter(torch.randn(4, 4)))
    with pytest.raises(RuntimeError, match="trainable shared parameter"):
        upload.ensure_weights(module, 0)


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-CUDA error path")
def test_prefetch_without_cuda_raises_and_empty_prefetch_is_noop():
    module, _ = _staged_module()
    with pytest.raises(RuntimeError, match="CUDA is not available"):
        upload.prefetch_weights(module, 0)
    empty = upload.NF4Prefetch([], torch.device("cuda:0"))
    assert empty.finalize() == 0 and empty.wait() == 0


def test_ensure_prefetched_weights_device_mismatch():
    pf = upload.NF4Prefetch([object()], torch.device("cuda:1"))
    with pytest.raises(ValueError, match="does not match"):
        upload.ensure_prefetched_weights(nn.Module(), 0, pf)


def test_layer_arena_packs_every_payload_aligned():
    module = nn.Module()
    for name, shape in (("a", (64, 128)), ("b", (32, 64))):
        w = torch.randn(*shape, dtype=torch.float16)
        packed, absmax = O.quantize_nf4(w, 64)
        p = nn.Parameter(torch.zeros(0, dtype=torch.float16), requires_grad=False)
        setattr(p, NF4_ATTR, NF4Payload(torch.from_numpy(packed).reshape(-1, 1), torch.from_numpy(absmax),
                                        torch.from_numpy(O.NF4_LEVELS.copy()), shape, torch.float16, 64, "nf4",
                                        w.numel(), w.numel() * 2, 0))
        module.register_parameter(name, p)
    arena = upload.build_layer_arena(module)
    for p in module.parameters():
        payload = getattr(p, NF4_ATTR)
        views = arena.views(arena.host, id(p), 3)
        for v, t in zip(views, payload.host_tensors()):
            assert torch.equal(v.cpu(), t)
        for i in range(3):
            assert arena.slots[(id(p), i)][0] % 256 == 0


# ------------------------------------------------------------ assign/stage --

def test_assign_matches_reference_distributions():
    # distributions printed by the reference's assign_layers_to_devices (stratum/assign.py)
    def dist(a, nd):
        return [list(a.values()).count(d) for d in range(nd)]
    assert dist(assign_layers_to_devices(32, n_devices=8), 8) == [5, 4, 4, 4, 4, 4, 4, 3]
    assert dist(assign_layers_to_devices(48, n_devices=8), 8) == [7, 6, 6, 6, 6, 6, 6, 5]
    assert dist(assign_layers_to_devices(28, n_devices=4), 4) == [8, 7, 7, 6]
    assert dist(assign_layers_to_devices(32, tensor_split=[10, 32]), 2) == [8, 24]
    assert dist(assign_layers_to_devices(4, tensor_split=[3, 1]), 2) == [4, 0]
    assert assign_layers_to_devices(5) == {i: 0 for i in range(5)}
    assert strata(assign_layers_to_devices(6, n_devices=2)) == [(0, [0, 1, 2, 3]), (1, [4, 5])]  # lower-bound rule
    with pytest.raises(ValueError):
        assign_layers_to_devices(4, tensor_split=[])
    with pytest.raises(ValueError):
        assign_layers_to_devices(4, n_devices=0)
    with pytest.raises(ValueError):
        assign_layers_to_devices(4, device_ids=[0, 1], n_devices=3)


class _AddLayer(nn.Module):
    def __init__(self, k):
        super().__init__()
        self.k = k

    def forward(self, data):
        hidden, *rest = data
        return (hidden + self.k, *rest)


def test_device_stage_forward_range_order_and_bounds():
    stage = DeviceStage([_AddLayer(1), _AddLayer(10), _AddLayer(100)], device_id=0)
    out = stage.forward_range((torch.zeros(2), "mask"), local_start=1)
    assert out[0].tolist() == [110.0, 110.0] and out[1] == "mask"
    assert stage((torch.zeros(1),))[0].item() == 111.0
    for bad in ((-1, 2), (0, 4), (2, 2)):
        with pytest.raises(ValueError):
            stage.forward_range((torch.zeros(1),), local_start=bad[0], local_stop=bad[1])


def test_balanced_strata_minimise_the_largest_load():
    from stratum_b200.assign import balanced_strata

    for L in (32, 48, 7):
        for n in (1, 2, 3, 4, 8):
            for tail in (0.0, 1.5, 2.0):
                st = balanced_strata(L, n, tail_cost=tail)
                assert len(st) == n
                assert [i for s in st for i in s] == list(range(L))  # contiguous, every layer once
                load = max(len(s) + (tail if i == n - 1 else 0.0) for i, s in enumerate(st))
                # no contiguous split does better: the bound ceil-ish of (L + tail) / n over integer counts
                best = min(max(max(-(-(L - c) // max(n - 1, 1)), 0) if n > 1 else L, c + tail) for c in range(L + 1)) \
                    if n > 1 else L + tail
                assert load <= best + 1e-9, (L, n, tail, [len(s) for s in st], load, best)
    assert [len(s) for s in balanced_strata(32, 8, tail_cost=1.5)] == [4, 4, 4, 4, 4, 4, 5, 3]


def test_to_nf4_experts_converts_staged_3d_experts():
    """HF-style experts with NF4-staged 3-D params become a streamed NF4Experts whose
    two placeholder parameters keep their payloads (the upload contract feeds them)."""
    from stratum_b200.experts import NF4Experts

    E, H, I = 4, 64, 32
    experts = nn.Module()
    experts.gate_up_proj = nn.Parameter(torch.randn(E, 2 * I, H, dtype=torch.float16), requires_grad=False)
    experts.down_proj = nn.Parameter(torch.randn(E, H, I, dtype=torch.float16), requires_grad=False)
    experts.act_fn = nn.SiLU()
    block = nn.Module()
    block.experts = experts
    _run_prepare(block, min_numel=8)
    assert upload.to_nf4_experts(block) == 1
    m = block.experts
    assert isinstance(m, NF4Experts) and m.streamed and not m.resident
    assert (m.num_experts, m.hidden_dim, m.intermediate_dim) == (E, H, I)
    names = dict(m.named_parameters())
    assert set(names) == {"gate_up_weight", "down_weight"}
    assert getattr(names["gate_up_weight"], NF4_ATTR).shape == (E, 2 * I, H)
    owner_map = upload._build_param_owner_map(block)
    own, pname = owner_map[id(names["down_weight"])]
    assert upload._fused_owner(own, pname) is not None
    with pytest.raises(RuntimeError):
        m(torch.zeros(2, H, dtype=torch.bfloat16), torch.zeros(2, 1, dtype=torch.long), torch.ones(2, 1))


def _stream_module():
    """A meta-device wrapped layer (idx 3) with a frozen linear, a 1-D norm and 3-D experts."""

    class Wrapped(nn.Module):
        def __init__(self):
            super().__init__()
            self.idx = 3
            self.layer = nn.Module()
            with torch.device("meta"):
                self.layer.q_proj = nn.Linear(64, 128, bias=False, dtype=torch.float16)
                self.layer.norm = nn.Module()
                self.layer.norm.weight = nn.Parameter(torch.empty(64, dtype=torch.float16))
                self.layer.mlp = nn.Module()
                self.layer.mlp.experts = nn.Module()
                self.layer.mlp.experts.gate_up_proj = nn.Parameter(torch.empty(2, 32, 64, dtype=torch.float16))
                self.layer.mlp.experts.down_proj = nn.Parameter(torch.empty(2, 64, 16, dtype=torch.float16))

    root = nn.Module()
    root.w = Wrapped()
    root.requires_grad_(False)
    return root


def _stream_ckpt(tmp_path, sharded: bool):
    from safetensors.torch import save_file

    g = torch.Generator().manual_seed(0)
    t = {"model.layers.3.q_proj.weight": torch.randn(128, 64, generator=g).half(),
         "model.layers.3.norm.weight": torch.randn(64, generator=g).half()}
    for e in range(2):
        t[f"model.layers.3.mlp.experts.{e}.gate_proj.weight"] = torch.randn(16, 64, generator=g).half()
        t[f"model.layers.3.mlp.experts.{e}.up_proj.weight"] = torch.randn(16, 64, generator=g).half()
        t[f"model.layers.3.mlp.experts.{e}.down_proj.weight"] = torch.randn(64, 16, generator=g).half()
    if sharded:
        import json

        names = sorted(t)
        a, b = names[: len(names) // 2], names[len(names) // 2:]
        save_file({k: t[k] for k in a}, str(tmp_path / "s1.safetensors"))
        save_file({k: t[k] for k in b}, str(tmp_path / "s2.safetensors"))
        wm = {k: "s1.safetensors" for k in a} | {k: "s2.safetensors" for k in b}
        # stacked experts are addressed by their fused name in a sharded index
        (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"weight_map": wm}))
    else:
        save_file(t, str(tmp_path / "model.safetensors"))
    return t


def test_stream_load_and_quantize_single_file(tmp_path):
    ckpt = _stream_ckpt(tmp_path, sharded=False)
    m = _stream_module()
    fake, calls = _fake_quantizer()
    cache = tmp_path / "cache"
    with mock.patch.object(upload, "_quantize_param", side_effect=fake):
        stats = upload.stream_load_and_quantize_module(m, str(tmp_path), min_numel=512, cache_dir=cache)
    assert stats is not None and stats.tensors == 3 and stats.cache_writes == 3
    q = m.w.layer.q_proj.weight
    assert getattr(q, NF4_ATTR).shape == (128, 64) and q.data.numel() == 0
    gu = m.w.layer.mlp.experts.gate_up_proj
    assert getattr(gu, NF4_ATTR).shape == (2, 32, 64)
    assert (2, 32, 64) in calls  # the stacked per-expert tensor went through the quantizer
    norm = m.w.layer.norm.weight
    assert norm.device.type == "cpu" and torch.equal(norm.data, ckpt["model.layers.3.norm.weight"])
    # a second pass over a fresh module is served from the payload cache
    m2 = _stream_module()
    with mock.patch.object(upload, "_quantize_param", side_effect=AssertionError("should hit the cache")):
        stats2 = upload.stream_load_and_quantize_module(m2, str(tmp_path), min_numel=512, cache_dir=cache)
    assert stats2.cache_hits == 3


def test_stream_load_sharded_and_missing_key(tmp_path):
    _stream_ckpt(tmp_path, sharded=True)
    m = _stream_module()
    del m.w.layer.mlp  # per-expert keys are stacked only for single-file checkpoints (as the reference)
    fake, _ = _fake_quantizer()
    with mock.patch.object(upload, "_quantize_param", side_effect=fake):
        stats = upload.stream_load_and_quantize_module(m, str(tmp_path), min_numel=512)
    assert stats is not None and stats.tensors == 1
    m3 = _stream_module()
    with torch.device("meta"):
        m3.w.layer.extra = nn.Parameter(torch.empty(8, 8), requires_grad=False)
    with mock.patch.object(upload, "_quantize_param", side_effect=fake):
        assert upload.stream_load_and_quantize_module(m3, str(tmp_path), min_numel=512) is None
