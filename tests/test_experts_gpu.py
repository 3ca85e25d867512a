"""GPU parity of the routed-expert path: routing sort, grouped NF4 GEMMs (plain,
routing-weight, SwiGLU epilogues; input gradient), combine, and NF4Experts
forward + backward against HF Qwen3MoeExperts semantics.

References are fp32 computations over the oracle-exact dequantized weights
(the codec tests pin the dequantizer bit for bit).  Tolerance for GEMM outputs
and gradients: ||a - b|| / ||b|| <= 1e-2; routing indices are exact."""

import pytest
import torch
import torch.nn.functional as TF

from oracle.nf4_oracle import relative_error
from stratum_b200 import _lib, ops
from stratum_b200 import functional as F
from stratum_b200.experts import NF4Experts

pytestmark = pytest.mark.gpu

DEV = "cuda"
TOL = 1e-2


def _expert_weight(E, N_e, K, seed, dq=False):
    g = torch.Generator(device=DEV).manual_seed(seed)
    w = (torch.randn(E * N_e, K, generator=g, device=DEV) * 0.02).to(torch.float16)
    packed, qs = F.quantize_4bit(w, compress_statistics=dq)
    w_deq = F.dequantize_4bit(packed, qs, out_dtype=torch.float32).reshape(E, N_e, K)
    return packed, qs, w_deq


def _routing_from_counts(counts, k=1, seed=0):
    """top_k_index [T, k] whose pairs hit expert e exactly counts[e] times, shuffled."""
    g = torch.Generator().manual_seed(seed)
    ids = torch.cat([torch.full((c,), e, dtype=torch.int64) for e, c in enumerate(counts)])
    ids = ids[torch.randperm(ids.numel(), generator=g)]
    assert ids.numel() % k == 0
    return ids.view(-1, k).to(DEV)


def _ref_route(top_k_index, E):
    flat = top_k_index.reshape(-1).cpu()
    bucket = torch.where((flat >= 0) & (flat < E), flat, torch.full_like(flat, E))
    order = torch.sort(bucket, stable=True).indices
    counts = torch.bincount(bucket, minlength=E + 1)
    offsets = torch.zeros(E + 1, dtype=torch.int64)
    offsets[1:] = torch.cumsum(counts[:E], 0)
    return order, offsets


# ------------------------------------------------------------------ routing --

@pytest.mark.parametrize("T,k,E", [(1, 1, 4), (37, 2, 8), (4096, 8, 128), (3000, 3, 1023), (2048, 8, 64)])
def test_route_is_a_stable_counting_sort(T, k, E):
    g = torch.Generator(device=DEV).manual_seed(T + k + E)
    idx = torch.randint(0, E, (T, k), generator=g, device=DEV)
    r = ops.moe_route(idx, E)
    order, offsets = _ref_route(idx, E)
    assert torch.equal(r.order.cpu().long(), order)
    assert torch.equal(r.offsets.cpu().long(), offsets)
    assert torch.equal(r.inv.cpu().long()[order], torch.arange(T * k))
    assert torch.equal(r.token_of.cpu().long(), order // k)


def test_route_drops_out_of_range_experts():
    E = 16
    g = torch.Generator(device=DEV).manual_seed(5)
    idx = torch.randint(-2, E + 3, (777, 4), generator=g, device=DEV)  # HF skips expert_idx == E
    r = ops.moe_route(idx, E)
    order, offsets = _ref_route(idx, E)
    assert torch.equal(r.order.cpu().long(), order)
    assert torch.equal(r.offsets.cpu().long(), offsets)
    valid = ((idx >= 0) & (idx < E)).sum().item()
    assert int(r.offsets[E]) == valid


def test_route_skewed_and_empty_experts():
    counts = [0, 1000, 0, 3, 257, 0, 0, 9000, 1, 0]
    idx = _routing_from_counts(counts, k=1, seed=3)
    r = ops.moe_route(idx, len(counts))
    _, offsets = _ref_route(idx, len(counts))
    assert torch.equal(r.offsets.cpu().long(), offsets)


# ----------------------------------------------------------- grouped GEMMs --

# empty, single, tile edges (256: one MMA; 257-320: a second, narrower MMA in the
# forward; 321: two balanced tiles), multi-tile (641, 700, 1024)
SKEWED = [0, 1, 255, 256, 257, 700, 0, 3, 1024, 64, 300, 320, 321, 641]


def _sorted_inputs(counts, K, dtype, seed):
    idx = _routing_from_counts(counts, k=1, seed=seed)
    r = ops.moe_route(idx, len(counts))
    g = torch.Generator(device=DEV).manual_seed(seed + 1)
    x = torch.randn(r.rows, K, generator=g, device=DEV).to(dtype)
    return r, x


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("dq", [False, True])
def test_grouped_fwd_plain(dtype, dq):
    E, N_e, K = len(SKEWED), 256, 192
    packed, qs, w_deq = _expert_weight(E, N_e, K, seed=1, dq=dq)
    r, x = _sorted_inputs(SKEWED, K, dtype, seed=2)
    y = ops.nf4_grouped_fwd(x, r, packed, qs)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    offs = r.offsets.cpu().tolist()
    for e in range(E):
        a, b = offs[e], offs[e + 1]
        if b == a:
            continue
        ref = x[a:b].float() @ w_deq[e].to(dtype).float().t()
        err = relative_error(y[a:b].float(), ref)
        assert err < TOL, f"expert {e} ({b - a} rows): rel err {err}"


def test_grouped_fwd_routing_weight_scales_rows():
    E, N_e, K = len(SKEWED), 128, 128
    packed, qs, w_deq = _expert_weight(E, N_e, K, seed=3)
    r, x = _sorted_inputs(SKEWED, K, torch.bfloat16, seed=4)
    rw = torch.rand(r.rows, device=DEV)
    y = ops.nf4_grouped_fwd(x, r, packed, qs, rw=rw)
    offs = r.offsets.cpu().tolist()
    for e in range(E):
        a, b = offs[e], offs[e + 1]
        if b > a:
            ref = (x[a:b].float() @ w_deq[e].to(torch.bfloat16).float().t()) * rw[a:b, None]
            assert relative_error(y[a:b].float(), ref) < TOL


@pytest.mark.parametrize("dq", [False, True])
def test_grouped_fwd_swiglu(dq):
    E, I, K = len(SKEWED), 192, 256
    packed, qs, w_deq = _expert_weight(E, 2 * I, K, seed=5, dq=dq)
    r, x = _sorted_inputs(SKEWED, K, torch.bfloat16, seed=6)
    h, gu = ops.nf4_grouped_fwd(x, r, packed, qs, swiglu=True, keep_gate_up=True)
    h_only = ops.nf4_grouped_fwd(x, r, packed, qs, swiglu=True)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    offs = r.offsets.cpu().tolist()
    for e in range(E):
        a, b = offs[e], offs[e + 1]
        if b == a:
            continue
        z = x[a:b].float() @ w_deq[e].to(torch.bfloat16).float().t()
        gate, up = z.chunk(2, dim=-1)
        ref = TF.silu(gate) * up
        assert relative_error(h[a:b].float(), ref) < TOL, f"expert {e}"
        assert relative_error(gu[a:b].float(), z) < TOL, f"expert {e} gate|up"
        assert torch.equal(h[a:b], h_only[a:b])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("N_e,K", [(256, 192), (192, 320), (2048, 768)])
def test_grouped_dx(dtype, N_e, K):
    counts = SKEWED if N_e < 1024 else [300, 0, 513, 1]
    E = len(counts)
    packed, qs, w_deq = _expert_weight(E, N_e, K, seed=7)
    r, dy = _sorted_inputs(counts, N_e, dtype, seed=8)
    dx = ops.nf4_grouped_dx(dy, r, packed, qs)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    offs = r.offsets.cpu().tolist()
    for e in range(E):
        a, b = offs[e], offs[e + 1]
        if b > a:
            ref = dy[a:b].float() @ w_deq[e].to(dtype).float()
            err = relative_error(dx[a:b].float(), ref)
            assert err < TOL, f"expert {e}: rel err {err}"


def _tiles_ref(offs, m_tiles, cap):
    """The tile table's rule: an expert's n tokens in ceil(n / cap) equal tiles
    rounded up to 16 tokens (the last one shorter), weight-row tiles innermost."""
    out = []
    for e in range(len(offs) - 1):
        a, b = offs[e], offs[e + 1]
        if b <= a:
            continue
        n = b - a
        parts = -(-n // cap)
        sz = (-(-n // parts) + 15) // 16 * 16
        for t0 in range(a, b, sz):
            out += [(e, m, t0, min(t0 + sz, b)) for m in range(m_tiles)]
    return out


@pytest.mark.parametrize("kind", ["fwd", "dx"])
def test_grouped_tile_table(kind, monkeypatch):
    E, N_e, K = len(SKEWED), 256, 384
    packed, qs, _ = _expert_weight(E, N_e, K, seed=9)
    r, x = _sorted_inputs(SKEWED, N_e if kind == "dx" else K, torch.bfloat16, seed=10)
    seen = []
    real = ops._table

    def spy(*a):
        t = real(*a)
        seen.append(t[0])
        return t

    monkeypatch.setattr(ops, "_table", spy)
    if kind == "fwd":
        ops.nf4_grouped_fwd(x, r, packed, qs)
        m_tiles, cap = N_e // 128, 320
    else:
        ops.nf4_grouped_dx(x, r, packed, qs)
        m_tiles, cap = -(-K // 128), 256
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    raw = seen[0].cpu()
    n = int(raw[:4].view(torch.int32)[0])
    got = [tuple(t) for t in raw[256:256 + 16 * n].view(torch.int32).view(-1, 4).tolist()]
    assert got == _tiles_ref(r.offsets.cpu().tolist(), m_tiles, cap)


def test_grouped_rejects_bad_offsets():
    E, N_e, K = 4, 128, 64
    packed, qs, _ = _expert_weight(E, N_e, K, seed=9)
    r, x = _sorted_inputs([10, 10, 10, 10], K, torch.bfloat16, seed=10)
    r.offsets.copy_(torch.tensor([0, 30, 20, 40, 40], dtype=torch.int32, device=DEV))  # decreasing
    ops.nf4_grouped_fwd(x, r, packed, qs)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0x201  # reported by the tile-table builder; no tile ran
    assert _lib.device_status() == 0  # the read cleared it


# ------------------------------------------------------- combine / SwiGLU --

def test_combine_and_its_gradient():
    T, k, E, W = 1000, 8, 32, 512
    g = torch.Generator(device=DEV).manual_seed(11)
    idx = torch.randint(0, E + 1, (T, k), generator=g, device=DEV)  # some pairs dropped (id == E)
    r = ops.moe_route(idx, E)
    rows = torch.randn(r.rows, W, generator=g, device=DEV).to(torch.bfloat16)
    w = torch.rand(T, k, generator=g, device=DEV)
    out = ops.moe_combine(rows, r, w)
    live = (idx < E).float()
    gathered = rows.float()[r.inv.long()].view(T, k, W)
    ref = (gathered * (w * live)[..., None]).sum(1)
    assert relative_error(out.float(), ref) < 4e-3
    dout = torch.randn(T, W, generator=g, device=DEV).to(torch.bfloat16)
    dy_sorted, dw = ops.moe_combine_grad(dout, r, w, rows)
    order = r.order.long()
    tok = r.token_of.long()
    live_sorted = (torch.arange(r.rows, device=DEV) < r.offsets[E]).float()
    ref_dy = dout.float()[tok] * (w.reshape(-1)[order] * live_sorted)[:, None]
    assert relative_error(dy_sorted.float(), ref_dy) < 4e-3
    ref_dw = torch.zeros(T * k, device=DEV)
    ref_dw[order] = (dout.float()[tok] * rows.float()).sum(-1) * live_sorted
    assert relative_error(dw, ref_dw) < 1e-4


def test_swiglu_grad():
    g = torch.Generator(device=DEV).manual_seed(12)
    gu = (torch.randn(513, 2 * 768, generator=g, device=DEV) * 2).to(torch.bfloat16).requires_grad_()
    dh = torch.randn(513, 768, generator=g, device=DEV).to(torch.bfloat16)
    got = ops.swiglu_grad(gu.detach(), dh)
    g32 = gu.detach().float().requires_grad_()
    gate, up = g32.chunk(2, dim=-1)
    (TF.silu(gate) * up).backward(dh.float())
    assert relative_error(got.float(), g32.grad) < 4e-3


# ----------------------------------------------------------- NF4Experts --

class _HFExperts(torch.nn.Module):
    """Qwen3MoeExperts.forward restated in fp32 over given 3-D weights (the
    reference's loop, transformers' modeling_qwen3_moe.py)."""

    def __init__(self, gate_up, down):
        super().__init__()
        self.gate_up_proj, self.down_proj = gate_up, down
        self.num_experts = gate_up.shape[0]

    def forward(self, hidden_states, top_k_index, top_k_weights):
        final = torch.zeros_like(hidden_states)
        mask = TF.one_hot(top_k_index, num_classes=self.num_experts + 1).permute(2, 1, 0)
        for e in range(self.num_experts):
            pos, tok = torch.where(mask[e])
            if tok.numel() == 0:
                continue
            gate, up = TF.linear(hidden_states[tok], self.gate_up_proj[e]).chunk(2, dim=-1)
            h = TF.silu(gate) * up
            y = TF.linear(h, self.down_proj[e]) * top_k_weights[tok, pos, None]
            final.index_add_(0, tok, y.to(final.dtype))
        return final


def _router(x, n_experts, top_k, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    wr = torch.randn(n_experts, x.shape[-1], generator=g, device=DEV) * 0.02
    probs = torch.softmax(x.float() @ wr.t(), dim=-1)
    vals, idx = torch.topk(probs, top_k, dim=-1)
    vals = vals / vals.sum(-1, keepdim=True)
    return idx, vals


@pytest.mark.parametrize("T,E,k,H,I", [(256, 8, 2, 256, 128), (4096, 128, 8, 2048, 768)])
def test_nf4_experts_forward_backward_matches_reference(T, E, k, H, I):
    g = torch.Generator(device=DEV).manual_seed(13)
    hf = torch.nn.Module()
    hf.gate_up_proj = torch.nn.Parameter((torch.randn(E, 2 * I, H, generator=g, device=DEV) * 0.02).half(),
                                         requires_grad=False)
    hf.down_proj = torch.nn.Parameter((torch.randn(E, H, I, generator=g, device=DEV) * 0.02).half(),
                                      requires_grad=False)
    hf.act_fn = torch.nn.SiLU()
    mod = NF4Experts.from_experts(hf)
    gu_deq, d_deq = mod.dequantized()
    x = torch.randn(T, H, generator=g, device=DEV).to(torch.bfloat16)
    idx, w = _router(x, E, k, seed=14)
    dout = torch.randn(T, H, generator=g, device=DEV).to(torch.bfloat16)

    xa = x.clone().requires_grad_()
    wa = w.clone().requires_grad_()
    out = mod(xa, idx, wa)
    out.backward(dout)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0

    ref_mod = _HFExperts(gu_deq.to(torch.bfloat16).float(), d_deq.to(torch.bfloat16).float())
    xr = x.float().requires_grad_()
    wr = w.clone().requires_grad_()
    ref = ref_mod(xr, idx, wr)
    ref.backward(dout.float())
    assert relative_error(out.float(), ref) < TOL
    assert relative_error(xa.grad.float(), xr.grad) < TOL
    assert relative_error(wa.grad.float(), wr.grad) < TOL


def test_nf4_experts_matches_transformers_module():
    """The installed HF Qwen3MoeExperts, given the dequantized weights, against NF4Experts."""
    from transformers import Qwen3MoeConfig
    from transformers.models.qwen3_moe.modeling_qwen3_moe import Qwen3MoeExperts

    cfg = Qwen3MoeConfig(hidden_size=512, moe_intermediate_size=256, num_experts=16, num_experts_per_tok=4,
                         hidden_act="silu")
    hf = Qwen3MoeExperts(cfg).to(DEV)
    g = torch.Generator(device=DEV).manual_seed(15)
    with torch.no_grad():
        hf.gate_up_proj.copy_(torch.randn(hf.gate_up_proj.shape, generator=g, device=DEV) * 0.02)
        hf.down_proj.copy_(torch.randn(hf.down_proj.shape, generator=g, device=DEV) * 0.02)
    mod = NF4Experts.from_experts(hf)
    gu_deq, d_deq = mod.dequantized()
    with torch.no_grad():
        hf.gate_up_proj.copy_(gu_deq)
        hf.down_proj.copy_(d_deq)
    hf = hf.to(torch.bfloat16)
    x = torch.randn(333, 512, generator=g, device=DEV).to(torch.bfloat16)
    idx, w = _router(x, 16, 4, seed=16)
    with torch.no_grad():
        ref = hf(x, idx, w)
        out = mod(x, idx, w)
    # HF rounds gate|up, h and each of the k products to bf16; the fused path keeps fp32 until the output
    assert relative_error(out.float(), ref.float()) < TOL


def test_streamed_experts_through_the_upload_contract():
    """prepare_nf4 -> to_nf4_experts -> ensure_weights gives the same forward as quantizing
    the experts directly; free_weights drops the device copies; a layer arena works too."""
    from stratum_b200 import upload

    E, H, I, T, k = 16, 256, 128, 300, 4
    g0 = torch.Generator(device=DEV).manual_seed(21)
    experts = torch.nn.Module()
    experts.gate_up_proj = torch.nn.Parameter((torch.randn(E, 2 * I, H, generator=g0, device=DEV) * 0.02).half(),
                                              requires_grad=False)
    experts.down_proj = torch.nn.Parameter((torch.randn(E, H, I, generator=g0, device=DEV) * 0.02).half(),
                                           requires_grad=False)
    experts.act_fn = torch.nn.SiLU()
    direct = NF4Experts.from_experts(experts)
    block = torch.nn.Module()
    block.experts = experts
    upload.prepare_nf4(block, verbose=False, device=DEV)
    assert upload.to_nf4_experts(block) == 1
    x = torch.randn(T, H, generator=g0, device=DEV).to(torch.bfloat16)
    wts, idx = torch.topk(torch.softmax(torch.randn(T, E, generator=g0, device=DEV), -1), k, -1)
    for arena in (False, True):
        if arena:
            upload.build_layer_arena(block)
        assert upload.ensure_weights(block, 0) == 2
        assert block.experts.resident
        with torch.no_grad():
            assert torch.equal(block.experts(x, idx, wts), direct(x, idx, wts))
        assert upload.free_weights(block) == 2
        assert not block.experts.resident
