"""Generate the golden NF4 fixtures in this directory (run here, where the reference is mounted).

    python tests/golden/make_golden.py /path/to/reference

The reference's own ``stratum.upload.prepare_nf4`` (stratum/upload.py:305-398)
is imported and run on small seeded modules, with ``bitsandbytes.functional``
replaced by a stand-in whose ``quantize_4bit`` is the CPU oracle
(oracle/nf4_oracle.py) -- bitsandbytes itself is not installable here.  The
reference writes its version-1 cache files (stratum/upload.py:287-302); those
files are the fixtures.  They pin:

* the reference's selection rules and payload metadata (which parameters are
  quantized, the 3-D -> [-1, last] reshape, shapes, dtypes, byte counts,
  the cache file naming and dict layout) -- produced by reference code;
* the codec numbers (packed nibbles, absmax) -- produced by the oracle, i.e.
  the restated bitsandbytes algorithm, so parity with bitsandbytes itself
  stays unpinned.

A manifest (manifest.json) records the inputs' seeds and the file names.
"""

from __future__ import annotations

import json
import sys
import types
from pathlib import Path

import numpy as np
import torch
import torch.nn as nn

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from oracle import nf4_oracle as O  # noqa: E402


class _QuantState:
    def __init__(self, absmax, shape, code, blocksize, quant_type, dtype):
        self.absmax, self.shape, self.code = absmax, shape, code
        self.blocksize, self.quant_type, self.dtype = blocksize, quant_type, dtype


def _fake_bnb():
    def quantize_4bit(A, blocksize=64, compress_statistics=False, quant_type="nf4", **_):
        assert quant_type == "nf4" and not compress_statistics
        packed, absmax = O.quantize_nf4(A, blocksize)
        return (torch.from_numpy(packed).reshape(-1, 1),
                _QuantState(torch.from_numpy(absmax), tuple(A.shape), torch.from_numpy(O.NF4_LEVELS.copy()),
                            blocksize, quant_type, A.dtype))

    functional = types.ModuleType("bitsandbytes.functional")
    functional.quantize_4bit = quantize_4bit
    functional.QuantState = _QuantState
    pkg = types.ModuleType("bitsandbytes")
    pkg.functional = functional
    return pkg, functional


def build_modules():
    """Small seeded modules with the shapes that matter (2-D linears, a 3-D expert stack,
    trainable / small / 1-D parameters that must be skipped)."""
    g = torch.Generator().manual_seed(0)

    class Block(nn.Module):
        def __init__(self):
            super().__init__()
            self.q_proj = nn.Linear(128, 256, bias=False)
            self.o_proj = nn.Linear(256, 128, bias=True)
            self.norm = nn.Parameter(torch.ones(128))
            self.small = nn.Parameter(torch.randn(8, 8, generator=g), requires_grad=False)
            self.gate_up_proj = nn.Parameter(torch.randn(4, 96, 64, generator=g) * 0.02, requires_grad=False)
            self.lora_like = nn.Parameter(torch.randn(16, 128, generator=g))

    m = Block()
    with torch.no_grad():
        m.q_proj.weight.copy_(torch.randn(256, 128, generator=g) * 0.02)
        m.o_proj.weight.copy_(torch.randn(128, 256, generator=g) * 0.02)
        m.o_proj.weight[3, 7] = 0.5  # outlier
        m.q_proj.weight[5] = 0.0  # zero blocks
        m.o_proj.bias.zero_()
    for p in (m.q_proj.weight, m.o_proj.weight, m.o_proj.bias):
        p.requires_grad_(False)
    m.half()
    m.lora_like.data = m.lora_like.data.float()
    return m


def main(ref_root: str) -> None:
    """``ref_root``: the checkout of the reference project (the directory that holds ``stratum/``)."""
    if not (Path(ref_root) / "stratum" / "upload.py").is_file():
        raise SystemExit(f"{ref_root}: not a checkout of the reference (no stratum/upload.py)")
    sys.path.insert(0, ref_root)
    pkg, functional = _fake_bnb()
    sys.modules["bitsandbytes"] = pkg
    sys.modules["bitsandbytes.functional"] = functional
    import stratum.upload as ref_upload  # the reference's own code

    cache = HERE / "nf4_cache_v1"
    if cache.exists():
        for f in cache.iterdir():
            f.unlink()
    module = build_modules()
    inputs = {n: p.detach().clone() for n, p in module.named_parameters()}
    ref_upload._pin_cpu = lambda t: t.detach().contiguous().cpu()  # no CUDA here
    stats = ref_upload.prepare_nf4(module, min_numel=4096, cache_dir=str(cache), verbose=False)
    torch.save({n: t for n, t in inputs.items()}, HERE / "nf4_inputs.pt")
    manifest = {
        "generator": "tests/golden/make_golden.py",
        "reference_call": "stratum.upload.prepare_nf4(module, min_numel=4096, cache_dir=...)",
        "codec": "oracle/nf4_oracle.py quantize_nf4 (bitsandbytes stand-in; parity with bitsandbytes unpinned)",
        "stats": {"tensors": stats.tensors, "source_bytes": stats.source_bytes, "payload_bytes": stats.payload_bytes,
                  "cache_writes": stats.cache_writes},
        "files": sorted(f.name for f in cache.iterdir()),
        "quantized_params": sorted(n for n, p in module.named_parameters() if hasattr(p, ref_upload.NF4_ATTR)),
    }
    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1) + "\n")
    print(json.dumps(manifest, indent=1))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_golden.py /path/to/reference")
    main(sys.argv[1])
