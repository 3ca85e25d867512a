"""stratum_b200: B200-native (sm_100a) kernels behind Stratum's NF4 frozen-weight path.

The package keeps the reference's hot-path names (stratum/__init__.py:51-54,
stratum/upload.py, stratum/nf4_linear.py, stratum/stage.py, stratum/assign.py)
so it drops in for that path; the compute runs in libstratum_nf4.so (C ABI:
include/stratum_nf4.h).
"""

from .assign import assign_layers_to_devices, balanced_strata, strata
from .boundary import DeviceTransferPool, make_boundary_hook
from .experts import NF4Experts
from .functional import QuantState, dequantize_4bit, dequantize_4bit_many, quantize_4bit
from .nf4_linear import NF4Linear
from .pipeline import RankPipeline, StratumPipeline
from .stage import DeviceStage
from .upload import (
    FP16_ATTR,
    NF4_ATTR,
    FP16StagedPayload,
    NF4Payload,
    NF4Prefetch,
    NF4Stats,
    build_layer_arena,
    ensure_prefetched_weights,
    ensure_weights,
    estimate_module_upload_gib,
    free_weights,
    prefetch_weights,
    prepare_fp16_staged,
    prepare_nf4,
    prepare_nf4_from_cache,
    stream_load_and_quantize_module,
    to_nf4_experts,
    to_nf4_linear,
    upload_stream,
)

__all__ = [
    "QuantState", "quantize_4bit", "dequantize_4bit", "NF4Linear", "DeviceStage", "assign_layers_to_devices",
    "NF4_ATTR", "FP16_ATTR", "NF4Payload", "FP16StagedPayload", "NF4Prefetch", "NF4Stats", "prepare_nf4",
    "prepare_nf4_from_cache", "prepare_fp16_staged", "ensure_weights", "free_weights", "prefetch_weights",
    "ensure_prefetched_weights", "upload_stream", "estimate_module_upload_gib", "build_layer_arena", "to_nf4_linear",
    "to_nf4_experts", "NF4Experts", "dequantize_4bit_many", "StratumPipeline", "RankPipeline", "DeviceTransferPool",
    "make_boundary_hook", "balanced_strata", "strata", "stream_load_and_quantize_module",
]
