"""B200-native (sm_100a) hot path of Qwen3-TTS serving: paged GQA attention
for the talker and code predictor, the fused logits sampler and the GPU
page planner, behind the reference engine's call surfaces.

Import with ``importlib.import_module("nari-qwen3-tts_b200")`` (the directory
name is not a Python identifier).  Kernels live in ``libnqt.so`` (C ABI in
include/nqt.h); build it with ``build.build()``.
"""

from . import kernels, planner, sampling, step_control, talker_kv
from ._lib import NqtError, lib
from .kernels import (
    cp_decode_attention_,
    decode_attn_nhd_short_cache,
    paired_qk_norm_rope_,
    paired_qk_norm_rope_dense_cache_,
    paired_qk_norm_rope_paged_cache_,
)
from .planner import DevicePagePlanner, KVAllocationError
from .sampling import (
    sample_code_predictor_cuda_graph,
    sample_logits_cuda_graph,
    sample_logits_stateless,
    sample_rows,
    sample_talker_cuda_graph,
)
from .step_control import DeviceStepControl, RequestSampling
from .talker_kv import (
    B200TalkerBinding,
    TalkerAttentionMetadata,
    batch_decode_paged,
    batch_prefill_paged,
    binding_factory,
)

__all__ = [
    "B200TalkerBinding",
    "DevicePagePlanner",
    "DeviceStepControl",
    "KVAllocationError",
    "NqtError",
    "RequestSampling",
    "TalkerAttentionMetadata",
    "batch_decode_paged",
    "batch_prefill_paged",
    "binding_factory",
    "cp_decode_attention_",
    "decode_attn_nhd_short_cache",
    "kernels",
    "lib",
    "paired_qk_norm_rope_",
    "paired_qk_norm_rope_dense_cache_",
    "paired_qk_norm_rope_paged_cache_",
    "planner",
    "sample_code_predictor_cuda_graph",
    "sample_logits_cuda_graph",
    "sample_logits_stateless",
    "sample_rows",
    "sample_talker_cuda_graph",
    "sampling",
    "step_control",
    "talker_kv",
]
