"""B200-native (sm_100a) chunked vocab-parallel token-logprob for gemma4-posttrain.

A drop-in ``backend="cuda"`` for the logprob path of yixiaoer/gemma4-posttrain-jax
(``gemma4_posttrain_jax/losses.py:55-343``): tied LM-head contraction with a fused online
log-sum-exp / target-pick epilogue, recompute backward into tensor-core dH / dW GEMMs,
response-token compaction, vocabulary sharding over NCCL / NVLink, and the rollout sampler's
full-vocabulary head (``sampler.py``). The kernels live in
``liblp_b200.so`` (C ABI: ``include/lp_logprob.h``); this package is the host side.
"""

from .logprob_protocol import CUDA_LOGPROB_PROTOCOL, logprob_run_metadata, validate_logprob_resume  # noqa: F401
from .losses import completion_logps, per_token_logps, sft_token_logps  # noqa: F401
from .sampler import lm_head_logits, sample_token  # noqa: F401
from .sharding import VocabMesh, make_mesh, shard_rows  # noqa: F401

__all__ = [
    "CUDA_LOGPROB_PROTOCOL",
    "VocabMesh",
    "completion_logps",
    "lm_head_logits",
    "logprob_run_metadata",
    "make_mesh",
    "per_token_logps",
    "sample_token",
    "sft_token_logps",
    "shard_rows",
    "validate_logprob_resume",
]
