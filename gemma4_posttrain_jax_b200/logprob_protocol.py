"""Checkpoint identity of the logprob backends.

Mirrors ``gemma4_posttrain_jax/logprob_protocol.py:1-14``: a run records which logprob
implementation produced its gradients, and resuming with a different backend or protocol
is refused. The reference knows "jax" (native, recorded as nothing for legacy
checkpoints) and "pallas"; this package adds "cuda".
"""

from __future__ import annotations

from collections.abc import Mapping
from typing import Any

PALLAS_LOGPROB_PROTOCOL = "v4-native-shared-bf16x3-v1"
# bf16 operands, f32 tensor-core accumulation, base-2 online log-sum-exp per 128x256
# tile, dZ rounded to bf16 once before the dH / dW GEMMs.
CUDA_LOGPROB_PROTOCOL = "b200-tcgen05-bf16-dz-v1"

BACKENDS = ("jax", "pallas", "cuda")


def logprob_run_metadata(backend: str) -> dict[str, str]:
    """Run-config entries identifying ``backend`` (empty for the native "jax" backend)."""
    if backend == "jax":
        return {}
    if backend == "pallas":
        return {"logprob_backend": backend, "logprob_protocol": PALLAS_LOGPROB_PROTOCOL}
    if backend == "cuda":
        return {"logprob_backend": backend, "logprob_protocol": CUDA_LOGPROB_PROTOCOL}
    raise ValueError(f"unknown logprob backend: {backend}")


def validate_logprob_resume(saved: Mapping[str, Any], current: Mapping[str, Any]) -> None:
    """Refuse a resume that changes the logprob backend or its protocol.

    Same rule as ``scripts/train_sft.py:157-170`` for these two fields: a checkpoint that
    recorded no backend was written by the native "jax" backend.
    """
    s = {"logprob_backend": "jax", **saved}
    c = {"logprob_backend": "jax", **current}
    diffs = {
        k: {"saved": s.get(k), "current": c.get(k)}
        for k in ("logprob_backend", "logprob_protocol")
        if s.get(k) != c.get(k)
    }
    if diffs:
        raise ValueError(f"resume config differs from checkpoint: {diffs}")
