"""CPU oracle for the chunked vocab-parallel token-logprob path (test infrastructure only).

This package is a numpy restatement of the reference's native JAX logprob backend,
``gemma4_posttrain_jax/losses.py:55-260`` (yixiaoer/gemma4-posttrain-jax), plus an
analytic float64 backward. It exists to CHECK the CUDA product path: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / ``--impl reference`` leg may
import it. The product package never imports it and has no CPU fallback.

Parity pinning: the reference is JAX-only and JAX cannot be installed in this image, so
no reference-produced golden values exist. The restatement is pinned to the relations
the reference's own tests assert (streaming == dense log-softmax, values and gradients,
``tests/test_losses.py:13-53``; normalisation stats == dense max / sum-exp,
``tests/test_native_logprob_stats.py:53-66``; vocab-parallel == single-partition,
``tests/test_sharding_tpu.py:47-101``) on the reference tests' own seeded inputs.
"""

from .logprob_oracle import (  # noqa: F401
    bf16_round,
    dense_logps,
    logps_grads_f64,
    single_partition_logps,
    vocab_parallel_logps_and_normalization,
    per_token_logps,
    compact_response,
)
