"""Command-line wiring of the logprob backend for training scripts.

The reference's training scripts take ``--logprob-backend {jax,pallas}``,
``--vocab-chunk``, ``--sequence-chunk`` and (SFT) ``--vocab-parallel``
(``scripts/train_sft.py:80-92``, ``scripts/train_grpo.py:212-219``) and refuse
configurations a backend cannot run with ``parser.error`` (exit status 2,
``scripts/train_sft.py:120-125``, ``scripts/train_grpo.py:251-259``) before any device
work; device-level conditions are checked when the mesh exists and raise ``ValueError``
(``scripts/train_grpo.py:537-540``). This module adds ``cuda`` to the choices and applies
the same two-stage rule to it: the CLI stage checks what the flags alone decide, the device
stage checks that every rank drives a B200 and that the vocabulary divides over the mesh.
No backend silently falls back to another.
"""

from __future__ import annotations

import argparse

from .logprob_protocol import BACKENDS

_HELP = {
    "jax": "native JAX chunked logprob (gemma4_posttrain_jax)",
    "pallas": "four-chip TPU v4 / BF16 Pallas dW kernel (gemma4_posttrain_jax)",
    "cuda": "B200 (sm_100a) tensor-core kernels of this package",
}


def add_logprob_arguments(parser: argparse.ArgumentParser, *, vocab_parallel: bool = True) -> argparse.ArgumentParser:
    """Add the logprob flags with the reference's names and defaults (backend default "jax")."""
    parser.add_argument(
        "--logprob-backend",
        choices=BACKENDS,
        default="jax",
        help="logprob backend: " + "; ".join(f"{k}: {v}" for k, v in _HELP.items()),
    )
    parser.add_argument("--vocab-chunk", type=int, default=8192)
    parser.add_argument("--sequence-chunk", type=int, default=256)
    if vocab_parallel:
        parser.add_argument(
            "--vocab-parallel",
            action=argparse.BooleanOptionalAction,
            default=True,
            help="keep the LM-head embedding vocabulary-sharded (default: enabled)",
        )
    return parser


def validate_logprob_arguments(
    args: argparse.Namespace, parser: argparse.ArgumentParser, *, compute_dtype: str = "bf16"
) -> None:
    """``parser.error`` (exit status 2) for flag combinations the chosen backend does not run.

    pallas: the reference's rule (BF16, vocabulary parallelism, vocab-chunk 8192,
    sequence-chunk 256). cuda: BF16 compute (the kernels take bf16 operands and accumulate
    in f32); the chunk sizes only have to be positive, since the kernels tile the
    vocabulary and the tokens themselves and give the same result for any chunking.
    """
    if args.vocab_chunk <= 0 or args.sequence_chunk <= 0:
        parser.error("vocab-chunk and sequence-chunk must be positive")
    vocab_parallel = getattr(args, "vocab_parallel", True)
    if args.logprob_backend == "pallas" and (
        not vocab_parallel or compute_dtype != "bf16" or (args.vocab_chunk, args.sequence_chunk) != (8192, 256)
    ):
        parser.error("Pallas logprob requires BF16, vocabulary parallelism, vocab-chunk=8192 and sequence-chunk=256")
    if args.logprob_backend == "cuda" and compute_dtype != "bf16":
        parser.error("CUDA logprob requires BF16 compute (bf16 operands, f32 accumulation)")


def validate_logprob_devices(backend: str, vocab_size: int, mesh=None) -> None:
    """Device-stage check of the cuda backend (``ValueError``, like the reference's mesh check
    for pallas): a B200 (sm_100) current device on this rank and a vocabulary that divides
    over the mesh. Other backends are validated by the reference itself."""
    if backend != "cuda":
        return
    import torch  # noqa: PLC0415

    if not torch.cuda.is_available():
        raise ValueError("CUDA logprob requires a B200 (sm_100) GPU on every rank; none is visible")
    major, minor = torch.cuda.get_device_capability()
    if (major, minor) != (10, 0):
        raise ValueError(f"CUDA logprob requires a B200 (sm_100) GPU on every rank; found sm_{major}{minor}")
    size = mesh.size if mesh is not None else 1
    if vocab_size % size:
        raise ValueError(f"vocab size {vocab_size} must be divisible by mesh axis {size}")
