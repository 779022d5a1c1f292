"""CLI wiring of the logprob backend, mirroring the reference's tests of
``scripts/train_sft.py`` / ``scripts/train_grpo.py`` (``tests/test_logprob_backends.py:33-48``,
``tests/test_grpo_logprob_backend.py:126-141``): unsupported configurations exit with
status 2 before any device work, the default stays "jax"."""

from __future__ import annotations

import argparse

import pytest

from gemma4_posttrain_jax_b200.cli import add_logprob_arguments, validate_logprob_arguments, validate_logprob_devices


def _parse(argv, compute_dtype="bf16", vocab_parallel=True):
    parser = add_logprob_arguments(argparse.ArgumentParser(), vocab_parallel=vocab_parallel)
    args = parser.parse_args(argv)
    validate_logprob_arguments(args, parser, compute_dtype=compute_dtype)
    return args


def test_backend_defaults_to_jax_and_accepts_cuda():
    assert _parse([]).logprob_backend == "jax"
    args = _parse(["--logprob-backend", "cuda", "--vocab-chunk", "4096", "--sequence-chunk", "128"])
    assert (args.logprob_backend, args.vocab_chunk, args.sequence_chunk) == ("cuda", 4096, 128)
    assert _parse(["--logprob-backend", "cuda", "--no-vocab-parallel"]).vocab_parallel is False


@pytest.mark.parametrize(
    "extra,dtype",
    [((), "f32"), (("--no-vocab-parallel",), "bf16"), (("--sequence-chunk", "128"), "bf16"),
     (("--vocab-chunk", "4096"), "bf16")],
)
def test_cli_rejects_unsupported_pallas_config(extra, dtype):
    with pytest.raises(SystemExit) as error:
        _parse(["--logprob-backend", "pallas", *extra], compute_dtype=dtype)
    assert error.value.code == 2


@pytest.mark.parametrize("argv,dtype", [(["--logprob-backend", "cuda"], "f32"),
                                        (["--logprob-backend", "cuda", "--vocab-chunk", "0"], "bf16"),
                                        (["--logprob-backend", "tpu"], "bf16")])
def test_cli_rejects_unsupported_cuda_config(argv, dtype):
    with pytest.raises(SystemExit) as error:
        _parse(argv, compute_dtype=dtype)
    assert error.value.code == 2


def test_device_stage_refuses_without_a_b200():
    import torch

    if torch.cuda.is_available() and torch.cuda.get_device_capability() == (10, 0):
        pytest.skip("a B200 is visible")
    with pytest.raises(ValueError, match="B200"):
        validate_logprob_devices("cuda", 262144)
    validate_logprob_devices("jax", 262144)  # other backends are the reference's to check
