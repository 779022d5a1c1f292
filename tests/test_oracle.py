"""Pin the CPU oracle: the reference tests' own relations, plus the committed fixtures.

Relations ported from the reference (yixiaoer/gemma4-posttrain-jax):
* streaming == dense log-softmax, values and gradients, for vocab/sequence chunks
  (5,4), (8,7), (23,10) and softcap None / 3.0 — ``tests/test_losses.py:20-53``;
* shape validation message — ``tests/test_losses.py:56-58``;
* vocab-parallel normalisation stats == dense max / sum-exp and finite / positive —
  ``tests/test_native_logprob_stats.py:16-66``;
* vocab-parallel == single-partition with a planted extreme per-shard max —
  ``tests/test_sharding_tpu.py:47-101``.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import logprob_oracle as orc
from tests.golden.make_golden import losses_inputs, shard_inputs, stats_inputs

GOLDEN = Path(__file__).resolve().parent / "golden" / "logprob_golden.npz"


def _torch_grads(e, h, t, g, softcap):
    E = torch.tensor(e, dtype=torch.float64, requires_grad=True)
    H = torch.tensor(h, dtype=torch.float64, requires_grad=True)
    lg = H @ E.T
    if softcap is not None:
        lg = torch.tanh(lg / softcap) * softcap
    lp = torch.log_softmax(lg, -1).gather(-1, torch.tensor(t, dtype=torch.int64)[..., None])[..., 0]
    (lp * torch.tensor(g, dtype=torch.float64)).sum().backward()
    return lp.detach().numpy(), E.grad.numpy(), H.grad.numpy()


@pytest.mark.parametrize("softcap", [None, 3.0])
@pytest.mark.parametrize("vocab_chunk,sequence_chunk", [(5, 4), (8, 7), (23, 10)])
def test_streaming_matches_dense(softcap, vocab_chunk, sequence_chunk):
    e, h, t = losses_inputs()
    got = orc.single_partition_logps(e, h, t, softcap=softcap, vocab_chunk=vocab_chunk, sequence_chunk=sequence_chunk)
    np.testing.assert_allclose(got, orc.dense_logps(e, h, t, softcap), atol=2e-6, rtol=2e-6)
    _, dW32, dH32 = orc.fwd_bwd_f32(e, h, t, np.ones(t.shape, np.float32), softcap=softcap, vocab_chunk=vocab_chunk,
                                    sequence_chunk=sequence_chunk)
    lp, dE, dH = orc.logps_grads_f64(e, h, t, np.ones(t.shape), softcap)
    np.testing.assert_allclose(dW32, dE, atol=3e-6, rtol=3e-6)
    np.testing.assert_allclose(dH32, dH, atol=3e-6, rtol=3e-6)


@pytest.mark.parametrize("softcap", [None, 3.0, 30.0])
def test_analytic_vjp_equals_autograd(softcap):
    e, h, t = losses_inputs()
    g = np.random.default_rng(1).normal(size=t.shape)
    lp, dE, dH = orc.logps_grads_f64(e, h, t, g, softcap, vocab_block=6)
    lp_t, dE_t, dH_t = _torch_grads(e, h, t, g, softcap)
    np.testing.assert_allclose(lp, lp_t, atol=1e-12)
    np.testing.assert_allclose(dE, dE_t, atol=1e-12)
    np.testing.assert_allclose(dH, dH_t, atol=1e-12)


def test_shape_validation_messages():
    with pytest.raises(ValueError, match="does not match"):
        orc.single_partition_logps(np.ones((7, 3)), np.ones((2, 4, 3)), np.ones((2, 3), np.int32), softcap=None)
    with pytest.raises(ValueError, match="incompatible embedding"):
        orc.single_partition_logps(np.ones((7, 3)), np.ones((2, 4)), np.ones((2,), np.int32), softcap=None)
    with pytest.raises(ValueError, match="must be positive"):
        orc.single_partition_logps(np.ones((7, 3)), np.ones((2, 3)), np.ones((2,), np.int32), softcap=None,
                                   vocab_chunk=0)
    with pytest.raises(ValueError, match="divisible"):
        orc.vocab_parallel_logps_and_normalization(np.ones((7, 3)), np.ones((2, 3)), np.ones((2,), np.int32),
                                                   num_shards=4, softcap=None)


@pytest.mark.parametrize("softcap", [None, 30.0])
@pytest.mark.parametrize("scale", [0.04, 1.5])
def test_vocab_parallel_normalization_matches_dense(softcap, scale):
    w, h, tok, _ = stats_inputs(scale)
    values, norm = orc.vocab_parallel_logps_and_normalization(w, h, tok, num_shards=4, softcap=softcap,
                                                              vocab_chunk=128, sequence_chunk=256)
    single = orc.single_partition_logps(w, h, tok, softcap=softcap, vocab_chunk=128, sequence_chunk=256)
    np.testing.assert_allclose(values, single, atol=2e-5, rtol=2e-5)
    np.testing.assert_allclose(norm, orc.dense_normalization(w, h, softcap), atol=2e-5, rtol=2e-5)
    assert np.isfinite(norm).all() and (norm[1] > 0).all()


def test_vocab_parallel_extreme_per_shard_max():
    e, h, t, wts = shard_inputs()
    dist = orc.vocab_parallel_logps_and_normalization(e, h, t, num_shards=4, softcap=30.0, vocab_chunk=17,
                                                      sequence_chunk=6)[0]
    single = orc.single_partition_logps(e, h, t, softcap=30.0, vocab_chunk=17, sequence_chunk=6)
    np.testing.assert_allclose((dist * wts).sum(), (single * wts).sum(), atol=5e-6, rtol=5e-6)
    np.testing.assert_allclose(dist, orc.dense_logps(e, h, t, 30.0), atol=5e-6)


def test_golden_fixtures_reproduce():
    gold = np.load(GOLDEN)
    e, h, t = losses_inputs()
    for name, cap in (("none", None), ("cap3", 3.0)):
        lp, dE, dH = orc.logps_grads_f64(e, h, t, np.ones(t.shape), cap)
        np.testing.assert_allclose(lp, gold[f"losses_{name}_logps"], rtol=1e-12, atol=1e-12)
        np.testing.assert_allclose(dE, gold[f"losses_{name}_dE"], rtol=1e-10, atol=1e-12)
        np.testing.assert_allclose(dH, gold[f"losses_{name}_dH"], rtol=1e-10, atol=1e-12)
        # the streaming float32 path reproduces the fixture within the reference's tolerance
        np.testing.assert_allclose(orc.single_partition_logps(e, h, t, softcap=cap, vocab_chunk=5, sequence_chunk=4),
                                   gold[f"losses_{name}_logps"], atol=2e-6)
    for scale in (0.04, 1.5):
        w, hh, tok, g = stats_inputs(scale)
        for name, cap in (("none", None), ("cap30", 30.0)):
            key = f"stats_s{scale}_{name}"
            got = orc.single_partition_logps(w, hh, tok, softcap=cap, vocab_chunk=128, sequence_chunk=256)
            np.testing.assert_allclose(got, gold[f"{key}_logps"], atol=2e-5)
            np.testing.assert_allclose(orc.dense_normalization(w, hh, cap), gold[f"{key}_norm"], rtol=1e-12)
    e, h, t, wts = shard_inputs()
    lp, dE, dH = orc.logps_grads_f64(e, h, t, wts, 30.0)
    np.testing.assert_allclose(lp, gold["shard_logps"], rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(dE, gold["shard_dE"], rtol=1e-10, atol=1e-12)


def test_bf16_round_ties_to_even():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e38, 1e-40], np.float32)
    r = orc.bf16_round(x)
    ref = torch.tensor(x).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(r, ref)


def test_compaction_order():
    m = np.array([[1, 0, 1], [0, 0, 0], [1, 1, 0]], bool)
    np.testing.assert_array_equal(orc.compact_response(m), [0, 2, 6, 7])


@pytest.mark.parametrize("softcap", [None, 3.0])
def test_sampler_head_oracle_consistent_with_dense(softcap):
    rng = np.random.default_rng(17)
    w = orc.bf16_round(rng.normal(size=(23, 7)) * 0.7)
    h = orc.bf16_round(rng.normal(size=(5, 7)))
    z, full, norm, top, top_logp = orc.lm_head(w, h, softcap)
    y = rng.integers(0, 23, size=5)
    np.testing.assert_allclose(full[np.arange(5), y], orc.dense_logps(w, h, y, softcap), atol=1e-12)
    np.testing.assert_allclose(norm, orc.dense_normalization(w, h, softcap), rtol=1e-12)
    np.testing.assert_allclose(np.exp(full).sum(-1), 1.0, atol=1e-12)
    assert (z[np.arange(5), top] == z.max(-1)).all()
    np.testing.assert_allclose(top_logp, full.max(-1), atol=1e-12)


def test_top_k_top_p_keep_semantics():
    scores = np.log(np.array([[0.5, 0.1, 0.3, 0.1], [0.25, 0.25, 0.25, 0.25]]))
    keep = orc.top_k_top_p_keep(scores, 2, 1.0)
    assert keep.tolist() == [[True, False, True, False], [True, True, False, False]]
    # top_p 0.6 keeps the shortest descending prefix reaching 0.6 (0.5 < 0.6, 0.5+0.3 >= 0.6)
    keep = orc.top_k_top_p_keep(scores, 0, 0.6)
    assert keep.tolist() == [[True, False, True, False], [True, True, True, False]]
    # the most likely column is always kept
    assert orc.top_k_top_p_keep(scores, 0, 1e-9).sum(-1).tolist() == [1, 1]
