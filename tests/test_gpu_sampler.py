"""Sampler LM head (lp_head) vs the CPU oracle: logits, full log-softmax, normaliser, greedy
token and its logp, and the stochastic sampling modes of ``_sample_token``
(``gemma4_posttrain_jax/sampler.py:145-184``) on top of it."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import logprob_oracle as orc

pytestmark = pytest.mark.gpu

LOGP_ATOL = 2e-3


def _inputs(dev, B, V, d, scale, seed):
    rng = np.random.default_rng(seed)
    w = orc.bf16_round(rng.normal(size=(V, d)) * scale)
    h = orc.bf16_round(rng.normal(size=(B, d)))
    W = torch.from_numpy(w).to(dev).to(torch.bfloat16)
    H = torch.from_numpy(h).to(dev).to(torch.bfloat16)
    return w, h, W, H


@pytest.mark.parametrize(
    "B,V,d,scale,softcap",
    [
        (1, 1036, 128, 1.5, 30.0),  # one decode row, vocabulary tail
        (37, 4099, 136, 0.7, 30.0),  # ragged rows, vocabulary and K tails
        (130, 70001, 256, 0.3, None),  # two M tiles, no softcap, odd V (padded logits rows)
        (16, 262144, 2048, 0.02, 30.0),  # the full head (BASELINE V, d)
    ],
)
def test_head_matches_oracle(cuda_device, B, V, d, scale, softcap):
    from gemma4_posttrain_jax_b200 import _lib, ops

    w, h, W, H = _inputs(cuda_device, B, V, d, scale, seed=B * 7 + V)
    logits, norm, top, top_logp = ops.head(W, H, softcap)
    lp_full, _, _, _ = ops.head(W, H, softcap, log_probs=True)
    g_top, g_logp = ops.head(W, H, softcap, want_logits=False)[2:]
    torch.cuda.synchronize()
    assert _lib.device_error(0) == 0
    z, full, nrm, top_ref, top_logp_ref = orc.lm_head(w, h, softcap)
    zg = logits.cpu().numpy()
    err_z = float(np.abs(zg - z).max())
    err_full = float(np.abs(lp_full.cpu().numpy() - full).max())
    tg = top.cpu().numpy()
    print(f"B={B} V={V} d={d}: logits max abs {err_z:.2e}, log-probs max abs {err_full:.2e}")
    assert err_z <= 2e-4 + 1e-4 * float(np.abs(z).max())
    assert err_full <= LOGP_ATOL
    np.testing.assert_allclose(norm[0].cpu().numpy(), nrm[0], atol=2e-4, rtol=2e-5)
    np.testing.assert_allclose(norm[1].cpu().numpy(), nrm[1], rtol=1e-4)
    # greedy: the oracle's argmax, unless two logits tie within the kernel's rounding
    rows = np.arange(B)
    assert (z[rows, tg] >= z[rows, top_ref] - 1e-4).all()
    assert (tg == top_ref).mean() >= 0.95
    assert np.abs(top_logp.cpu().numpy() - full[rows, tg]).max() <= LOGP_ATOL
    # the greedy-only launch (no logits written) gives the same token and logp
    assert torch.equal(g_top, top) and torch.equal(g_logp, top_logp)


def test_head_ties_pick_the_first_column(cuda_device):
    from gemma4_posttrain_jax_b200 import ops

    V, d = 3000, 64
    w = np.zeros((V, d), np.float32)
    w[[7, 700, 2999], 0] = 2.0  # three identical maximal logits per row
    h = np.ones((5, d), np.float32)
    W = torch.from_numpy(w).to(cuda_device).to(torch.bfloat16)
    H = torch.from_numpy(h).to(cuda_device).to(torch.bfloat16)
    _, _, top, _ = ops.head(W, H, 30.0, want_logits=False)
    assert top.cpu().tolist() == [7] * 5


def test_sample_token_modes(cuda_device):
    from gemma4_posttrain_jax_b200 import lm_head_logits, sample_token

    B, V, d = 24, 5003, 128
    w, h, W, H = _inputs(cuda_device, B, V, d, 0.8, seed=11)
    z, full, _, top_ref, top_logp_ref = orc.lm_head(w, h, 30.0)
    gen = torch.Generator(device=cuda_device).manual_seed(3)
    tok, lp = sample_token(W, H, 30.0, temperature=0.0, top_k=0)
    assert (tok.cpu().numpy() == top_ref).all()
    assert np.abs(lp.cpu().numpy() - top_logp_ref).max() <= LOGP_ATOL
    # top_k = 1 and a tiny top_p both reduce to the greedy token
    tok1, _ = sample_token(W, H, 30.0, temperature=0.7, top_k=1, generator=gen)
    assert (tok1.cpu().numpy() == top_ref).all()
    tokp, _ = sample_token(W, H, 30.0, temperature=0.7, top_k=0, top_p=1e-6, generator=gen)
    assert (tokp.cpu().numpy() == top_ref).all()
    # sampled tokens stay inside the kept set; logp is the untempered full log-softmax
    for top_k, top_p in ((40, 1.0), (0, 0.9), (200, 0.5)):
        keep = orc.top_k_top_p_keep(z / 0.7, top_k, top_p)
        for _ in range(3):
            t, l = sample_token(W, H, 30.0, temperature=0.7, top_k=top_k, top_p=top_p, generator=gen)
            t = t.cpu().numpy()
            assert keep[np.arange(B), t].all()
            assert np.abs(l.cpu().numpy() - full[np.arange(B), t]).max() <= LOGP_ATOL
    # lm_head_logits keeps the leading shape
    out = lm_head_logits(W, H.reshape(4, 6, d), 30.0)
    assert out.shape == (4, 6, V)
    assert float(np.abs(out.reshape(B, V).cpu().numpy() - z).max()) <= 1e-3


def test_sampler_argument_errors(cuda_device):
    from gemma4_posttrain_jax_b200 import ops, sample_token

    _, _, W, H = _inputs(cuda_device, 4, 300, 64, 0.5, seed=1)
    with pytest.raises(ValueError, match=r"\[B, d\]"):
        sample_token(W, H.reshape(2, 2, 64), None, temperature=1.0, top_k=0)
    with pytest.raises(ValueError, match="top_p"):
        sample_token(W, H, None, temperature=1.0, top_k=0, top_p=0.0)
    with pytest.raises(ValueError, match="log_probs"):
        ops.head(W, H, None, want_logits=False, log_probs=True)


@pytest.mark.parametrize(
    "temperature,top_k,top_p",
    [(1.0, 0, 1.0), (0.7, 0, 1.0), (0.8, 3, 1.0), (0.8, 0, 0.85), (0.8, 4, 0.7), (0.8, 0, 1e-50)],
)
def test_sampling_distribution_matches_transformers_warpers(cuda_device, temperature, top_k, top_p):
    """The reference's distribution test (``tests/test_sampler.py:175-205``): transformers'
    temperature / top-k / top-p warpers give the expected distribution independently; 8192
    draws per row must match it within 0.025 and never leave its support, and the recorded
    logp is the untempered full log-softmax. The head reproduces the given logits exactly:
    hidden = e_0 and W[v, 0] = logit (bf16-rounded)."""
    from transformers.generation.logits_process import TemperatureLogitsWarper, TopKLogitsWarper, TopPLogitsWarper

    from gemma4_posttrain_jax_b200 import sample_token

    logits = orc.bf16_round(np.array([[1.1, -0.7, 0.3, 2.0, -2.0], [-1.0, 1.3, 0.6, -2.3, 0.1]], np.float32))
    V, d, count = logits.shape[1], 8, 8192
    gen = torch.Generator(device=cuda_device).manual_seed(128)
    H = torch.zeros((count, d), dtype=torch.bfloat16, device=cuda_device)
    H[:, 0] = 1.0
    for row in range(2):
        w = np.zeros((V, d), np.float32)
        w[:, 0] = logits[row]
        W = torch.from_numpy(w).to(cuda_device).to(torch.bfloat16)
        scores = TemperatureLogitsWarper(temperature)(None, torch.from_numpy(logits[row : row + 1]))
        if top_k:
            scores = TopKLogitsWarper(top_k)(None, scores)
        if top_p < 1:
            scores = TopPLogitsWarper(top_p)(None, scores)
        expected = torch.softmax(scores, dim=-1)[0].numpy()
        raw = torch.log_softmax(torch.from_numpy(logits[row]).double(), dim=-1).numpy()
        tokens, logps = sample_token(W, H, None, temperature=temperature, top_k=top_k, top_p=top_p, generator=gen)
        t = tokens.cpu().numpy()
        assert np.all(expected[t] > 0), "sampled a token outside the filtered support"
        np.testing.assert_allclose(np.bincount(t, minlength=V) / count, expected, atol=0.025, rtol=0)
        np.testing.assert_allclose(logps.cpu().numpy(), raw[t], atol=1e-5, rtol=0)


def test_top_p_keeps_the_threshold_crossing_token(cuda_device):
    """``tests/test_sampler.py:208-218``: probabilities (0.5, 0.3, 0.2) with top_p 0.6 keep the
    first two columns (0.5 + 0.3 crosses 0.6), sampled 0.625 / 0.375."""
    from gemma4_posttrain_jax_b200 import sample_token

    V, d, count = 3, 8, 8192
    w = np.zeros((V, d), np.float32)
    w[:, 0] = orc.bf16_round(np.log(np.array([0.5, 0.3, 0.2], np.float32)))
    W = torch.from_numpy(w).to(cuda_device).to(torch.bfloat16)
    H = torch.zeros((count, d), dtype=torch.bfloat16, device=cuda_device)
    H[:, 0] = 1.0
    gen = torch.Generator(device=cuda_device).manual_seed(29)
    tokens, _ = sample_token(W, H, None, temperature=1.0, top_k=0, top_p=0.6, generator=gen)
    t = tokens.cpu().numpy()
    assert set(t.tolist()) == {0, 1}
    assert abs(float((t == 0).mean()) - 0.625) <= 0.025


@pytest.mark.parametrize("top_p", [0.0, -0.5, 1.01, float("nan"), float("inf")])
def test_invalid_top_p_is_rejected(cuda_device, top_p):
    """``tests/test_sampler.py:221-228``."""
    from gemma4_posttrain_jax_b200 import sample_token

    _, _, W, H = _inputs(cuda_device, 2, 300, 64, 0.5, seed=2)
    with pytest.raises(ValueError, match="top_p"):
        sample_token(W, H, None, temperature=1.0, top_k=0, top_p=top_p)
