"""The rollout sampler's LM head on the B200 kernels.

Mirrors ``forward_lm_head`` (``gemma4_posttrain_jax/model.py:676-680``: logits of the
tied head with the final softcap) and ``_sample_token``
(``gemma4_posttrain_jax/sampler.py:145-184``: full f32 log-softmax, greedy or
temperature / top-k / top-p sampling, and the logp of the chosen token under the full
policy). The head itself -- one tensor-core GEMM over the whole vocabulary with the softcap,
a running log-sum-exp and the row argmax fused into its epilogue -- is ``lp_head``; greedy
decoding never writes the [B, V] logits. The random draw of the stochastic modes uses
torch's sampler on the device (the reference draws with ``jax.random.categorical``, so
the two do not produce the same token stream for a given seed; the distribution is the
same).
"""

from __future__ import annotations

import torch

from . import ops


def _rows_of(hidden: torch.Tensor) -> torch.Tensor:
    if hidden.ndim < 1:
        raise ValueError("hidden must have a trailing feature axis")
    return hidden.reshape(-1, hidden.shape[-1])


def lm_head_logits(
    embed_tokens: torch.Tensor, hidden: torch.Tensor, softcap: float | None, *, log_probs: bool = False
) -> torch.Tensor:
    """``forward_lm_head``: hidden [..., d] -> float32 logits [..., V] (softcapped).

    ``log_probs=True`` returns the full log-softmax instead (the ``full_logps`` of
    ``_sample_token``, ``sampler.py:153-158``).
    """
    if embed_tokens.ndim != 2 or hidden.shape[-1] != embed_tokens.shape[-1]:
        raise ValueError(f"incompatible embedding {tuple(embed_tokens.shape)} and hidden {tuple(hidden.shape)}")
    h = _rows_of(hidden)
    logits, _, _, _ = ops.head(embed_tokens, h, softcap, want_logits=True, log_probs=log_probs)
    return logits.reshape(*hidden.shape[:-1], embed_tokens.shape[0])


def sample_token(
    embed_tokens: torch.Tensor,
    hidden: torch.Tensor,
    softcap: float | None,
    *,
    temperature: float,
    top_k: int,
    top_p: float = 1.0,
    generator: torch.Generator | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """``_sample_token`` on the last-position hidden states [B, d]: (token int32 [B], logp [B]).

    temperature <= 0 is greedy (first maximal logit, no logits written); otherwise the
    scores ``logits / temperature`` are restricted to the ``top_k`` largest (when
    0 < top_k < V) and then, when top_p < 1, to the shortest descending prefix whose
    probability reaches top_p (the most likely column is always kept), and a token is drawn
    from the remaining softmax. logp is the token's log-probability under the full,
    untempered policy, as in the reference.
    """
    if hidden.ndim != 2:
        raise ValueError(f"hidden must be [B, d], got {tuple(hidden.shape)}")
    if embed_tokens.ndim != 2 or hidden.shape[-1] != embed_tokens.shape[-1]:
        raise ValueError(f"incompatible embedding {tuple(embed_tokens.shape)} and hidden {tuple(hidden.shape)}")
    if not 0.0 < top_p <= 1.0:
        raise ValueError("top_p must be in (0, 1]")
    if temperature <= 0:
        _, _, top, top_logp = ops.head(embed_tokens, hidden, softcap, want_logits=False)
        return top, top_logp
    logits, norm, _, _ = ops.head(embed_tokens, hidden, softcap, want_logits=True)
    V = logits.shape[-1]
    scores = logits / float(temperature)
    indices = None
    if 0 < top_k < V:
        scores, indices = torch.topk(scores, top_k, dim=-1, largest=True, sorted=True)
    elif top_p < 1:
        scores, indices = torch.sort(scores, dim=-1, descending=True, stable=True)
    if top_p < 1:
        probs = torch.softmax(scores, dim=-1)
        previous = torch.cumsum(probs, dim=-1) - probs
        keep = previous < top_p
        keep[:, 0] = True
        scores = scores.masked_fill(~keep, float("-inf"))
    selected = torch.multinomial(torch.softmax(scores, dim=-1), 1, generator=generator)[:, 0]
    token = selected if indices is None else torch.gather(indices, 1, selected[:, None])[:, 0]
    lse = norm[0] + torch.log(norm[1])
    logp = torch.gather(logits, 1, token[:, None])[:, 0] - lse
    return token.to(torch.int32), logp
