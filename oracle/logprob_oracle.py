"""Numpy restatement of the reference's native chunked logprob (TEST INFRASTRUCTURE ONLY).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may use
this module, and only as the checker. Every function names the reference lines it follows
(paths inside yixiaoer/gemma4-posttrain-jax).

Parity status: pinned to the reference tests' own relations (dense log-softmax for values
and gradients, dense max/sum-exp for the normalisation stats, vocab-parallel ==
single-partition) on the reference tests' seeded inputs. The reference itself (JAX) cannot
run in this image, so no reference-produced golden values exist.

Arithmetic: bf16 operands are widened to float32 exactly; products of two bf16 values are
exact in float32, and sums accumulate in float32, as ``_matmul_f32`` does with
``Precision.HIGHEST`` + ``preferred_element_type=float32`` (``losses.py:61-69``). The
backward is written analytically in float64 (``logps_grads_f64``) or as the reference's
recompute-per-tile structure in float32 (``fwd_bwd_f32``, the timed CPU baseline).
"""

from __future__ import annotations

import math

import numpy as np

_LOG2E = 1.4426950408889634


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even); return them as float32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    bias = ((u >> 16) & 1) + np.uint32(0x7FFF)
    return ((u + bias) & np.uint32(0xFFFF0000)).view(np.float32)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """The uint16 bit patterns of ``bf16_round(x)`` (what a bf16 device buffer holds)."""
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def _softcap(logits: np.ndarray, softcap: float | None) -> np.ndarray:
    """``losses.py:55-58``: c * tanh(z / c), identity when c is None."""
    if softcap is None:
        return logits
    return (np.tanh(logits / np.float32(softcap)) * np.float32(softcap)).astype(logits.dtype)


def _check_shapes(embed: np.ndarray, hidden: np.ndarray, targets: np.ndarray, vocab_chunk: int, sequence_chunk: int):
    """The three ``ValueError`` checks of ``losses.py:91-96`` / ``:281-286``, same messages."""
    if tuple(hidden.shape[:-1]) != tuple(targets.shape):
        raise ValueError(f"hidden prefix {hidden.shape[:-1]} does not match targets {targets.shape}")
    if embed.ndim != 2 or hidden.shape[-1] != embed.shape[-1]:
        raise ValueError(f"incompatible embedding {embed.shape} and hidden {hidden.shape}")
    if vocab_chunk <= 0 or sequence_chunk <= 0:
        raise ValueError("vocab_chunk and sequence_chunk must be positive")


def _blocked_stats(
    embed: np.ndarray,
    flat_hidden: np.ndarray,
    flat_targets: np.ndarray,
    *,
    softcap: float | None,
    vocab_chunk: int,
    sequence_chunk: int,
    vocab_offset: int = 0,
    owned_only: bool = False,
):
    """Token-block x vocab-block online log-sum-exp over one vocabulary partition.

    Follows ``losses.py:98-144`` (single partition) and the per-shard body of
    ``losses.py:199-248`` (vocab parallel): tokens padded to a ``sequence_chunk`` multiple,
    vocab padded to a ``vocab_chunk`` multiple with the tail masked to -inf, the target
    logit taken by a separate gather + row dot + softcap, and the running (max, sum)
    rescaled by exp(old_max - new_max) per vocab block. Returns float32 arrays
    (target_logit, running_max, running_sum) of length ``num_tokens``.
    """
    num_tokens, hidden_size = flat_hidden.shape
    vocab_size = embed.shape[0]
    n_seq = math.ceil(num_tokens / sequence_chunk) if num_tokens else 0
    n_voc = math.ceil(vocab_size / vocab_chunk)
    seq_pad = n_seq * sequence_chunk - num_tokens
    voc_pad = n_voc * vocab_chunk - vocab_size
    h = np.pad(np.asarray(flat_hidden, dtype=np.float32), ((0, seq_pad), (0, 0)))
    t = np.pad(flat_targets.astype(np.int64), ((0, seq_pad),))
    # The reference pads the table to a vocab_chunk multiple (losses.py:106); only the last
    # block needs the padding, so it is padded block by block instead of copying the table.
    e = np.asarray(embed, dtype=np.float32)
    del voc_pad
    tgt_out = np.zeros(n_seq * sequence_chunk, np.float32)
    max_out = np.zeros(n_seq * sequence_chunk, np.float32)
    sum_out = np.zeros(n_seq * sequence_chunk, np.float32)
    for sb in range(n_seq):
        rows = slice(sb * sequence_chunk, (sb + 1) * sequence_chunk)
        hb, tb = h[rows], t[rows]
        if owned_only:
            owned = (tb >= vocab_offset) & (tb < vocab_offset + vocab_size)
            local = np.clip(tb - vocab_offset, 0, vocab_size - 1)
        else:
            owned = np.ones_like(tb, dtype=bool)
            local = tb
        tgt = np.einsum("nm,nm->n", hb, embed[local].astype(np.float32), dtype=np.float32)
        tgt = _softcap(tgt, softcap)
        tgt_out[rows] = np.where(owned, tgt, np.float32(0.0))
        run_max = np.full(sequence_chunk, -np.inf, np.float32)
        run_sum = np.zeros(sequence_chunk, np.float32)
        for vb in range(n_voc):
            cols = slice(vb * vocab_chunk, (vb + 1) * vocab_chunk)
            blk = e[cols]
            if blk.shape[0] < vocab_chunk:
                blk = np.pad(blk, ((0, vocab_chunk - blk.shape[0]), (0, 0)))
            logits = _softcap(hb @ blk.T, softcap)
            valid = vb * vocab_chunk + np.arange(vocab_chunk) < vocab_size
            logits = np.where(valid[None, :], logits, np.float32(-np.inf))
            new_max = np.maximum(run_max, logits.max(axis=-1))
            run_sum = run_sum * np.exp(run_max - new_max)
            run_sum = run_sum + np.exp(logits - new_max[:, None]).sum(axis=-1, dtype=np.float32)
            run_max = new_max
        max_out[rows] = run_max
        sum_out[rows] = run_sum
    return tgt_out[:num_tokens], max_out[:num_tokens], sum_out[:num_tokens]


def single_partition_logps(
    embed: np.ndarray,
    hidden: np.ndarray,
    targets: np.ndarray,
    *,
    softcap: float | None,
    vocab_chunk: int = 8192,
    sequence_chunk: int = 256,
) -> np.ndarray:
    """``losses.py:72-147`` ``_single_partition_logps``: float32 target log-probabilities."""
    _check_shapes(embed, hidden, targets, vocab_chunk, sequence_chunk)
    out_shape = targets.shape
    flat_h = hidden.reshape(-1, hidden.shape[-1])
    flat_t = targets.reshape(-1)
    tgt, mx, sm = _blocked_stats(
        embed, flat_h, flat_t, softcap=softcap, vocab_chunk=vocab_chunk, sequence_chunk=sequence_chunk
    )
    return (tgt - (mx + np.log(sm))).astype(np.float32).reshape(out_shape)


def vocab_parallel_logps_and_normalization(
    embed: np.ndarray,
    hidden: np.ndarray,
    targets: np.ndarray,
    *,
    num_shards: int,
    softcap: float | None,
    vocab_chunk: int = 8192,
    sequence_chunk: int = 256,
):
    """``losses.py:172-260``: P vocab shards, owned-target psum, pmax / rescaled psum combine.

    Returns ``(values, normalization)`` with ``normalization[0]`` the global max and
    ``normalization[1]`` the global sum of exp(logit - max), shaped ``(2, *targets.shape)``.
    """
    _check_shapes(embed, hidden, targets, vocab_chunk, sequence_chunk)
    if embed.shape[0] % num_shards:
        raise ValueError(f"vocab size {embed.shape[0]} must be divisible by mesh axis {num_shards}")
    vs = embed.shape[0] // num_shards
    flat_h = hidden.reshape(-1, hidden.shape[-1])
    flat_t = targets.reshape(-1)
    parts = [
        _blocked_stats(
            embed[r * vs : (r + 1) * vs],
            flat_h,
            flat_t,
            softcap=softcap,
            vocab_chunk=vocab_chunk,
            sequence_chunk=sequence_chunk,
            vocab_offset=r * vs,
            owned_only=True,
        )
        for r in range(num_shards)
    ]
    tgt = np.sum([p[0] for p in parts], axis=0, dtype=np.float32)
    gmax = np.max([p[1] for p in parts], axis=0)
    gsum = np.sum([p[2] * np.exp(p[1] - gmax) for p in parts], axis=0, dtype=np.float32)
    values = (tgt - gmax - np.log(gsum)).astype(np.float32)
    norm = np.stack((gmax, gsum)).astype(np.float32)
    return values.reshape(targets.shape), norm.reshape((2, *targets.shape))


def per_token_logps(
    embed: np.ndarray,
    hidden: np.ndarray,
    targets: np.ndarray,
    *,
    softcap: float | None,
    vocab_chunk: int = 8192,
    sequence_chunk: int = 256,
    num_shards: int = 1,
) -> np.ndarray:
    """``losses.py:263-304`` dispatch: vocab-parallel when more than one shard, else single partition."""
    if num_shards > 1:
        return vocab_parallel_logps_and_normalization(
            embed,
            hidden,
            targets,
            num_shards=num_shards,
            softcap=softcap,
            vocab_chunk=vocab_chunk,
            sequence_chunk=sequence_chunk,
        )[0]
    return single_partition_logps(
        embed, hidden, targets, softcap=softcap, vocab_chunk=vocab_chunk, sequence_chunk=sequence_chunk
    )


def dense_logps(embed: np.ndarray, hidden: np.ndarray, targets: np.ndarray, softcap: float | None) -> np.ndarray:
    """The reference tests' dense oracle (``tests/test_losses.py:13-17``), in float64."""
    h = hidden.reshape(-1, hidden.shape[-1]).astype(np.float64)
    logits = h @ embed.astype(np.float64).T
    if softcap is not None:
        logits = np.tanh(logits / softcap) * softcap
    m = logits.max(axis=-1, keepdims=True)
    lse = m[:, 0] + np.log(np.exp(logits - m).sum(axis=-1))
    t = targets.reshape(-1)
    return (logits[np.arange(t.size), t] - lse).reshape(targets.shape)


def dense_normalization(embed: np.ndarray, hidden: np.ndarray, softcap: float | None) -> np.ndarray:
    """Dense (max, sum exp(logit - max)) per token, ``tests/test_native_logprob_stats.py:53-58``."""
    h = hidden.reshape(-1, hidden.shape[-1]).astype(np.float64)
    logits = h @ embed.astype(np.float64).T
    if softcap is not None:
        logits = np.tanh(logits / softcap) * softcap
    m = logits.max(axis=-1)
    s = np.exp(logits - m[:, None]).sum(axis=-1)
    return np.stack((m, s)).reshape((2, *hidden.shape[:-1]))


def logps_grads_f64(
    embed: np.ndarray,
    hidden: np.ndarray,
    targets: np.ndarray,
    g: np.ndarray,
    softcap: float | None,
    *,
    vocab_block: int = 16384,
    want_dw: bool = True,
):
    """Analytic VJP of the logprob path in float64: returns ``(logp, dW, dH)`` (dW is None
    with ``want_dw=False``, which checks sampled rows of a large vocabulary cheaply).

    With x = h . w_v, z = softcap(x), p = softmax(z):
      d logp_t / d z_tv = 1[v = y_t] - p_tv          (the max shift has no gradient,
                                                       ``losses.py:241-243``)
      d z / d x = 1 - tanh(x / c)^2                   (``_softcap`` chain rule)
      dH = dX . W,  dW = dX^T . H,  dX = g * (onehot - p) * (1 - tanh^2)
    This is what JAX AD through the checkpointed scans computes (``losses.py:141``),
    accumulated in float64 instead of the reference's float32/bf16.
    """
    d = hidden.shape[-1]
    h = hidden.reshape(-1, d).astype(np.float64)
    t = targets.reshape(-1).astype(np.int64)
    gg = g.reshape(-1).astype(np.float64)
    e = embed.astype(np.float64)
    V = e.shape[0]
    T = h.shape[0]
    # pass 1: log normaliser
    run_max = np.full(T, -np.inf)
    run_sum = np.zeros(T)
    for v0 in range(0, V, vocab_block):
        x = h @ e[v0 : v0 + vocab_block].T
        z = np.tanh(x / softcap) * softcap if softcap is not None else x
        nm = np.maximum(run_max, z.max(axis=1))
        run_sum = run_sum * np.exp(run_max - nm) + np.exp(z - nm[:, None]).sum(axis=1)
        run_max = nm
    lse = run_max + np.log(run_sum)
    xt = np.einsum("nm,nm->n", h, e[t])
    zt = np.tanh(xt / softcap) * softcap if softcap is not None else xt
    logp = zt - lse
    # pass 2: gradients
    dH = np.zeros_like(h)
    dW = np.zeros_like(e) if want_dw else None
    rows = np.arange(T)
    for v0 in range(0, V, vocab_block):
        x = h @ e[v0 : v0 + vocab_block].T
        if softcap is not None:
            th = np.tanh(x / softcap)
            z = th * softcap
            chain = 1.0 - th * th
        else:
            z = x
            chain = 1.0
        dz = -np.exp(z - lse[:, None])
        inblk = (t >= v0) & (t < v0 + x.shape[1])
        dz[rows[inblk], t[inblk] - v0] += 1.0
        dx = gg[:, None] * dz * chain
        dH += dx @ e[v0 : v0 + vocab_block]
        if want_dw:
            dW[v0 : v0 + vocab_block] += dx.T @ h
    return logp.reshape(targets.shape), dW, dH.reshape(hidden.shape)


def fwd_bwd_f32(
    embed: np.ndarray,
    hidden: np.ndarray,
    targets: np.ndarray,
    g: np.ndarray,
    *,
    softcap: float | None,
    vocab_chunk: int = 8192,
    sequence_chunk: int = 256,
):
    """The reference's native fwd + recompute bwd structure in float32 (the timed CPU baseline).

    Forward: ``_blocked_stats`` (``losses.py:98-147``). Backward: for every token block and
    vocab block the logits tile is recomputed (the ``jax.checkpoint`` of ``losses.py:141``),
    dZ formed from the saved (max, sum), then dH += dZ . W_blk and dW_blk += dZ^T . H_blk,
    plus the target-gather term. Returns ``(logp, dW, dH)`` float32.
    """
    d = hidden.shape[-1]
    h = np.asarray(hidden, dtype=np.float32).reshape(-1, d)
    t = targets.reshape(-1).astype(np.int64)
    gg = g.reshape(-1).astype(np.float32)
    e = np.asarray(embed, dtype=np.float32)
    V = e.shape[0]
    T = h.shape[0]
    tgt, mx, sm = _blocked_stats(e, h, t, softcap=softcap, vocab_chunk=vocab_chunk, sequence_chunk=sequence_chunk)
    lse = (mx + np.log(sm)).astype(np.float32)
    logp = tgt - lse
    dH = np.zeros_like(h)
    dW = np.zeros_like(e)
    for s0 in range(0, T, sequence_chunk):
        rows = slice(s0, min(T, s0 + sequence_chunk))
        hb, tb, gb, lb = h[rows], t[rows], gg[rows], lse[rows]
        for v0 in range(0, V, vocab_chunk):
            x = hb @ e[v0 : v0 + vocab_chunk].T
            if softcap is not None:
                th = np.tanh(x / np.float32(softcap))
                z = th * np.float32(softcap)
                chain = np.float32(1.0) - th * th
            else:
                z = x
                chain = None
            dz = -np.exp(z - lb[:, None]) * gb[:, None]
            if chain is not None:
                dz *= chain
            dH[rows] += dz @ e[v0 : v0 + vocab_chunk]
            dW[v0 : v0 + vocab_chunk] += dz.T @ hb
        # target term (transpose of the gather + row dot): g * dz/dx at the target
        xt = np.einsum("nm,nm->n", hb, e[tb])
        ct = (np.float32(1.0) - np.tanh(xt / np.float32(softcap)) ** 2) if softcap is not None else np.float32(1.0)
        coef = (gb * ct).astype(np.float32)
        dH[rows] += coef[:, None] * e[tb]
        np.add.at(dW, tb, coef[:, None] * hb)
    return logp.reshape(targets.shape), dW, dH.reshape(hidden.shape)


def compact_response(completion_mask: np.ndarray):
    """Row-major indices of valid response slots (the compaction the CUDA path performs).

    The reference computes every padded slot and zeroes invalid ones afterwards
    (``losses.py:667-682``); compaction keeps only ``completion_mask`` slots, in the same
    flattened [B, N] order, so logps scattered back match ``where(mask, logps, 0)``.
    """
    flat = np.asarray(completion_mask).reshape(-1).astype(bool)
    return np.nonzero(flat)[0].astype(np.int64)


def lm_head(embed: np.ndarray, hidden: np.ndarray, softcap: float | None):
    """Sampler head: ``forward_lm_head`` (``model.py:676-680``) then the full log-softmax and
    greedy pick of ``_sample_token`` (``sampler.py:150-161,184``), in float64.

    Returns (logits [B, V], full_logps [B, V], (max, sum exp(z - max)) [2, B], argmax [B]
    (first column of the row maximum, as ``jnp.argmax``), logp of the argmax [B]).
    """
    h = hidden.reshape(-1, hidden.shape[-1]).astype(np.float64)
    logits = h @ embed.astype(np.float64).T
    if softcap is not None:
        logits = np.tanh(logits / softcap) * softcap
    m = logits.max(axis=-1)
    s = np.exp(logits - m[:, None]).sum(axis=-1)
    full = logits - (m + np.log(s))[:, None]
    top = logits.argmax(axis=-1)
    return logits, full, np.stack((m, s)), top, full[np.arange(top.size), top]


def top_k_top_p_keep(scores: np.ndarray, top_k: int, top_p: float) -> np.ndarray:
    """Boolean [B, V] of the columns ``_sample_token`` may sample (``sampler.py:162-181``):
    the ``top_k`` largest scores (0 or >= V: all), then within them (or within all columns,
    sorted descending, stable) the shortest prefix whose probability reaches ``top_p``; the
    most likely column is always kept."""
    B, V = scores.shape
    order = np.argsort(-scores, axis=-1, kind="stable")
    if 0 < top_k < V:
        order = order[:, :top_k]
    keep = np.zeros((B, V), dtype=bool)
    for b in range(B):
        cols = order[b]
        if top_p < 1:
            sc = scores[b, cols].astype(np.float64)
            w = np.exp(sc - sc.max())
            p = w / w.sum()
            prev = np.concatenate(([0.0], np.cumsum(p)[:-1]))
            cols = cols[(prev < top_p) | (np.arange(cols.size) == 0)]
        keep[b, cols] = True
    return keep
