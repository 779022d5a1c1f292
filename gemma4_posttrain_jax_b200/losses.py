"""The reference's logprob-backend interface, served by the B200 kernels.

``per_token_logps`` keeps the signature, argument meaning and error behaviour of
``gemma4_posttrain_jax/losses.py:307-343`` and adds ``backend="cuda"``: a
``torch.autograd.Function`` (the analogue of the reference's ``jax.custom_vjp``,
``pallas/lm_head_logprob_tpuv4.py:69-94``) whose forward runs ``lp_fwd`` (``lp_fwd_sum``,
or NCCL all-gather + ``lp_combine``, when the vocabulary is sharded) and whose backward
runs ``lp_bwd`` (+ the dH sum over shards). The callers on the path are mirrored too:
``sft_token_logps`` (the shift of ``losses.py:910-926``) and ``completion_logps`` (the
response slice of ``losses.py:667-682``, with the padded slots compacted away).

There is no fallback: other backends raise, CPU tensors raise, a missing library raises.
"""

from __future__ import annotations

import math
import os

import torch

from . import _lib, ops
from .phase_timer import phase
from .sharding import (
    VocabMesh,
    all_gather_stats,
    all_reduce_sum,
    dh_sum_buffer,
    peer_timeout_ms,
    poison,
    stats_exchange,
    vocab_offset,
)


# A backward skips the rows whose upstream gradient is exactly zero (they add nothing to dH
# or dW) when at least this fraction of the rows are zero; the reference's Pallas backward
# skips all-zero 256-row blocks the same way (pallas/lm_head_logprob_tpuv4.py:185-193).
_SKIP_ZERO_GRAD_MIN_FRACTION = 0.01


def _check_device(device: torch.device, where: str) -> None:
    """Raise if a kernel that has completed on ``device`` recorded a device-side error. Costs
    a host load, no CUDA call: used right after the host has waited for the stream anyway."""
    _lib.raise_on_device_error(device.index if device.index is not None else torch.cuda.current_device(), where)


def _check_mesh_call(device: torch.device, mesh: VocabMesh, where: str) -> None:
    """Wait for the current stream and raise if one of its kernels gave up waiting for another
    rank (its outputs hold NaN where a result was missing). The mesh's multicast buffers are
    then out of step between ranks, so they are marked unusable."""
    torch.cuda.current_stream(device).synchronize()
    try:
        _check_device(device, where)
    except _lib.DeviceTimeoutError:
        poison(mesh, device)
        raise


def _debug_checks() -> bool:
    return os.environ.get("LP_B200_DEBUG", "0") not in ("", "0")


def _nonzero_grad_rows(g: torch.Tensor):
    """Compaction of the rows with g != 0: (idx [m] int32, pos [n] int32, m) or None when dense.

    pos[i] is the compact row of row i, or -1 where g[i] == 0. One device-to-host read of m.
    """
    n = g.numel()
    if n == 0:
        return None
    mask = (g != 0).view(1, n)
    _, _, idx, pos, count = ops.compact(mask)
    m = int(count.item())
    _check_device(g.device, "backward")  # the forward and everything before it have completed
    if n - m < _SKIP_ZERO_GRAD_MIN_FRACTION * n:
        return None
    return idx[:m], pos, m


def _gather_rows(src: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    """src rows at idx (a row gather through lp_scatter_rows); src is [n] or [n, w]."""
    out = torch.empty((idx.numel(), *src.shape[1:]), dtype=src.dtype, device=src.device)
    return ops.scatter_rows(src.contiguous(), idx, out)


def _backward_rows(embed, H, y, softcap, norm, g, *, mesh, vocab_offset, need_dh, need_dw, dh_dtype, dw_dtype,
                   token_chunk, skip_zero_grad):
    """shard_backward on the rows with nonzero g, with the dH partials summed over the mesh.

    Returns (dH rows in compact order or None, dW, pos, shared): pos maps every row to its dH
    row (-1 = zero row), or is None (dense). With more than one shard the sum runs inside the
    dH GEMM through the mesh's NVLS multicast buffer when available -- dH is then a view of
    that buffer (``shared`` True: copy it out before the next backward) -- else as an
    all-reduce after the GEMM.
    """
    sel = _nonzero_grad_rows(g) if skip_zero_grad else None
    if sel is None:
        idx = pos = None
        rows = H.reshape(-1, H.shape[-1]).shape[0]
    else:
        idx, pos, rows = sel
        if rows == 0:
            dW = torch.zeros(embed.shape, dtype=dw_dtype, device=embed.device) if need_dw else None
            dH = torch.zeros((0, H.shape[-1]), dtype=dh_dtype, device=H.device) if need_dh else None
            return dH, dW, pos, False
    if idx is not None:
        Hz = _gather_rows(H.reshape(-1, H.shape[-1]), idx)
        yz = _gather_rows(y.reshape(-1).to(torch.int32).view(torch.float32), idx).view(torch.int32)
        gz = _gather_rows(g.reshape(-1).to(torch.float32), idx)
        nz = torch.stack([_gather_rows(norm[0].contiguous(), idx), _gather_rows(norm[1].contiguous(), idx)])
    else:
        Hz, yz, gz, nz = H, y, g, norm
    P = mesh.size if mesh is not None else 1
    buf = dh_sum_buffer(mesh, rows, H.shape[-1], H.device) if (need_dh and P > 1) else None
    if buf is not None:
        timeout = peer_timeout_ms()
        # No barrier before the call: the counters are zero (zeroed at creation, and after each
        # call, below), and another rank's sums reach this rank's dH copy only after this rank
        # has started the call's dH GEMM, i.e. after it has consumed the previous dH.
        dH, dW = ops.shard_backward(embed, Hz, yz, softcap, nz, gz, vocab_offset=vocab_offset, need_dh=True,
                                    need_dw=need_dw, dh_dtype=torch.bfloat16, dw_dtype=dw_dtype,
                                    token_chunk=token_chunk, dh_mesh_sum=buf)
        # Every rank reduces a share of every row block, so this rank's counters reached their
        # final counts inside its dH GEMM: zeroed now, before the barrier that the next call's
        # increments follow, they start the next call at zero.
        buf.counters[: int(ops.bwd_sum_counters(rows))].zero_()
        with phase("dh_peer_barrier"):
            ops.peer_barrier(buf, timeout)  # every rank's share of the sum has landed everywhere
        _check_mesh_call(H.device, mesh, "lp_bwd_sum (dH summed over the mesh)")
        return dH, dW, pos, True
    dH, dW = ops.shard_backward(embed, Hz, yz, softcap, nz, gz, vocab_offset=vocab_offset, need_dh=need_dh,
                                need_dw=need_dw, dh_dtype=dh_dtype, dw_dtype=dw_dtype, token_chunk=token_chunk)
    if dH is not None and P > 1:
        with phase("dh_all_reduce"):
            all_reduce_sum(dH, mesh)
    return dH, dW, pos, False


def _mesh_forward(embed, H, y, softcap, mesh, off):
    """Global (logp, normalization) of rows H over the vocabulary mesh: the pmax / psum
    combine of ``losses.py:219,243-245``, exchanged over NVLink inside the forward
    (``lp_fwd_sum``) where the mesh has a multicast buffer, else NCCL all-gather + combine."""
    xch = stats_exchange(mesh, H.shape[0], H.device)
    if xch is not None:
        out = ops.shard_forward_sum(embed, H, y, softcap, xch, vocab_offset=off, timeout_ms=peer_timeout_ms())
        _check_mesh_call(H.device, mesh, "lp_fwd_sum (triples exchanged over the mesh)")
        return out
    stats, _ = ops.shard_forward(embed, H, y, softcap, vocab_offset=off, want_logp=False)
    with phase("stats_all_gather"):
        gathered = all_gather_stats(stats, mesh)
    return ops.combine(gathered)


def _validate(embed: torch.Tensor, hidden: torch.Tensor, targets: torch.Tensor, vocab_chunk: int, sequence_chunk: int):
    """The three argument checks of ``losses.py:281-286``, same messages."""
    if tuple(hidden.shape[:-1]) != tuple(targets.shape):
        raise ValueError(f"hidden prefix {tuple(hidden.shape[:-1])} does not match targets {tuple(targets.shape)}")
    if embed.ndim != 2 or hidden.shape[-1] != embed.shape[-1]:
        raise ValueError(f"incompatible embedding {tuple(embed.shape)} and hidden {tuple(hidden.shape)}")
    if vocab_chunk <= 0 or sequence_chunk <= 0:
        raise ValueError("vocab_chunk and sequence_chunk must be positive")


def _validate_softcap(softcap: float | None) -> None:
    if softcap is not None and (not math.isfinite(softcap) or softcap <= 0):
        raise ValueError("softcap must be finite and positive, or None")


class _CudaTokenLogps(torch.autograd.Function):
    """logp[t] of targets under softcap(H . W^T); grads for W (local shard) and H."""

    @staticmethod
    def forward(ctx, embed, hidden2d, targets1d, softcap, mesh, token_chunk, stats_out, dh_reduce_f32=False,
                skip_zero_grad=True):
        P = mesh.size if mesh is not None else 1
        if P > 1:
            off = vocab_offset(embed.shape[0], mesh)
            logp, norm = _mesh_forward(embed, hidden2d, targets1d, softcap, mesh, off)
        else:
            off = 0
            stats, logp = ops.shard_forward(embed, hidden2d, targets1d, softcap, want_logp=True)
            norm = stats[:2]
        if stats_out is not None:
            stats_out.append(norm)
        ctx.save_for_backward(embed, hidden2d, targets1d, norm)
        ctx.softcap = softcap
        ctx.mesh = mesh
        ctx.offset = off
        ctx.token_chunk = token_chunk
        ctx.dh_reduce_f32 = dh_reduce_f32
        ctx.skip_zero_grad = skip_zero_grad
        ctx.mark_non_differentiable(norm)
        return logp

    @staticmethod
    def backward(ctx, g):
        embed, hidden2d, targets1d, norm = ctx.saved_tensors
        mesh: VocabMesh | None = ctx.mesh
        P = mesh.size if mesh is not None else 1
        need_dw, need_dh = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        if not (need_dw or need_dh):
            return None, None, None, None, None, None, None, None, None
        # Shards sum their dH partials in the hidden dtype, as the reference's psum of the
        # bf16 cotangent does (losses.py:253-259 transposed); dh_reduce_f32 sums in f32 instead.
        dh_dtype = torch.float32 if (P > 1 and ctx.dh_reduce_f32) else torch.bfloat16
        dH, dW, pos, shared = _backward_rows(
            embed,
            hidden2d,
            targets1d,
            ctx.softcap,
            norm,
            g,
            mesh=mesh,
            vocab_offset=ctx.offset,
            need_dh=need_dh,
            need_dw=need_dw,
            dh_dtype=dh_dtype,
            dw_dtype=embed.dtype if embed.dtype in (torch.bfloat16, torch.float32) else torch.float32,
            token_chunk=ctx.token_chunk,
            skip_zero_grad=ctx.skip_zero_grad,
        )
        if dH is not None and pos is not None:
            # back to one row per token: rows with zero upstream gradient get zero
            full = torch.empty(hidden2d.shape, dtype=hidden2d.dtype, device=hidden2d.device)
            dH = ops.scatter_rows(dH, pos, full)
        elif dH is not None and (dH.dtype != hidden2d.dtype or shared):
            dH = dH.to(hidden2d.dtype, copy=True)
        return dW, dH, None, None, None, None, None, None, None


def per_token_logps(
    embed_tokens: torch.Tensor,
    hidden: torch.Tensor,
    targets: torch.Tensor,
    *,
    softcap: float | None,
    vocab_chunk: int = 8192,
    sequence_chunk: int = 256,
    mesh: VocabMesh | None = None,
    backend: str = "cuda",
    token_chunk: int | None = None,
    normalization_out: list | None = None,
    dh_reduce_f32: bool = False,
    skip_zero_grad: bool = True,
) -> torch.Tensor:
    """Selected-token log-probabilities without materialising ``[..., vocab]`` logits.

    Same contract as ``gemma4_posttrain_jax/losses.py:307-343``. With a ``mesh`` of size
    > 1, ``embed_tokens`` is this rank's row block (``V / mesh.size`` rows, the
    ``P("d", None)`` layout) and ``hidden`` / ``targets`` are replicated; the result is
    replicated. ``vocab_chunk`` / ``sequence_chunk`` are validated as in the reference;
    the CUDA kernels tile by 128 tokens x 256 vocabulary rows and stream the whole shard,
    so results do not depend on them. ``token_chunk`` bounds the backward's dZ scratch.
    ``normalization_out``, if given, receives the [2, T] (max, sum) statistics of
    ``_vocab_parallel_logps_and_normalization`` (``losses.py:246-260``).
    ``dh_reduce_f32`` sums the per-shard dH partials in f32 (default: bf16, the reference's
    precision) before the single rounding to the hidden dtype. ``skip_zero_grad`` runs the
    backward only on the rows whose upstream gradient is nonzero (results are identical).
    """
    if backend != "cuda":
        if backend in ("jax", "pallas"):
            raise ValueError(
                f"logprob backend {backend!r} is implemented by gemma4_posttrain_jax itself; this package provides "
                "backend='cuda'"
            )
        raise ValueError(f"unknown logprob backend: {backend}")
    _validate(embed_tokens, hidden, targets, vocab_chunk, sequence_chunk)
    _validate_softcap(softcap)
    if mesh is not None and mesh.size > 1 and mesh.axis_names != ("d",):
        raise ValueError(f"vocab-parallel mesh needs axis 'd': {mesh.axis_names}")
    out_shape = targets.shape
    h2 = hidden.reshape(-1, hidden.shape[-1])
    y = targets.reshape(-1)
    if y.numel() == 0:
        return torch.zeros(out_shape, dtype=torch.float32, device=hidden.device)
    logp = _CudaTokenLogps.apply(embed_tokens, h2, y, softcap, mesh, token_chunk, normalization_out, dh_reduce_f32,
                                 skip_zero_grad)
    return logp.reshape(out_shape)


class _CompletionLogps(torch.autograd.Function):
    """Compacted response-token logprobs; scatters results and dH back to the slot layout."""

    @staticmethod
    def forward(ctx, embed, hidden, completion_ids, completion_mask, prompt_width, softcap, mesh, token_chunk, num_valid,
                dh_reduce_f32=False, skip_zero_grad=True):
        B, N = completion_mask.shape
        Hc, yc, idx, pos, count = ops.compact(completion_mask, hidden, completion_ids, row_offset=prompt_width - 1)
        if num_valid is None:
            n = int(count.item())
            _check_device(hidden.device, "completion_logps")
        else:
            n = int(num_valid)
            if _debug_checks():
                _check_num_valid(count, n)
        Hn, yn = Hc[:n], yc[:n]
        P = mesh.size if mesh is not None else 1
        off = vocab_offset(embed.shape[0], mesh) if P > 1 else 0
        if n > 0:
            if P > 1:
                logp_c, norm = _mesh_forward(embed, Hn, yn, softcap, mesh, off)
                if num_valid is not None and not _debug_checks():
                    _check_num_valid(count, n)  # the mesh forward has waited for the stream: free
            else:
                stats, logp_c = ops.shard_forward(embed, Hn, yn, softcap, want_logp=True)
                norm = stats[:2]
        else:
            logp_c = torch.zeros((1,), dtype=torch.float32, device=hidden.device)
            norm = torch.zeros((2, 0), dtype=torch.float32, device=hidden.device)
        out = torch.empty((B * N,), dtype=torch.float32, device=hidden.device)
        ops.scatter_rows(logp_c, pos, out)  # out[s] = logp_c[pos[s]] or 0
        ctx.save_for_backward(embed, Hn, yn, norm, idx[:n], pos)
        ctx.meta = (B, N, n, prompt_width, softcap, mesh, off, token_chunk, tuple(hidden.shape), hidden.dtype,
                    dh_reduce_f32, skip_zero_grad)
        return out.reshape(B, N)

    @staticmethod
    def backward(ctx, g):
        embed, Hn, yn, norm, idx_n, pos = ctx.saved_tensors
        B, N, n, prompt_width, softcap, mesh, off, token_chunk, hshape, hdtype, dh_reduce_f32, skip_zero_grad = ctx.meta
        P = mesh.size if mesh is not None else 1
        need_dw, need_dh = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        dW = dhidden = None
        if n > 0 and (need_dw or need_dh):
            gc = torch.empty((n,), dtype=torch.float32, device=g.device)
            ops.scatter_rows(g.reshape(-1).to(torch.float32).contiguous(), idx_n, gc)  # gc[i] = g[idx[i]]
            dHc, dW, posz, _ = _backward_rows(
                embed, Hn, yn, softcap, norm, gc, mesh=mesh, vocab_offset=off, need_dh=need_dh, need_dw=need_dw,
                dh_dtype=torch.float32 if (P > 1 and dh_reduce_f32) else torch.bfloat16, dw_dtype=embed.dtype,
                token_chunk=token_chunk, skip_zero_grad=skip_zero_grad,
            )
            if posz is not None:
                # slot -> compact row -> nonzero-gradient row (or -1)
                pos = torch.where(pos >= 0, posz[pos.clamp(min=0).long()], torch.full_like(pos, -1))
            if dHc is not None:
                with phase("dh_zero_fill"):
                    # rows outside the response slice get 0; the scatter writes every slice row
                    dhidden = torch.empty(hshape, dtype=hdtype, device=g.device)
                    if prompt_width > 1:
                        dhidden[:, : prompt_width - 1].zero_()
                    if prompt_width - 1 + N < hshape[1]:
                        dhidden[:, prompt_width - 1 + N :].zero_()
                # response slice hidden[:, P-1 : P-1+N] receives dHc at valid slots (summed f32
                # partials are rounded to bf16 by the scatter), 0 elsewhere
                ops.scatter_rows(dHc, pos, dhidden[:, prompt_width - 1 : prompt_width - 1 + N])
        if need_dw and dW is None:
            dW = torch.zeros_like(embed)
        if need_dh and dhidden is None:
            dhidden = torch.zeros(hshape, dtype=hdtype, device=g.device)
        return dW, dhidden, None, None, None, None, None, None, None, None, None


def _check_num_valid(count: torch.Tensor, n: int) -> None:
    """A caller's ``num_valid`` must be the mask's popcount: fewer would drop valid slots and
    more would read compacted rows that were never written."""
    c = int(count.item())
    if c != n:
        raise ValueError(f"num_valid={n} but completion_mask has {c} valid slots")


def completion_logps(
    embed_tokens: torch.Tensor,
    hidden: torch.Tensor,
    completion_ids: torch.Tensor,
    completion_mask: torch.Tensor,
    *,
    prompt_width: int,
    softcap: float | None,
    mesh: VocabMesh | None = None,
    token_chunk: int | None = None,
    num_valid: int | None = None,
    dh_reduce_f32: bool = False,
    skip_zero_grad: bool = True,
) -> torch.Tensor:
    """Response-token logprobs of ``trainer_completion_logps`` (``losses.py:667-682``).

    ``hidden`` is the model output [B, P + N, d]; completion token j of row b is predicted
    by position ``prompt_width + j - 1``. Only ``completion_mask`` slots are computed
    (compaction); invalid slots return 0, as ``where(completion_mask, logps, 0)`` does.
    ``num_valid`` (the mask's popcount, when the caller knows it on the host) avoids one
    device-to-host read; it is checked against the device count wherever the call waits for
    the GPU anyway (vocabulary-sharded calls) and always with ``LP_B200_DEBUG=1``.
    ``dh_reduce_f32``, ``skip_zero_grad``: see ``per_token_logps``.
    """
    if hidden.ndim != 3 or completion_ids.ndim != 2 or completion_mask.shape != completion_ids.shape:
        raise ValueError("hidden must be [B, S, d] and completion ids / mask [B, N]")
    if prompt_width < 1 or prompt_width - 1 + completion_ids.shape[1] > hidden.shape[1]:
        raise ValueError("prompt_width and completion width do not fit the hidden sequence")
    _validate_softcap(softcap)
    return _CompletionLogps.apply(
        embed_tokens, hidden, completion_ids, completion_mask, int(prompt_width), softcap, mesh, token_chunk, num_valid,
        dh_reduce_f32, skip_zero_grad,
    )


def sft_token_logps(
    embed_tokens: torch.Tensor,
    hidden: torch.Tensor,
    labels: torch.Tensor,
    *,
    softcap: float | None,
    mesh: VocabMesh | None = None,
    attention_mask: torch.Tensor | None = None,
    token_chunk: int | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """SFT next-token logps of ``losses.py:910-926``: returns (logps [B, S-1], loss_mask).

    Targets are ``labels[:, 1:]`` with ``-100`` (and padding) masked to id 0, predicted by
    ``hidden[:, :-1]``; the masked loss is ``-where(mask, logps, 0).sum() / max(mask.sum(), 1)``.
    """
    if labels.ndim != 2 or hidden.ndim != 3 or hidden.shape[:2] != labels.shape:
        raise ValueError("hidden must be [B, S, d] and labels [B, S]")
    if labels.shape[1] < 2:
        raise ValueError("SFT sequences need at least two tokens")
    targets = labels[:, 1:]
    mask = targets != -100
    if attention_mask is not None:
        mask = mask & attention_mask[:, 1:].to(torch.bool)
    safe = torch.where(mask, targets, torch.zeros_like(targets)).to(torch.int32)
    logps = per_token_logps(embed_tokens, hidden[:, :-1], safe, softcap=softcap, mesh=mesh, token_chunk=token_chunk)
    return logps, mask
