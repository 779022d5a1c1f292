"""Torch-facing wrappers over the C ABI: raw device pointers in, torch tensors out.

torch supplies device memory, the current CUDA stream and (in ``sharding``) the NCCL
process group; all arithmetic runs in liblp_b200.so. Nothing here computes on the host
and nothing falls back to torch ops: a missing library or a non-CUDA tensor raises.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

_MIN_ALIGN = 1024


def _require_cuda(*tensors: torch.Tensor | None) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("the cuda logprob backend needs CUDA tensors; it has no CPU fallback")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} and {t.device}")
    if dev is None:
        raise ValueError("no tensor given")
    return dev


def _ptr(t: torch.Tensor | None) -> ctypes.c_void_p | None:
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _workspace(nbytes: int, device: torch.device) -> tuple[torch.Tensor, ctypes.c_void_p, int]:
    """A scratch buffer from torch's caching allocator, aligned to 1 KiB."""
    buf = torch.empty(int(nbytes) + _MIN_ALIGN, dtype=torch.uint8, device=device)
    base = buf.data_ptr()
    off = (-base) % _MIN_ALIGN
    return buf, ctypes.c_void_p(base + off), int(nbytes)


def _rows(h: torch.Tensor) -> tuple[torch.Tensor, int]:
    """View ``h`` as [T, d] with unit column stride; returns (view, row stride)."""
    h2 = h.reshape(-1, h.shape[-1])
    if h2.stride(-1) != 1 or (h2.shape[0] > 1 and h2.stride(0) % 8 != 0):
        h2 = h2.contiguous()
    ld = h2.stride(0) if h2.shape[0] > 1 else h2.shape[1]
    return h2, int(ld)


def _check_bf16(name: str, t: torch.Tensor) -> None:
    if t.dtype != torch.bfloat16:
        raise ValueError(f"the cuda logprob backend needs bf16 {name}, got {t.dtype}")


def shard_forward(
    embed: torch.Tensor,
    hidden: torch.Tensor,
    targets: torch.Tensor,
    softcap: float | None,
    *,
    vocab_offset: int = 0,
    want_logp: bool = True,
) -> tuple[torch.Tensor, torch.Tensor | None]:
    """``lp_fwd`` on one vocabulary shard.

    Returns ``stats`` f32 [3, T] (shard max, shard sum exp(z - max), owned target logit)
    and, when ``want_logp``, logp f32 [T] (valid when the shard is the whole vocabulary).
    """
    dev = _require_cuda(embed, hidden, targets)
    _check_bf16("embedding", embed)
    _check_bf16("hidden", hidden)
    lib = _lib.load()
    h2, ldh = _rows(hidden)
    T, d = h2.shape
    Vs = embed.shape[0]
    w = embed if embed.is_contiguous() else embed.contiguous()
    y = targets.reshape(-1).to(torch.int32).contiguous()
    stats = torch.empty((3, T), dtype=torch.float32, device=dev)
    logp = torch.empty((T,), dtype=torch.float32, device=dev) if want_logp else None
    if T == 0:
        return stats, logp
    ws, wsp, wsn = _workspace(lib.lp_fwd_workspace_bytes(T, Vs), dev)
    cap = float(softcap) if softcap is not None else 0.0
    rc = lib.lp_fwd(
        _stream(dev), _ptr(h2), T, d, ldh, _ptr(w), Vs, int(vocab_offset), _ptr(y), cap, _ptr(stats), _ptr(logp), wsp, wsn
    )
    _lib.check(rc, "lp_fwd")
    return stats, logp


def shard_forward_sum(
    embed: torch.Tensor,
    hidden: torch.Tensor,
    targets: torch.Tensor,
    softcap: float | None,
    exchange,
    *,
    vocab_offset: int,
    timeout_ms: int,
) -> tuple[torch.Tensor, torch.Tensor]:
    """``lp_fwd_sum``: the forward of this rank's shard with the triples exchanged over
    NVLink (``exchange`` is a ``sharding.StatsExchange`` with room for T rows; every rank of
    the mesh makes the same call). Returns the global (logp [T], normalization [2, T])."""
    dev = _require_cuda(embed, hidden, targets)
    _check_bf16("embedding", embed)
    _check_bf16("hidden", hidden)
    lib = _lib.load()
    h2, ldh = _rows(hidden)
    T, d = h2.shape
    Vs = embed.shape[0]
    if T > exchange.rows:
        raise ValueError(f"stats exchange holds {exchange.rows} rows, {T} needed")
    w = embed if embed.is_contiguous() else embed.contiguous()
    y = targets.reshape(-1).to(torch.int32).contiguous()
    logp = torch.empty((T,), dtype=torch.float32, device=dev)
    norm = torch.empty((2, T), dtype=torch.float32, device=dev)
    if T == 0:
        return logp, norm
    ws, wsp, wsn = _workspace(lib.lp_fwd_workspace_bytes(T, Vs), dev)
    cap = float(softcap) if softcap is not None else 0.0
    xch, xch_mc, cnt, cnt_mc, arr, epoch = exchange.next_call()
    rc = lib.lp_fwd_sum(
        _stream(dev), _ptr(h2), T, d, ldh, _ptr(w), Vs, int(vocab_offset), _ptr(y), cap, ctypes.c_void_p(xch),
        ctypes.c_void_p(xch_mc), exchange.rows, ctypes.c_void_p(cnt), ctypes.c_void_p(cnt_mc), ctypes.c_void_p(arr),
        epoch, exchange.rank, exchange.world, int(timeout_ms), _ptr(logp), _ptr(norm), wsp, wsn,
    )
    _lib.check(rc, "lp_fwd_sum")
    return logp, norm


def head(
    embed: torch.Tensor,
    hidden: torch.Tensor,
    softcap: float | None,
    *,
    want_logits: bool = True,
    log_probs: bool = False,
) -> tuple[torch.Tensor | None, torch.Tensor, torch.Tensor, torch.Tensor]:
    """``lp_head`` over the whole vocabulary for B rows: (logits f32 [B, V] or None,
    normalization [2, B], argmax int32 [B], logp of the argmax [B]). ``log_probs`` makes the
    first output the full log-softmax instead of the logits."""
    dev = _require_cuda(embed, hidden)
    _check_bf16("embedding", embed)
    _check_bf16("hidden", hidden)
    if log_probs and not want_logits:
        raise ValueError("log_probs needs want_logits")
    lib = _lib.load()
    h2, ldh = _rows(hidden)
    B, d = h2.shape
    V = embed.shape[0]
    w = embed if embed.is_contiguous() else embed.contiguous()
    ld = -(-V // 4) * 4
    logits = torch.empty((B, ld), dtype=torch.float32, device=dev)[:, :V] if want_logits else None
    norm = torch.empty((2, B), dtype=torch.float32, device=dev)
    top = torch.empty((B,), dtype=torch.int32, device=dev)
    top_logp = torch.empty((B,), dtype=torch.float32, device=dev)
    if B == 0:
        return logits, norm, top, top_logp
    ws, wsp, wsn = _workspace(lib.lp_head_workspace_bytes(B, V), dev)
    cap = float(softcap) if softcap is not None else 0.0
    rc = lib.lp_head(
        _stream(dev), _ptr(h2), B, d, ldh, _ptr(w), V, cap, _ptr(logits), ld,
        _lib.LP_HEAD_LOGPROBS if log_probs else 0, _ptr(norm), _ptr(top), _ptr(top_logp), wsp, wsn,
    )
    _lib.check(rc, "lp_head")
    return logits, norm, top, top_logp


def combine(shard_stats: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """``lp_combine``: [P, 3, T] per-shard triples -> (logp [T], normalization [2, T])."""
    dev = _require_cuda(shard_stats)
    lib = _lib.load()
    s = shard_stats.to(torch.float32).contiguous()
    P, three, T = s.shape
    if three != 3:
        raise ValueError(f"shard stats must be [P, 3, T], got {tuple(s.shape)}")
    logp = torch.empty((T,), dtype=torch.float32, device=dev)
    norm = torch.empty((2, T), dtype=torch.float32, device=dev)
    _lib.check(lib.lp_combine(_stream(dev), _ptr(s), P, T, _ptr(logp), _ptr(norm)), "lp_combine")
    return logp, norm


def shard_backward(
    embed: torch.Tensor,
    hidden: torch.Tensor,
    targets: torch.Tensor,
    softcap: float | None,
    norm: torch.Tensor,
    grad_logp: torch.Tensor,
    *,
    vocab_offset: int = 0,
    need_dh: bool = True,
    need_dw: bool = True,
    dh_dtype: torch.dtype = torch.bfloat16,
    dw_dtype: torch.dtype = torch.float32,
    token_chunk: int | None = None,
    dh_out: torch.Tensor | None = None,
    dh_mesh_sum=None,
) -> tuple[torch.Tensor | None, torch.Tensor | None]:
    """``lp_bwd`` on one vocabulary shard: (dH [T, d] partial over this shard, dW [Vs, d]).

    With ``dh_mesh_sum`` (a ``sharding.DhSumBuffer`` with at least T rows; every rank makes
    the same call, its counters zero, and zeroes them again and calls ``peer_barrier`` after it)
    this is ``lp_bwd_sum``: the returned dH is this rank's bf16 copy, which holds the sum over
    the mesh's shards once that barrier has passed.
    """
    dev = _require_cuda(embed, hidden, targets, norm, grad_logp)
    _check_bf16("embedding", embed)
    _check_bf16("hidden", hidden)
    if dh_dtype not in (torch.bfloat16, torch.float32) or dw_dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("dH / dW dtypes must be bf16 or f32")
    lib = _lib.load()
    h2, ldh = _rows(hidden)
    T, d = h2.shape
    Vs = embed.shape[0]
    w = embed if embed.is_contiguous() else embed.contiguous()
    y = targets.reshape(-1).to(torch.int32).contiguous()
    g = grad_logp.reshape(-1).to(torch.float32).contiguous()
    nrm = norm.reshape(2, -1).to(torch.float32).contiguous()
    flags = 0
    dH = dW = None
    if need_dh and dh_mesh_sum is not None:
        if dh_mesh_sum.rows < T or dh_mesh_sum.d != d or dh_dtype != torch.bfloat16:
            raise ValueError("dh_mesh_sum needs a buffer of at least [T, d] rows and a bf16 dH")
        dH = dh_mesh_sum.local(T)
    elif need_dh:
        if dh_out is not None:
            if dh_out.shape != (T, d) or dh_out.dtype != dh_dtype or dh_out.stride(-1) != 1:
                raise ValueError("dh_out must be a [T, d] row-major tensor of dh_dtype")
            dH = dh_out
        else:
            dH = torch.empty((T, d), dtype=dh_dtype, device=dev)
        if dh_dtype == torch.float32:
            flags |= _lib.LP_BWD_DH_F32
    else:
        flags |= _lib.LP_BWD_NO_DH
    if need_dw:
        dW = torch.empty((Vs, d), dtype=dw_dtype, device=dev)
        if dw_dtype == torch.bfloat16:
            flags |= _lib.LP_BWD_DW_BF16
    else:
        flags |= _lib.LP_BWD_NO_DW
    chunk = int(token_chunk) if token_chunk else 0
    ws, wsp, wsn = _workspace(lib.lp_bwd_workspace_bytes(T, d, Vs, chunk, flags), dev)
    cap = float(softcap) if softcap is not None else 0.0
    ld_dh = int(dH.stride(0)) if dH is not None and T > 1 else d
    if need_dh and dh_mesh_sum is not None:
        from .sharding import peer_timeout_ms  # noqa: PLC0415

        m = dh_mesh_sum
        rc = lib.lp_bwd_sum(
            _stream(dev), _ptr(h2), T, d, ldh, _ptr(w), Vs, int(vocab_offset), _ptr(y), cap, _ptr(nrm), _ptr(g),
            _ptr(dH), ctypes.c_void_p(m.dh_mc), ld_dh, _ptr(m.counters), ctypes.c_void_p(m.counters_mc), m.rank,
            m.world, peer_timeout_ms(), _ptr(dW), flags, chunk, wsp, wsn,
        )
        _lib.check(rc, "lp_bwd_sum")
        return dH, dW
    rc = lib.lp_bwd(
        _stream(dev), _ptr(h2), T, d, ldh, _ptr(w), Vs, int(vocab_offset), _ptr(y), cap, _ptr(nrm), _ptr(g), _ptr(dH),
        ld_dh, _ptr(dW), flags, chunk, wsp, wsn,
    )
    _lib.check(rc, "lp_bwd")
    return dH, dW


def compact(
    mask: torch.Tensor,
    hidden: torch.Tensor | None = None,
    ids: torch.Tensor | None = None,
    *,
    row_offset: int = 0,
):
    """``lp_compact``: valid slots of ``mask`` [B, N] in slot order.

    With ``hidden`` [B, S, d] (bf16) and ``ids`` [B, N], also gathers the rows
    ``hidden[b, j + row_offset]`` and targets ``ids[b, j]`` of the valid slots. Returns
    ``(H_c [B*N, d] | None, y_c [B*N] | None, idx [B*N], pos [B*N], count [1])``; only the
    first ``count`` rows of H_c / y_c / idx are meaningful.
    """
    dev = _require_cuda(mask, hidden, ids)
    lib = _lib.load()
    if mask.ndim != 2:
        raise ValueError(f"mask must be [B, N], got {tuple(mask.shape)}")
    B, N = mask.shape
    m = mask.to(torch.uint8).contiguous()
    idx = torch.empty((B * N,), dtype=torch.int32, device=dev)
    pos = torch.empty((B * N,), dtype=torch.int32, device=dev)
    count = torch.empty((1,), dtype=torch.int32, device=dev)
    Hc = yc = None
    hb = hr = d = 0
    if hidden is not None:
        _check_bf16("hidden", hidden)
        if hidden.ndim != 3 or hidden.shape[0] != B or hidden.stride(-1) != 1:
            raise ValueError("hidden must be [B, S, d] with unit last stride")
        if row_offset < 0 or row_offset + N > hidden.shape[1]:
            raise ValueError("row_offset + N exceeds the hidden sequence length")
        d = hidden.shape[-1]
        hb, hr = hidden.stride(0), hidden.stride(1)
        Hc = torch.empty((B * N, d), dtype=torch.bfloat16, device=dev)
        if ids is not None:
            if ids.shape != (B, N):
                raise ValueError("ids must match the mask shape")
            ids = ids.to(torch.int32).contiguous()
            yc = torch.empty((B * N,), dtype=torch.int32, device=dev)
    ws, wsp, wsn = _workspace(lib.lp_compact_workspace_bytes(B, N), dev)
    rc = lib.lp_compact(
        _stream(dev), _ptr(m), B, N, _ptr(hidden), hb, hr, int(row_offset), d, _ptr(ids), _ptr(Hc), _ptr(yc), _ptr(idx),
        _ptr(pos), _ptr(count), wsp, wsn,
    )
    _lib.check(rc, "lp_compact")
    return Hc, yc, idx, pos, count


def scatter_rows(src: torch.Tensor, pos: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """``lp_scatter_rows``: out row s = src[pos[s]] where pos[s] >= 0, else 0.

    ``out`` is [slots] / [slots, width] or a strided [B, N, width] view (slot s = b * N + j),
    e.g. the response slice of a [B, S, d] gradient. Also serves as a row gather
    (``pos`` = source row of every output row). f32 ``src`` may be written to a bf16 ``out``.
    """
    dev = _require_cuda(src, pos, out)
    lib = _lib.load()
    if src.dtype not in (torch.bfloat16, torch.float32) or not (
        src.dtype == out.dtype or (src.dtype == torch.float32 and out.dtype == torch.bfloat16)
    ):
        raise ValueError("src / out must share a bf16 or f32 dtype, or be f32 -> bf16")
    if out.ndim == 3:
        B, N, width = out.shape
        rows_per_group, group_stride, row_stride = N, int(out.stride(0)), int(out.stride(1))
        if out.stride(2) != 1:
            raise ValueError("scatter needs unit column stride")
    else:
        o2 = out.reshape(out.shape[0], -1) if out.ndim > 1 else out.reshape(-1, 1)
        if o2.stride(-1) != 1:
            raise ValueError("scatter needs unit column stride")
        B, (N, width) = 1, o2.shape
        rows_per_group, row_stride = N, int(o2.stride(0))
        group_stride = N * row_stride
    s2 = src.reshape(src.shape[0], width)
    slots = B * N
    if s2.stride(-1) != 1:
        s2 = s2.contiguous()
    if pos.numel() != slots or s2.shape[1] != width:
        raise ValueError("pos / src / out shapes disagree")
    p = pos.to(torch.int32).contiguous()
    # an empty src is never read (every pos is -1); any valid pointer stands in for it
    src_ptr = _ptr(s2) if s2.shape[0] > 0 else _ptr(out)
    src_ld = int(s2.stride(0)) if s2.shape[0] > 0 else width
    rc = lib.lp_scatter_rows(
        _stream(dev), src_ptr, src_ld, _ptr(p), slots, width, src.element_size(), _ptr(out), row_stride,
        rows_per_group, group_stride, out.element_size(),
    )
    _lib.check(rc, "lp_scatter_rows")
    return out


def peer_barrier(buf, timeout_ms: int) -> None:
    """``lp_peer_barrier`` over the signal pads of a ``sharding.DhSumBuffer``, on the current
    stream of its device (every rank of the mesh must make the same calls in the same order)."""
    lib = _lib.load()
    rc = lib.lp_peer_barrier(_stream(buf.device), ctypes.c_void_p(buf.pads_dev), buf.rank, buf.world, buf.channel,
                             int(timeout_ms))
    _lib.check(rc, "lp_peer_barrier")


def bwd_sum_counters(rows: int) -> int:
    """Number of u32 row-block counters ``lp_bwd_sum`` uses for ``rows`` rows."""
    return int(_lib.load().lp_bwd_sum_counters(int(rows)))
