"""Vocabulary-parallel layout of the tied LM head over a torch.distributed process group.

The reference shards ``embed_tokens`` row-wise on its single mesh axis "d"
(``gemma4_posttrain_jax/sharding.py:30-39`` builds the mesh, ``:119-121`` forces the
embedding to ``P("d", None)``), replicates hidden states and targets at the
``shard_map`` boundary (``losses.py:253-259``) and combines per-shard statistics with
``pmax`` / ``psum`` (``losses.py:219,243-245``). Here one process drives one GPU; the
mesh axis is a process group, the shard is the local row block, and the exchanges are
NCCL collectives (gloo on CPU for the host-logic tests):

  * exchange of the per-shard (max, sum, owned target logit) triples, 12 bytes/token:
    inside the forward's finalize kernel through an NVLS multicast buffer
    (``StatsExchange``, ``lp_fwd_sum``) where the GPUs support it, else an NCCL all-gather
    merged on the device by ``lp_combine``;
  * sum of the per-shard dH partials: inside the dH GEMM through an NVLS multicast buffer
    (``DhSumBuffer``, multimem reductions from the GEMM epilogue) where the GPUs support
    it, else an NCCL all-reduce (reduce-scatter when the caller's hidden states are
    batch-sharded);
  * optional all-gather of batch-sharded hidden rows / targets before the head.
dW never leaves its shard.
"""

from __future__ import annotations

import os
from dataclasses import dataclass

import torch
import torch.distributed as dist

DATA_AXIS = "d"


@dataclass(frozen=True)
class VocabMesh:
    """A 1-D vocabulary-parallel mesh: a process group whose ranks each hold V / size rows."""

    group: dist.ProcessGroup | None = None

    @property
    def size(self) -> int:
        return dist.get_world_size(self.group) if dist.is_available() and dist.is_initialized() else 1

    @property
    def rank(self) -> int:
        return dist.get_rank(self.group) if dist.is_available() and dist.is_initialized() else 0

    @property
    def axis_names(self) -> tuple[str, ...]:
        return (DATA_AXIS,)

    @property
    def shape(self) -> dict[str, int]:
        return {DATA_AXIS: self.size}


def make_mesh(group: dist.ProcessGroup | None = None) -> VocabMesh:
    """Mesh over ``group`` (default: the world), the analogue of ``sharding.make_mesh``."""
    return VocabMesh(group)


def shard_rows(embed: torch.Tensor, mesh: VocabMesh) -> torch.Tensor:
    """This rank's row block of the full embedding, ``P("d", None)`` (``sharding.py:119-121``)."""
    V = embed.shape[0]
    if V % mesh.size:
        raise ValueError(f"vocab size {V} must be divisible by mesh axis {mesh.size}")
    vs = V // mesh.size
    return embed[mesh.rank * vs : (mesh.rank + 1) * vs]


def vocab_offset(local_rows: int, mesh: VocabMesh) -> int:
    """First global vocabulary id of this rank's shard (``lax.axis_index * local_vocab``)."""
    return mesh.rank * local_rows


def _is_nccl(mesh: VocabMesh) -> bool:
    return dist.get_backend(mesh.group) == "nccl"


def all_gather_stats(stats: torch.Tensor, mesh: VocabMesh) -> torch.Tensor:
    """[3, T] per-shard triples -> [P, 3, T] in rank order (one collective per call)."""
    P = mesh.size
    if P == 1:
        return stats.unsqueeze(0)
    s = stats.contiguous()
    if _is_nccl(mesh):
        out = torch.empty((P, *s.shape), dtype=s.dtype, device=s.device)
        dist.all_gather_into_tensor(out, s, group=mesh.group)
        return out
    parts = [torch.empty_like(s) for _ in range(P)]
    dist.all_gather(parts, s, group=mesh.group)
    return torch.stack(parts)


def all_reduce_sum(t: torch.Tensor, mesh: VocabMesh) -> torch.Tensor:
    """In-place sum over the mesh (dH partials of replicated hidden states)."""
    if mesh.size > 1:
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=mesh.group)
    return t


def all_gather_rows(local: torch.Tensor, mesh: VocabMesh) -> torch.Tensor:
    """Batch-sharded rows [n, ...] -> replicated [P * n, ...] (rank order)."""
    P = mesh.size
    if P == 1:
        return local
    x = local.contiguous()
    if _is_nccl(mesh):
        out = torch.empty((P * x.shape[0], *x.shape[1:]), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(out, x, group=mesh.group)
        return out
    parts = [torch.empty_like(x) for _ in range(P)]
    dist.all_gather(parts, x, group=mesh.group)
    return torch.cat(parts)


def reduce_scatter_rows(full: torch.Tensor, mesh: VocabMesh) -> torch.Tensor:
    """Replicated partial sums [P * n, ...] -> this rank's summed block [n, ...]."""
    P = mesh.size
    if P == 1:
        return full
    x = full.contiguous()
    if x.shape[0] % P:
        raise ValueError(f"rows {x.shape[0]} not divisible by mesh size {P}")
    n = x.shape[0] // P
    if _is_nccl(mesh):
        out = torch.empty((n, *x.shape[1:]), dtype=x.dtype, device=x.device)
        dist.reduce_scatter_tensor(out, x, op=dist.ReduceOp.SUM, group=mesh.group)
        return out
    dist.all_reduce(x, op=dist.ReduceOp.SUM, group=mesh.group)
    return x[mesh.rank * n : (mesh.rank + 1) * n].clone()


# ----------------------------------------------------------------------------- multicast dH sum
# Signal-pad row used by lp_peer_barrier (row 0 is left to torch's own symmetric-memory ops).
_BARRIER_CHANNEL = 1
_DH_BUFFERS: dict[tuple, "DhSumBuffer"] = {}
_MULTICAST_UNAVAILABLE: set[tuple] = set()


def dh_reduce_mode(mesh: VocabMesh | None) -> str:
    """How the dH partials are summed across shards: "none" (one shard), "multimem" (inside
    the dH GEMM through an NVLS multicast buffer) or "nccl" (all-reduce after it).
    ``LP_B200_DH_REDUCE=nccl`` forces the all-reduce."""
    if mesh is None or mesh.size == 1:
        return "none"
    if os.environ.get("LP_B200_DH_REDUCE", "multimem") != "multimem" or not _is_nccl(mesh):
        return "nccl"
    return "multimem"


def peer_timeout_ms() -> int:
    """Bound of every device-side wait for another rank (``LP_B200_PEER_TIMEOUT_MS``).

    The waits cover the skew between ranks reaching the same call: another rank's forward
    or dH GEMM (about 0.1 s for the config-2 batch on one GPU) plus that rank's host-side
    stalls. The default of 10 s is about 30 times the longest of those GEMMs; a rank that
    has not arrived by then is treated as lost and the call raises."""
    return max(1, int(os.environ.get("LP_B200_PEER_TIMEOUT_MS", "10000")))


class MulticastUnavailable(RuntimeError):
    """The mesh cannot use NVLS multicast buffers (decided by every rank together)."""


def _all_ranks_agree(mesh: VocabMesh, ok: bool, device: torch.device) -> bool:
    """True only where ``ok`` holds on every rank of the mesh. One all-reduce, so every rank
    takes the same branch: a rank whose allocation failed never leaves its peers waiting in
    a rendezvous or in a kernel that expects it."""
    flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=device)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=mesh.group)
    return bool(int(flag.item()) == 1)


def _symmetric_alloc(mesh: VocabMesh, nbytes: int, device: torch.device):
    """(storage, rendezvous handle) of ``nbytes`` of symmetric memory with a multicast
    mapping on every rank, or MulticastUnavailable on every rank alike."""
    group = mesh.group if mesh.group is not None else dist.group.WORLD
    storage = None
    try:
        import torch.distributed._symmetric_memory as symm_mem  # noqa: PLC0415 - CUDA + NCCL only

        storage = symm_mem.empty((nbytes,), dtype=torch.uint8, device=device)
    except (RuntimeError, ImportError):  # includes torch.OutOfMemoryError
        storage = None
    if not _all_ranks_agree(mesh, storage is not None, device):
        raise MulticastUnavailable("symmetric memory could not be allocated on every rank")
    handle = symm_mem.rendezvous(storage, group)
    if not _all_ranks_agree(mesh, int(handle.multicast_ptr) != 0, device):
        raise MulticastUnavailable("symmetric memory has no multicast mapping on every rank")
    return storage, handle


# Meshes whose multicast buffers a device-side peer timeout left out of step (their exchange
# counters no longer agree between ranks): later calls on them raise instead of waiting.
_POISONED: set[tuple] = set()


def poison(mesh: VocabMesh, device: torch.device) -> None:
    """Mark the mesh's multicast buffers on ``device`` unusable after a peer timeout."""
    _POISONED.add((id(mesh.group), device.index))


def _check_not_poisoned(gkey: tuple) -> None:
    if gkey in _POISONED:
        raise RuntimeError(
            "an earlier call on this vocabulary mesh gave up waiting for another rank, which left its NVLink "
            "exchange buffers out of step; create a new process group (and mesh) before calling again"
        )


class DhSumBuffer:
    """Symmetric memory bound to an NVLS multicast object on every rank of the mesh: a bf16
    [rows, d] dH buffer and the u32 row-block counters of ``lp_bwd_sum``. The dH GEMM stores
    each rank's partial tiles into its own copy and sums them across the copies through the
    NVSwitch, so every rank ends with the sum over vocabulary shards -- the psum of the dH
    partials (``losses.py:253-259`` transposed) done while the GEMM runs."""

    def __init__(self, mesh: VocabMesh, rows: int, d: int, device: torch.device):
        from . import _lib  # noqa: PLC0415

        self.rows, self.d, self.device = int(rows), int(d), device
        self.n_counters = int(_lib.load().lp_bwd_sum_counters(self.rows))
        dh_bytes = -(-self.rows * self.d * 2 // 4096) * 4096
        total = dh_bytes + -(-self.n_counters * 4 // 4096) * 4096
        self.storage, self.handle = _symmetric_alloc(mesh, total, device)
        self.dh = self.storage[: self.rows * self.d * 2].view(torch.bfloat16).view(self.rows, self.d)
        self.counters = self.storage[dh_bytes : dh_bytes + self.n_counters * 4].view(torch.int32)
        self.counters.zero_()
        torch.cuda.synchronize(device)
        # counters are zero on every rank before any rank's first lp_bwd_sum adds to them
        _all_ranks_agree(mesh, True, device)
        mc = int(self.handle.multicast_ptr)
        # the same on every rank (same world size and signal pad size)
        if (_BARRIER_CHANNEL + 1) * self.handle.world_size * 4 > self.handle.signal_pad_size:
            raise MulticastUnavailable("signal pad too small for the barrier channel")
        self.dh_mc = mc
        self.counters_mc = mc + dh_bytes
        self.pads_dev = int(self.handle.signal_pad_ptrs_dev)
        self.rank, self.world = int(self.handle.rank), int(self.handle.world_size)
        self.channel = _BARRIER_CHANNEL

    def local(self, rows: int) -> torch.Tensor:
        """This rank's copy of the first ``rows`` dH rows (the sum, after the second barrier)."""
        return self.dh[:rows]


def dh_sum_buffer(mesh: VocabMesh, rows: int, d: int, device: torch.device) -> DhSumBuffer | None:
    """The mesh's multicast dH buffer with room for ``rows`` x ``d`` (collective when it has to
    grow: every rank holds the same row count because the upstream gradient is replicated),
    or None where the multicast path is off or the system has no NVLS multicast."""
    gkey = (id(mesh.group), device.index)
    _check_not_poisoned(gkey)
    if dh_reduce_mode(mesh) != "multimem":
        return None
    if gkey in _MULTICAST_UNAVAILABLE:
        return None
    key = (*gkey, int(d))
    buf = _DH_BUFFERS.get(key)
    if buf is None or buf.rows < rows:
        grow = max(int(rows), -(-int(rows * 5 // 4) // 1024) * 1024)
        if buf is not None:
            torch.cuda.synchronize(device)  # no launch of this GPU still reads the old buffer
        _DH_BUFFERS.pop(key, None)
        buf = None
        try:
            buf = DhSumBuffer(mesh, grow, d, device)
        except MulticastUnavailable:
            _MULTICAST_UNAVAILABLE.add(gkey)
            return None
        _DH_BUFFERS[key] = buf
    return buf


# ----------------------------------------------------------------------------- multicast stats exchange
_STATS_EXCHANGES: dict[tuple, "StatsExchange"] = {}


def stats_exchange_mode(mesh: VocabMesh | None) -> str:
    """How the per-shard triples are exchanged: "none" (one shard), "multimem" (inside the
    forward's finalize kernel over NVLS multicast) or "nccl" (all-gather + ``lp_combine``).
    ``LP_B200_STATS_EXCHANGE=nccl`` forces the all-gather."""
    if mesh is None or mesh.size == 1:
        return "none"
    if os.environ.get("LP_B200_STATS_EXCHANGE", "multimem") != "multimem" or not _is_nccl(mesh):
        return "nccl"
    return "multimem"


class StatsExchange:
    """Symmetric memory bound to an NVLS multicast object on every rank of the mesh: two
    f32x4 [world, rows] exchange buffers, one u32 exchange counter each and a local arrival
    counter, the operands of ``lp_fwd_sum``. Calls alternate between the two buffers, and
    call number k of a buffer waits for counter == k * world, so the counters are never
    reset and no barrier is needed between calls (the pmax / psum of
    ``losses.py:219,243-245`` as one NVLink exchange inside the forward)."""

    def __init__(self, mesh: VocabMesh, rows: int, device: torch.device):
        self.rows, self.device = int(rows), device
        world = mesh.size
        slot_bytes = -(-world * self.rows * 16 // 4096) * 4096
        self.slot_bytes = slot_bytes
        total = 2 * slot_bytes + 4096  # two exchange buffers + counters (128 B apart) + arrivals
        self.storage, self.handle = _symmetric_alloc(mesh, total, device)
        self.storage[2 * slot_bytes :].zero_()
        torch.cuda.synchronize(device)
        # counters are zero on every rank before any rank signals
        _all_ranks_agree(mesh, True, device)
        mc = int(self.handle.multicast_ptr)
        self.base, self.base_mc = int(self.storage.data_ptr()), mc
        self.rank, self.world = int(self.handle.rank), int(self.handle.world_size)
        self.calls = 0

    def next_call(self) -> tuple[int, int, int, int, int, int]:
        """(exchange, exchange_mc, counter, counter_mc, arrivals, epoch) of the next call."""
        k = self.calls
        self.calls += 1
        slot, epoch = k % 2, k // 2 + 1
        cnt = 2 * self.slot_bytes + 128 * slot
        arrivals = 2 * self.slot_bytes + 256
        return (self.base + slot * self.slot_bytes, self.base_mc + slot * self.slot_bytes, self.base + cnt,
                self.base_mc + cnt, self.base + arrivals, epoch)


def stats_exchange(mesh: VocabMesh, rows: int, device: torch.device) -> StatsExchange | None:
    """The mesh's multicast stats exchange with room for ``rows`` tokens (collective when it
    has to grow: every rank holds the same token count because hidden states and targets
    are replicated), or None where the multicast path is off or unavailable."""
    gkey = (id(mesh.group), device.index)
    _check_not_poisoned(gkey)
    if stats_exchange_mode(mesh) != "multimem":
        return None
    if gkey in _MULTICAST_UNAVAILABLE:
        return None
    buf = _STATS_EXCHANGES.get(gkey)
    if buf is None or buf.rows < rows:
        grow = max(int(rows), -(-int(rows * 5 // 4) // 1024) * 1024)
        if buf is not None:
            torch.cuda.synchronize(device)  # the old buffer's last exchange has finished here
        _STATS_EXCHANGES.pop(gkey, None)
        try:
            buf = StatsExchange(mesh, grow, device)
        except MulticastUnavailable:
            _MULTICAST_UNAVAILABLE.add(gkey)
            return None
        _STATS_EXCHANGES[gkey] = buf
    return buf
