"""Vocabulary-parallel layout of the tied LM head over a torch.distributed process group.

The reference shards ``embed_tokens`` row-wise on its single mesh axis "d"
(``gemma4_posttrain_jax/sharding.py:30-39`` builds the mesh, ``:119-121`` forces the
embedding to ``P("d", None)``), replicates hidden states and targets at the
``shard_map`` boundary (``losses.py:253-259``) and combines per-shard statistics with
``pmax`` / ``psum`` (``losses.py:219,243-245``). Here one process drives one GPU; the
mesh axis is a process group, the shard is the local row block, and the exchanges are
NCCL collectives (gloo on CPU for the host-logic tests):

  * all-gather of the per-shard (max, sum, owned target logit) triples, 12 bytes/token,
    merged on the device by ``lp_combine``;
  * sum of the per-shard dH partials (all-reduce, or reduce-scatter when the caller's
    hidden states are batch-sharded);
  * optional all-gather of batch-sharded hidden rows / targets before the head.
dW never leaves its shard.
"""

from __future__ import annotations

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
