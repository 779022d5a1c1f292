"""The vocab-parallel host logic across processes (world size 2, gloo on CPU, 127.0.0.1).

Each rank holds one vocabulary shard. The per-shard statistics come from the oracle (the
CUDA kernels need a GPU; they are checked shard by shard in tests/test_gpu_parity.py); what
is tested here is the product's exchange layer in ``sharding.py``: the all-gather of the
[3, T] triples in rank order, row all-gather / reduce-scatter, the dH sum — and that a rank
which fails before a collective makes the others fail fast instead of hanging.
"""

from __future__ import annotations

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))


def _vocab_parallel_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        from gemma4_posttrain_jax_b200.sharding import (
            all_gather_rows,
            all_gather_stats,
            all_reduce_sum,
            dh_reduce_mode,
            dh_sum_buffer,
            make_mesh,
            reduce_scatter_rows,
            shard_rows,
            stats_exchange,
            stats_exchange_mode,
            vocab_offset,
        )
        from oracle import logprob_oracle as orc

        mesh = make_mesh()
        rng = np.random.default_rng(7)
        V, d, T = 96, 8, 20
        w = rng.normal(0.0, 0.2, (V, d)).astype(np.float32)
        h = rng.normal(0.0, 0.3, (T, d)).astype(np.float32)
        w[3, 0], w[51, 1] = 30.0, 40.0
        h[:, 0], h[:, 1] = 1.0, 0.5
        t = rng.integers(0, V, size=T).astype(np.int32)
        t[:4] = [0, 47, 48, 95]
        local = shard_rows(torch.from_numpy(w), mesh).numpy()
        off = vocab_offset(local.shape[0], mesh)
        tgt, mx, sm = orc._blocked_stats(local, h, t, softcap=30.0, vocab_chunk=17, sequence_chunk=6, vocab_offset=off,
                                         owned_only=True)
        stats = torch.from_numpy(np.stack([mx, sm, tgt]))
        gathered = all_gather_stats(stats, mesh).numpy()  # [P, 3, T]
        assert gathered.shape == (world, 3, T)
        gmax = gathered[:, 0].max(0)
        gsum = (gathered[:, 1] * np.exp(gathered[:, 0] - gmax)).sum(0)
        logp = gathered[:, 2].sum(0) - gmax - np.log(gsum)
        ref = orc.dense_logps(w, h, t, 30.0)
        err = float(np.abs(logp - ref).max())
        # rows: all-gather then reduce-scatter returns P x the local block
        rows = torch.full((3, 4), float(rank + 1))
        full = all_gather_rows(rows, mesh)
        back = reduce_scatter_rows(full.clone(), mesh)
        summed = all_reduce_sum(torch.ones(5) * (rank + 1), mesh)
        # a gloo mesh sums dH with a collective after the GEMM: no multicast buffer is made
        assert dh_reduce_mode(mesh) == "nccl"
        assert dh_sum_buffer(mesh, 16, 8, torch.device("cpu")) is None
        # ... and exchanges the per-shard triples with an all-gather, not a multicast buffer
        assert stats_exchange_mode(mesh) == "nccl"
        assert stats_exchange(mesh, 16, torch.device("cpu")) is None
        q.put((rank, err, full[:, 0].tolist(), back[:, 0].tolist(), summed[0].item()))
        dist.destroy_process_group()
    except Exception as exc:  # noqa: BLE001
        q.put((rank, repr(exc), None, None, None))


def test_vocab_parallel_exchange_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_vocab_parallel_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for rank, err, full, back, summed in results:
        assert not isinstance(err, str), err
        assert err < 5e-6
        assert full == [1.0] * 3 + [2.0] * 3
        # both ranks hold the same gathered rows; the reduce-scatter sums them (x2) and
        # hands rank r its own block back
        assert back == ([2.0] * 3 if rank == 0 else [4.0] * 3)
        assert summed == 3.0


def _failing_worker(rank, world, port, q):
    _init(rank, world, port, timeout_s=5)
    if rank == 1:
        # this rank dies between steps, before the next collective, and never joins it
        q.put((rank, "failed as planned"))
        q.close()
        q.join_thread()  # flush the message before the abrupt exit
        os._exit(0)
    try:
        from gemma4_posttrain_jax_b200.sharding import all_gather_stats, make_mesh

        all_gather_stats(torch.zeros((3, 4)), make_mesh())
        q.put((rank, "completed"))
    except Exception as exc:  # noqa: BLE001
        q.put((rank, type(exc).__name__))


def test_failed_rank_is_detected_without_hanging():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert got[1] == "failed as planned"
    assert got[0] != "completed"  # the surviving rank's collective errors out (timeout / closed peer)
