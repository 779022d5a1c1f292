"""Host side of failure detection, on CPU: a device error recorded by a kernel becomes an
exception at the library's next host synchronisation, a peer timeout retires the mesh's
multicast buffers, a wrong ``num_valid`` is refused, and the choice between NVLink
multicast buffers and NCCL is made by all ranks together (world size 2, gloo), so a rank
whose allocation fails never leaves its peer waiting in a rendezvous."""

from __future__ import annotations

import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gemma4_posttrain_jax_b200 import _lib, losses, sharding


def test_poll_reads_zero_without_a_gpu():
    # the host-mapped error slots do not exist before the library has run on a device
    assert _lib.device_error_poll(0) == 0
    _lib.raise_on_device_error(0, "nothing ran")


def test_recorded_peer_timeout_raises_with_its_name(monkeypatch):
    monkeypatch.setattr(_lib, "device_error_poll", lambda device: 5)
    with pytest.raises(_lib.DeviceTimeoutError, match="DEV_TIMEOUT_PEER"):
        _lib.raise_on_device_error(0, "lp_fwd_sum")
    monkeypatch.setattr(_lib, "device_error_poll", lambda device: 2)
    with pytest.raises(_lib.DeviceTimeoutError, match="DEV_TIMEOUT_MMA"):
        losses._check_device(torch.device("cuda", 0), "backward")


def test_mesh_call_after_a_timeout_retires_the_buffers(monkeypatch):
    class _Stream:
        def synchronize(self):
            pass

    monkeypatch.setattr(torch.cuda, "current_stream", lambda device=None: _Stream())
    monkeypatch.setattr(_lib, "device_error_poll", lambda device: 5)
    mesh = sharding.VocabMesh(None)
    dev = torch.device("cuda", 3)
    monkeypatch.setattr(sharding, "_POISONED", set())
    with pytest.raises(_lib.DeviceTimeoutError):
        losses._check_mesh_call(dev, mesh, "lp_bwd_sum")
    # every later call on this mesh and device refuses to touch the out-of-step buffers
    with pytest.raises(RuntimeError, match="out of step"):
        sharding.stats_exchange(mesh, 16, dev)
    with pytest.raises(RuntimeError, match="out of step"):
        sharding.dh_sum_buffer(mesh, 16, 8, dev)
    # other devices of the process are not affected
    assert sharding.stats_exchange(mesh, 16, torch.device("cuda", 2)) is None


def test_num_valid_must_match_the_mask():
    losses._check_num_valid(torch.tensor([7], dtype=torch.int32), 7)
    with pytest.raises(ValueError, match="num_valid=6 but completion_mask has 7 valid slots"):
        losses._check_num_valid(torch.tensor([7], dtype=torch.int32), 6)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _alloc_worker(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
        import torch.distributed._symmetric_memory as symm_mem

        def empty(shape, dtype, device):
            if rank == 1:  # this rank runs out of device memory
                raise torch.OutOfMemoryError("no room for the multicast buffer")
            return torch.empty(shape, dtype=dtype)

        def rendezvous(*a, **k):
            raise AssertionError("rendezvous reached although a rank has no buffer")

        symm_mem.empty = empty
        symm_mem.rendezvous = rendezvous
        try:
            sharding._symmetric_alloc(sharding.make_mesh(), 4096, torch.device("cpu"))
            q.put((rank, "allocated"))
        except sharding.MulticastUnavailable:
            q.put((rank, "fell back"))
        dist.destroy_process_group()
    except Exception as exc:  # noqa: BLE001
        q.put((rank, repr(exc)))


def test_multicast_fallback_is_decided_by_all_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_alloc_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert got == {0: "fell back", 1: "fell back"}
