"""Failure detection on the GPU without a fault: a bounded device-side wait that runs out.

lp_peer_barrier is called as rank 0 of a two-rank mesh whose second rank never exists: the
wait for rank 1's signal (a flag nothing sets) gives up after its time limit, the kernel
records DEV_TIMEOUT_PEER for the host and returns, and the CUDA context stays usable for
the next launches. The pads are this GPU's own zeroed memory (plain system-scope atomics;
no multicast, no peer mapping).
"""

from __future__ import annotations

import ctypes
import time

import numpy as np
import pytest
import torch

from oracle import logprob_oracle as orc

pytestmark = pytest.mark.gpu

DEV_TIMEOUT_PEER = 5


def test_peer_barrier_gives_up_on_a_missing_rank(cuda_device):
    from gemma4_posttrain_jax_b200 import _lib
    from gemma4_posttrain_jax_b200.ops import _stream

    lib = _lib.load()
    pads = [torch.zeros(64, dtype=torch.int32, device=cuda_device) for _ in range(2)]
    ptrs = torch.tensor([p.data_ptr() for p in pads], dtype=torch.int64, device=cuda_device)
    torch.cuda.synchronize()
    assert _lib.device_error(0) == 0
    t0 = time.perf_counter()
    rc = lib.lp_peer_barrier(_stream(cuda_device), ctypes.c_void_p(ptrs.data_ptr()), 0, 2, 1, 200)
    assert rc == _lib.LP_OK
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert _lib.device_error(0) == DEV_TIMEOUT_PEER  # read (and cleared) by the host
    assert 0.15 <= waited < 20.0
    # rank 0 raised its signal in the missing rank's pad and consumed its own
    assert pads[1][2].item() == 1 and pads[0][2].item() == 0
    # a one-rank barrier passes at once
    rc = lib.lp_peer_barrier(_stream(cuda_device), ctypes.c_void_p(ptrs.data_ptr()), 0, 1, 1, 200)
    torch.cuda.synchronize()
    assert rc == _lib.LP_OK and _lib.device_error(0) == 0


def test_context_usable_after_a_timed_out_wait(cuda_device):
    from gemma4_posttrain_jax_b200 import _lib, per_token_logps
    from gemma4_posttrain_jax_b200.ops import _stream

    lib = _lib.load()
    pads = [torch.zeros(64, dtype=torch.int32, device=cuda_device) for _ in range(2)]
    ptrs = torch.tensor([p.data_ptr() for p in pads], dtype=torch.int64, device=cuda_device)

    lib.lp_peer_barrier(_stream(cuda_device), ctypes.c_void_p(ptrs.data_ptr()), 0, 2, 1, 100)
    torch.cuda.synchronize()
    assert _lib.device_error(0) == DEV_TIMEOUT_PEER
    rng = np.random.default_rng(3)
    w = orc.bf16_round(rng.normal(size=(300, 64)) * 0.5)
    h = orc.bf16_round(rng.normal(size=(40, 64)))
    y = rng.integers(0, 300, size=40).astype(np.int32)
    lp = per_token_logps(torch.from_numpy(w).to(cuda_device).to(torch.bfloat16),
                         torch.from_numpy(h).to(cuda_device).to(torch.bfloat16),
                         torch.from_numpy(y).to(cuda_device), softcap=30.0)
    torch.cuda.synchronize()
    assert _lib.device_error(0) == 0
    assert np.abs(lp.cpu().numpy() - orc.dense_logps(w, h, y, 30.0)).max() <= 2e-3


def test_recorded_timeout_raises_at_the_next_host_sync(cuda_device):
    """A device error is not silent in the product path: the first place where the library
    waits for the GPU (here the backward's row count, and completion_logps' valid-slot
    count) raises, naming the code, until the code is read and cleared."""
    from gemma4_posttrain_jax_b200 import _lib, completion_logps, per_token_logps
    from gemma4_posttrain_jax_b200.ops import _stream

    lib = _lib.load()
    pads = [torch.zeros(64, dtype=torch.int32, device=cuda_device) for _ in range(2)]
    ptrs = torch.tensor([p.data_ptr() for p in pads], dtype=torch.int64, device=cuda_device)
    lib.lp_peer_barrier(_stream(cuda_device), ctypes.c_void_p(ptrs.data_ptr()), 0, 2, 1, 100)
    torch.cuda.synchronize()
    assert _lib.device_error_poll(0) == DEV_TIMEOUT_PEER  # visible on the host without a CUDA call

    rng = np.random.default_rng(4)
    w = orc.bf16_round(rng.normal(size=(300, 64)) * 0.5)
    h = orc.bf16_round(rng.normal(size=(40, 64)))
    y = rng.integers(0, 300, size=40).astype(np.int32)
    g = rng.normal(size=40).astype(np.float32)
    g[:10] = 0.0
    W = torch.from_numpy(w).to(cuda_device).to(torch.bfloat16).requires_grad_(True)
    H = torch.from_numpy(h).to(cuda_device).to(torch.bfloat16).requires_grad_(True)
    lp = per_token_logps(W, H, torch.from_numpy(y).to(cuda_device), softcap=30.0)
    with pytest.raises(_lib.DeviceTimeoutError, match="DEV_TIMEOUT_PEER"):
        lp.backward(torch.from_numpy(g).to(cuda_device))
    mask = torch.ones((2, 20), dtype=torch.bool, device=cuda_device)
    with pytest.raises(_lib.DeviceTimeoutError, match="DEV_TIMEOUT_PEER"):
        completion_logps(W, H.detach().view(2, 20, 64), torch.from_numpy(y).to(cuda_device).view(2, 20), mask,
                         prompt_width=1, softcap=30.0)
    assert _lib.device_error(0) == DEV_TIMEOUT_PEER  # read and cleared (both copies)
    assert _lib.device_error_poll(0) == 0
    lp = per_token_logps(W, H, torch.from_numpy(y).to(cuda_device), softcap=30.0)
    lp.backward(torch.from_numpy(g).to(cuda_device))
    torch.cuda.synchronize()
    assert np.abs(lp.detach().cpu().numpy() - orc.dense_logps(w, h, y, 30.0)).max() <= 2e-3
