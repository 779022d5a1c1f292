"""The allocation-free forward (lp_fwd_noalloc) against the workspace forward (lp_fwd).

lp_fwd_noalloc serves callers that cannot allocate device memory at the call site (an FFI
custom call that only receives its input and output buffers, a host loop that must not
grow device memory after start-up); its scratch is a fixed array inside the library. This
test calls it through the C ABI twice in a row, on the same inputs as the existing entry
point, and checks both calls against lp_fwd with the tolerances of the other forward tests
(per-token logp within 2e-3; statistics as in test_forward_stats_and_logps), and a sample
of rows against the CPU oracle. The largest case needs more scratch than lp_fwd's tile
plan would use, so the entry point widens its vocabulary groups (fewer groups of more
tiles) to fit. It lives in its own file so pytest collects it last, and it must pass in a
fresh process as well as after the other tests.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import logprob_oracle as orc

pytestmark = pytest.mark.gpu

LOGP_ATOL = 2e-3


def _inputs(dev, T, V, d, scale, seed):
    rng = np.random.default_rng(seed)
    w = orc.bf16_round(rng.normal(size=(V, d)) * scale)
    h = orc.bf16_round(rng.normal(size=(T, d)))
    y = rng.integers(0, V, size=T).astype(np.int32)
    W = torch.from_numpy(w).to(dev).to(torch.bfloat16)
    H = torch.from_numpy(h).to(dev).to(torch.bfloat16)
    return W, H, torch.from_numpy(y).to(dev)


def _noalloc(lib, dev, W, H, Y, softcap, v_off=0, want_logp=True):
    from gemma4_posttrain_jax_b200 import _lib
    from gemma4_posttrain_jax_b200.ops import _ptr, _stream

    T, d = H.shape
    stats = torch.full((3, T), float("nan"), dtype=torch.float32, device=dev)
    logp = torch.full((T,), float("nan"), dtype=torch.float32, device=dev) if want_logp else None
    rc = lib.lp_fwd_noalloc(_stream(dev), _ptr(H), T, d, H.stride(0), _ptr(W), W.shape[0], v_off, _ptr(Y),
                            float(softcap or 0.0), _ptr(stats), _ptr(logp))
    _lib.check(rc, "lp_fwd_noalloc")
    return stats, logp


def _default_groups(T, V):
    """Vocabulary groups of lp_fwd's plan (lp_capi.cu plan_fwd) and the scratch they need."""
    tiles = -(-V // 256)
    g = 1
    while g < tiles and 2 * (-(-tiles // g)) * T * 8 > (128 << 20):
        g *= 2
    g = max(g, min(4, tiles))
    groups = -(-tiles // g)
    up = lambda x: -(-x // 256) * 256  # noqa: E731
    return groups, up(2 * groups * T * 8) + up(4 * T)


def test_widening_case_exceeds_the_default_plan():
    # the last case below would need more than the fixed scratch with lp_fwd's groups
    groups, need = _default_groups(60000, 70000)
    assert groups == 69 and need > (8 << 20)


@pytest.mark.parametrize(
    "T,V,d,scale,softcap,v_off",
    [(513, 1036, 128, 1.5, 30.0, 0), (513, 1036, 128, 0.04, None, 0), (4099, 70000, 256, 0.3, 30.0, 12345),
     (60000, 70000, 64, 0.5, 30.0, 0)],
)
def test_noalloc_forward_matches_workspace_forward(cuda_device, T, V, d, scale, softcap, v_off):
    from gemma4_posttrain_jax_b200 import _lib, ops

    lib = _lib.load()
    W, H, Y = _inputs(cuda_device, T, V, d, scale, seed=T + V)
    Y = Y + v_off  # some targets fall outside the shard when v_off > 0 ... and some inside
    Y[: T // 2] -= v_off
    want_logp = v_off == 0
    ref_stats, ref_logp = ops.shard_forward(W, H, Y, softcap, vocab_offset=v_off, want_logp=want_logp)
    torch.cuda.synchronize()
    for _ in range(2):  # two calls in a row share (and reuse) the library's scratch
        stats, logp = _noalloc(lib, cuda_device, W, H, Y, softcap, v_off=v_off, want_logp=want_logp)
        torch.cuda.synchronize()
        assert _lib.device_error(cuda_device.index or 0) == 0
        s, r = stats.cpu().numpy(), ref_stats.cpu().numpy()
        assert np.isfinite(s).all()
        np.testing.assert_allclose(s[0], r[0], atol=2e-4, rtol=2e-5)
        np.testing.assert_allclose(s[1], r[1], rtol=1e-4)
        np.testing.assert_allclose(s[2], r[2], atol=2e-4, rtol=2e-5)
        if want_logp:
            assert np.abs(logp.cpu().numpy() - ref_logp.cpu().numpy()).max() <= LOGP_ATOL
    if want_logp:
        # a sample of rows against the CPU oracle (float64 dense log-softmax)
        rows = np.random.default_rng(T).choice(T, size=min(T, 384), replace=False)
        w = W.float().cpu().numpy()
        h = H.float().cpu().numpy()[rows]
        ref = orc.dense_logps(w, h, Y.cpu().numpy()[rows], softcap)
        assert np.abs(logp.cpu().numpy()[rows] - ref).max() <= LOGP_ATOL


def test_noalloc_forward_refuses_oversized_requests(cuda_device):
    from gemma4_posttrain_jax_b200 import _lib
    from gemma4_posttrain_jax_b200.ops import _ptr, _stream

    lib = _lib.load()
    W, H, Y = _inputs(cuda_device, 8, 64, 64, 0.1, seed=1)
    stats = torch.empty((3, 8), dtype=torch.float32, device=cuda_device)
    # the size check runs before any device work, so the small buffers are never touched
    rc = lib.lp_fwd_noalloc(_stream(cuda_device), _ptr(H), 2_000_000, 64, 64, _ptr(W), 64, 0, _ptr(Y), 0.0,
                            _ptr(stats), None)
    assert rc == _lib.LP_EINVAL
    assert b"LP_NOALLOC_SCRATCH_BYTES" in lib.lp_last_error()
