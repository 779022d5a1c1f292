"""bench.py's float32 parity check, run on the CPU with the oracle's float64 results in place
of the library's: it must agree with the oracle (so the check used on every bench line and
in the multi-GPU worker computes the reference's math), and it must flag a wrong dH, dW or
logp. One shard (world 1); the cross-shard combine is the same all-reduce arithmetic."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402
from oracle import logprob_oracle as orc  # noqa: E402


def _case(seed=5, T=300, V=700, d=64):
    rng = np.random.default_rng(seed)
    w = orc.bf16_round(rng.normal(size=(V, d)) * 0.5)
    h = orc.bf16_round(rng.normal(size=(T, d)))
    y = rng.integers(0, V, size=T).astype(np.int32)
    g = rng.normal(size=T).astype(np.float32)
    g[::7] = 0.0
    lp, dW, dH = orc.logps_grads_f64(w, h, y, g, 30.0)
    t = lambda a, dt=torch.float32: torch.from_numpy(np.ascontiguousarray(a)).to(dt)  # noqa: E731
    return dict(W=t(w, torch.bfloat16), Hv=t(h, torch.bfloat16), yv=t(y, torch.int32), gv=t(g),
                lp_v=t(lp), dW=t(dW), dHv=t(dH))


def _check(**kw):
    return bench.parity_check(kw.pop("W"), softcap=30.0, rank=0, world=1, dev=torch.device("cpu"), rows=64, **kw)


def test_float32_check_agrees_with_the_oracle():
    r = _check(**_case())
    assert r["ok"], r
    assert r["logp_max_abs"] < 1e-5 and r["dh_rel_l2"] < 1e-5 and r["dw_rel_l2"] < 1e-5
    assert r["tokens_checked"] == 300 and r["dh_rows"] == 64 and r["zero_grad_rows_zero"]


@pytest.mark.parametrize("what", ["lp_v", "dHv", "dW", "zero_row"])
def test_float32_check_flags_wrong_results(what):
    c = _case()
    if what == "lp_v":
        c["lp_v"] = c["lp_v"] + 5e-3
    elif what == "dHv":
        c["dHv"] = c["dHv"] * 1.05
    elif what == "dW":
        c["dW"] = c["dW"] * 0.95
    else:
        c["dHv"][0] = 1.0  # row 0 has g == 0: its dH must be exactly zero
    r = _check(**c)
    assert not r["ok"], r


def _parity_rank(rank, world, port, q):
    import os
    from datetime import timedelta

    import torch.distributed as dist

    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        c = _case(seed=9, V=800)
        vs = 800 // world
        W = c.pop("W")[rank * vs : (rank + 1) * vs]
        c["dW"] = c["dW"][rank * vs : (rank + 1) * vs]
        r = bench.parity_check(W, softcap=30.0, rank=rank, world=world, dev=torch.device("cpu"), rows=64, **c)
        c["dHv"] = c["dHv"] * 1.05  # a wrong dH sum must fail on every rank
        bad = bench.parity_check(W, softcap=30.0, rank=rank, world=world, dev=torch.device("cpu"), rows=64, **c)
        q.put((rank, r["ok"], r["logp_max_abs"], r["dh_rel_l2"], r["dw_rel_l2"], bad["ok"]))
        dist.destroy_process_group()
    except Exception as exc:  # noqa: BLE001
        q.put((rank, repr(exc), None, None, None, None))


def test_float32_check_combines_shards_over_ranks():
    """Two gloo ranks, each holding half of the vocabulary: the check's pmax / psum combine
    and its summed dH rows reproduce the single-partition oracle, on both ranks alike."""
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_parity_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for rank, ok, e_lp, e_dh, e_dw, bad_ok in got:
        assert ok is True, (rank, ok)
        assert e_lp < 1e-5 and e_dh < 1e-5 and e_dw < 1e-5
        assert bad_ok is False
    assert got[0][2:5] == got[1][2:5]  # the reported errors are the same on every rank
