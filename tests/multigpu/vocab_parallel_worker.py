"""One rank of the multi-GPU parity check (launched by tests/test_gpu_multirank.py via torchrun).

Every rank draws the same seeded inputs, keeps its vocabulary row block, and runs the
public API (per_token_logps and completion_logps, forward + backward) over an NCCL mesh.
Rank 0 gathers the dW shards and checks logps, dH and dW against the CPU oracle. A
config-2-shaped case (32768 vocabulary rows per rank, d = 2048, 12288 tokens, zero-gradient
rows) runs the production plan of the fused NVLink forward exchange and in-GEMM dH sum; it
is checked in full against a float32 PyTorch computation on the GPUs (bench.py's parity
check: every logp, 256 dH rows, 256 dW rows per shard) and on sampled rows against the
oracle.
"""

from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from gemma4_posttrain_jax_b200 import completion_logps, make_mesh, per_token_logps, shard_rows, sharding  # noqa: E402
from oracle import logprob_oracle as orc  # noqa: E402


def rel_l2(a, b):
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


LOGPS: dict = {}


def check_per_token(mesh, dev, rank, world, mode, V, T, d, seed, stats_mode="multimem") -> bool:
    """per_token_logps fwd + bwd on the mesh with the dH sum done by `mode` and the triples
    exchanged by `stats_mode`; rank 0 checks (logps of both exchanges must be bit-identical)."""
    os.environ["LP_B200_DH_REDUCE"] = mode
    os.environ["LP_B200_STATS_EXCHANGE"] = stats_mode
    rng = np.random.default_rng(seed)
    w = orc.bf16_round(rng.normal(size=(V, d)) * 1.5)
    h = orc.bf16_round(rng.normal(size=(T, d)))
    y = rng.integers(0, V, size=T).astype(np.int32)
    y[:4] = [0, V // world - 1, V // world, V - 1]
    g = rng.normal(size=T).astype(np.float32)
    g[5:40] = 0.0  # rows the backward skips
    W = shard_rows(torch.from_numpy(w), mesh).to(dev).to(torch.bfloat16).requires_grad_(True)
    H = torch.from_numpy(h).to(dev).to(torch.bfloat16).requires_grad_(True)
    ok = True
    for _ in range(2):  # the second pass reuses the (re-zeroed) multicast buffer
        W.grad = H.grad = None
        lp = per_token_logps(W, H, torch.from_numpy(y).to(dev), softcap=30.0, mesh=mesh)
        (lp * torch.from_numpy(g).to(dev)).sum().backward()
        dW_parts = [torch.empty_like(W.grad) for _ in range(world)]
        dist.all_gather(dW_parts, W.grad)
        used = sharding.dh_reduce_mode(mesh)
        if mode == "multimem" and used == "multimem" and not sharding._DH_BUFFERS:
            used = "nccl (no NVLS multicast on this system)"
        xused = sharding.stats_exchange_mode(mesh)
        if xused == "multimem" and not sharding._STATS_EXCHANGES:
            xused = "nccl (no NVLS multicast on this system)"
        key = (V, T, d, seed)
        lp_host = lp.detach().cpu().numpy()
        same = True
        if key in LOGPS:
            same = bool(np.array_equal(LOGPS[key], lp_host))
        else:
            LOGPS[key] = lp_host
        if rank == 0:
            lp_ref, dW_ref, dH_ref = orc.logps_grads_f64(w, h, y, g, 30.0)
            e_lp = float(np.abs(lp.detach().cpu().numpy() - lp_ref).max())
            e_h = rel_l2(H.grad.float().cpu().numpy(), dH_ref)
            e_w = rel_l2(torch.cat(dW_parts).float().cpu().numpy(), dW_ref)
            zero_rows = bool((H.grad[5:40] == 0).all())
            print(f"world={world} T={T} d={d} dH sum={used} stats={xused}: logp max abs {e_lp:.2e}, "
                  f"dH rel-L2 {e_h:.2e}, dW rel-L2 {e_w:.2e}, skipped rows zero: {zero_rows}, "
                  f"logps identical across exchanges: {same}", flush=True)
            ok = ok and e_lp <= 2e-3 and e_h <= 1e-2 and e_w <= 1e-2 and zero_rows and same
        # the other ranks wait here (host side) while rank 0 runs the CPU oracle, not inside
        # the next call's bounded device-side wait for rank 0
        dist.barrier(device_ids=[dev.index])
    return ok


def check_config2_shape(mesh, dev, rank, world, seed, T=12288, d=2048, Vs=32768) -> bool:
    """The production plan (Vs = 32768 per rank as in config 2 at 8 GPUs, d = 2048) of the
    NVLink forward exchange and the in-GEMM dH sum, checked in full and against the oracle."""
    from bench import parity_check

    os.environ["LP_B200_DH_REDUCE"] = "multimem"
    os.environ["LP_B200_STATS_EXCHANGE"] = "multimem"
    V = Vs * world
    gen = torch.Generator(device=dev).manual_seed(seed)
    W_full = (torch.randn((V, d), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
    H = torch.randn((T, d), generator=gen, device=dev).to(torch.bfloat16)
    y = torch.randint(0, V, (T,), generator=gen, device=dev, dtype=torch.int32)
    y[:4] = torch.tensor([0, Vs - 1, Vs, V - 1], dtype=torch.int32, device=dev)
    g = torch.randn((T,), generator=gen, device=dev) * (torch.rand((T,), generator=gen, device=dev) < 0.9)
    g[256:768] = 0.0  # two whole zero-gradient row blocks
    W = W_full[rank * Vs : (rank + 1) * Vs].clone().requires_grad_(True)
    w_host = W_full.float().cpu().numpy() if rank == 0 else None
    ok = True
    for rep in range(2):  # the second call reuses the multicast buffers
        W.grad = None
        Hq = H.clone().requires_grad_(True)
        lp = per_token_logps(W, Hq, y, softcap=30.0, mesh=mesh)
        lp.backward(g)
        torch.cuda.synchronize()
        par = parity_check(W, H, y, g, lp.detach(), W.grad, Hq.grad, softcap=30.0, rank=rank, world=world, dev=dev)
        if rank == 0:
            gen_r = np.random.default_rng(seed + rep)
            rows = np.sort(gen_r.choice(np.nonzero(g.cpu().numpy())[0], size=16, replace=False))
            h = H.float().cpu().numpy()[rows]
            lp_o, _, dh_o = orc.logps_grads_f64(w_host, h, y.cpu().numpy()[rows], g.cpu().numpy()[rows], 30.0,
                                                want_dw=False)
            e_lp_o = float(np.abs(lp.detach().cpu().numpy()[rows] - lp_o).max())
            e_dh_o = rel_l2(Hq.grad.float().cpu().numpy()[rows], dh_o)
            print(f"world={world} config-2 shape (Vs={Vs}, d={d}, T={T}) call {rep + 1}: dH sum="
                  f"{sharding.dh_reduce_mode(mesh)} stats={sharding.stats_exchange_mode(mesh)}; float32 check: "
                  f"logp max abs {par['logp_max_abs']:.2e} (all {T} tokens), dH rel-L2 {par['dh_rel_l2']:.2e}, "
                  f"dW rel-L2 {par['dw_rel_l2']:.2e}, zero rows zero {par['zero_grad_rows_zero']}; oracle on 16 "
                  f"rows: logp {e_lp_o:.2e}, dH rel-L2 {e_dh_o:.2e}", flush=True)
            ok = ok and par["ok"] and e_lp_o <= 2e-3 and e_dh_o <= 1e-2
        del lp, Hq
        # the other ranks wait here (host side) while rank 0 runs the CPU oracle, not inside
        # the next call's bounded device-side wait for rank 0
        dist.barrier(device_ids=[dev.index])
    return ok


def main() -> int:
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    os.environ.setdefault("LP_B200_PEER_TIMEOUT_MS", "10000")
    if rank == 0:  # the CPU oracle may use every core (torchrun gives each rank one thread)
        from threadpoolctl import threadpool_limits

        threadpool_limits(limits=len(os.sched_getaffinity(0)), user_api="blas")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    mesh = make_mesh()
    ok = True
    for mode in ("multimem", "nccl"):
        ok = check_per_token(mesh, dev, rank, world, mode, 1024 * world, 777, 160, 20260925) and ok
    ok = check_per_token(mesh, dev, rank, world, "nccl", 1024 * world, 777, 160, 20260925, stats_mode="nccl") and ok
    # several M / N tiles, split K over the vocabulary shard, ragged edges; the stats
    # exchange buffer grows (a new multicast buffer) for the larger token count
    ok = check_per_token(mesh, dev, rank, world, "multimem", 8192 * world, 2100, 392, 7) and ok
    ok = check_per_token(mesh, dev, rank, world, "multimem", 8192 * world, 2100, 392, 7, stats_mode="nccl") and ok
    ok = check_config2_shape(mesh, dev, rank, world, seed=11) and ok
    os.environ["LP_B200_DH_REDUCE"] = "multimem"
    os.environ["LP_B200_STATS_EXCHANGE"] = "multimem"
    rng = np.random.default_rng(20260926)
    V, d = 1024 * world, 160
    w = orc.bf16_round(rng.normal(size=(V, d)) * 1.5)
    W = shard_rows(torch.from_numpy(w), mesh).to(dev).to(torch.bfloat16)
    # GRPO caller, response slots compacted, same mesh
    B, Pw, N = 3, 5, 40
    hid = orc.bf16_round(rng.normal(size=(B, Pw + N, d)))
    ids = rng.integers(0, V, size=(B, N)).astype(np.int32)
    mask = np.arange(N)[None, :] < np.array([40, 7, 0])[:, None]
    Hd = torch.from_numpy(hid).to(dev).to(torch.bfloat16).requires_grad_(True)
    out = completion_logps(W, Hd, torch.from_numpy(ids).to(dev), torch.from_numpy(mask).to(dev),
                           prompt_width=Pw, softcap=30.0, mesh=mesh)
    out.sum().backward()
    if rank == 0:
        resp = hid[:, Pw - 1: Pw - 1 + N]
        ref = orc.dense_logps(w, resp, np.where(mask, ids, 0), 30.0)
        got = out.detach().cpu().numpy()
        e2 = float(np.abs(got[mask] - ref[mask]).max())
        print(f"world={world}: completion logp max abs {e2:.2e}, invalid slots zero: {(got[~mask] == 0).all()}",
              flush=True)
        ok = ok and e2 <= 2e-3 and bool((got[~mask] == 0).all())
        bi, ji = np.nonzero(mask)
        _, _, dHr = orc.logps_grads_f64(w, resp[bi, ji], ids[bi, ji], np.ones(len(bi), np.float32), 30.0)
        ref_dh = np.zeros(hid.shape)
        ref_dh[bi, Pw - 1 + ji] = dHr
        e3 = rel_l2(Hd.grad.float().cpu().numpy(), ref_dh)
        print(f"world={world}: completion dH rel-L2 {e3:.2e}", flush=True)
        ok = ok and e3 <= 1e-2
    flag = torch.tensor([1 if ok else 0], device=dev)
    dist.broadcast(flag, 0)
    dist.destroy_process_group()
    return 0 if int(flag.item()) == 1 else 1


if __name__ == "__main__":
    sys.exit(main())
