#!/usr/bin/env python
"""Benchmark of the B200 logprob path (one JSON line on rank 0).

Workload (the metric's configuration): GRPO-shaped response-only
logprob, forward + backward, tied LM head V=262144, d=2048, bf16, softcap 30. 128
sequences of 2048 (512 prompt + 1536 response slots), response lengths uniform in
[64, 1536], so ~102k valid response tokens per step; only those are computed
(compaction). Upstream dlogp = per-sequence advantage ~ N(0,1) x Bernoulli(0.9) keep.
The vocabulary is sharded over the N ranks (strong scaling: the global batch is fixed);
hidden states / targets are replicated as at the reference's shard_map boundary, the
per-token (max, sum, target) triples are all-gathered and merged, dH partials all-reduced.

A step = one call of the public API (``completion_logps``) + its backward on that batch:
compaction, fused LM-head GEMM + online LSE, combine, recompute backward into dZ, dH and dW
tensor-core GEMMs, scatter back. ``value`` has the inputs resident in HBM; ``e2e`` adds the
host->device copy of every step's inputs (pinned; double-buffered, so step k+1's copy runs
on the copy engines while step k computes) and the device->host read of the logps.

``--impl reference`` times the CPU restatement of the reference's native path
(``oracle/``; the reference itself is JAX-only and JAX is not installable here) on this
host's cores, on bounded samples of the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

B, PROMPT, RESP, D, V = 128, 512, 1536, 2048, 262144
SOFTCAP = 30.0
SEED = 0
METRIC = "logprob fwd+bwd tokens/s @V=262144,d=2048 (GRPO response tokens, vocab-sharded)"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# DRAM bytes (read + write) per launch of each GEMM on this workload at N=1, from one ncu
# capture (profiles/dram_traffic_grpo_config2_1gpu.md); backward launches: an 8192-row chunk.
NCU_TRAFFIC_PER_LAUNCH_N1 = {
    "fwd_lse_gemm": 20.01e9,
    "bwd_dz_gemm": 5.98e9,
    "bwd_dh_gemm": 10.92e9,
    "bwd_dw_gemm": 8.37e9,
}


# Dense-token BASELINE configs: (tokens, hidden, frozen head, extra forward-only pass).
DENSE_CONFIGS = {1: (256, 2048, False, False), 3: (65536, 2560, False, True), 4: (32768, 3840, True, False)}


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=("cuda", "reference"), default="cuda")
    p.add_argument("--softcap", type=float, default=SOFTCAP, help="<= 0 disables the softcap")
    p.add_argument("--batch", type=int, default=B, help="sequences (default: config 2's 128)")
    p.add_argument("--config", type=int, default=2, choices=(1, 2, 3, 4),
                   help="BASELINE config: 2 = GRPO response tokens (the metric's workload, default); "
                        "1 = T=256 dense; 3 = T=65536, d=2560 + forward-only pass of a perturbed head; "
                        "4 = T=32768, d=3840, frozen head (forward + dH)")
    p.add_argument("--tokens", type=int, default=0, help="override T of configs 1 / 3 / 4")
    p.add_argument("--token-chunk", type=int, default=0, help="backward token chunk (0 = library default)")
    p.add_argument("--cta-group", type=int, default=0, choices=(0, 1, 2),
                   help="tensor-core CTA group of the GEMMs (0 = library default, the CTA pair)")
    p.add_argument("--sampler-head", type=int, default=0, metavar="B",
                   help="instead: time the rollout sampler's LM head (lp_head) on B decode rows")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    return p.parse_args()


def load_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            d = json.loads(path.read_text())
            return {k: float(d[k]) for k in FALLBACK_PEAKS}, "measured"
        except Exception:  # noqa: BLE001
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def make_batch(batch: int, seed: int = SEED):
    """Seeded synthetic GRPO batch (host numpy for masks / ids / advantages)."""
    rng = np.random.default_rng(seed)
    prompt_len = rng.integers(128, PROMPT + 1, size=batch)  # left-padded to 512: does not move the slice
    resp_len = rng.integers(64, RESP + 1, size=batch)
    mask = np.arange(RESP)[None, :] < resp_len[:, None]
    ids = rng.integers(0, V, size=(batch, RESP)).astype(np.int32)
    adv = rng.normal(size=(batch, 1)).astype(np.float32)
    keep = rng.random((batch, RESP)) < 0.9
    g = np.where(mask & keep, adv, 0.0).astype(np.float32)
    return prompt_len, resp_len, mask, ids, g


def config_dict(batch, n_valid, world, softcap):
    return {
        "workload": "grpo_response_logprob_fwd_bwd (BASELINE config 2)",
        "global_batch": batch,
        "seq_len": PROMPT + RESP,
        "prompt_width": PROMPT,
        "response_width": RESP,
        "valid_tokens": int(n_valid),
        "hidden": D,
        "vocab": V,
        "vocab_per_gpu": V // world,
        "softcap": softcap if softcap > 0 else None,
        "parallelism": f"vocab{world}",
        "l2": "no flush: W shard + hidden exceed the 126 MB L2 (>= 0.8 GB each)",
    }


def cta_group_of_run():
    from gemma4_posttrain_jax_b200 import _lib

    return _lib.cta_group()


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = (
        "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
        "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
        "clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, indices):
        self.indices = indices
        self.proc = None
        self.file = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", ",".join(map(str, self.indices))],
                stdout=self.file, stderr=subprocess.DEVNULL,
            )
        except Exception:  # noqa: BLE001
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:  # noqa: BLE001
                self.proc.kill()

    def summary(self):
        if self.file is None:
            return None
        self.file.flush()
        rows = [r.split(",") for r in Path(self.file.name).read_text().splitlines() if r.strip()]
        os.unlink(self.file.name)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            r = [x.strip() for x in r]
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
            except ValueError:
                continue
            for name, val in zip(names, r[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": float(max(mx)), "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------------------- CPU baseline
def blas_threads() -> int:
    try:
        from threadpoolctl import threadpool_info

        n = [i.get("num_threads", 0) for i in threadpool_info() if i.get("user_api") == "blas"]
        if n:
            return int(max(n))
    except Exception:  # noqa: BLE001
        pass
    return os.cpu_count() or 1


def cpu_sample(W_host_f32, H_host, ids, mask, g, tokens, softcap):
    """Oracle fwd+bwd (float32, the reference's chunking) on the first `tokens` valid slots."""
    from oracle import logprob_oracle as orc

    b, j = np.nonzero(mask)
    b, j = b[:tokens], j[:tokens]
    h = H_host[b, j]
    t0 = time.perf_counter()
    orc.fwd_bwd_f32(W_host_f32, h, ids[b, j], g[b, j], softcap=softcap if softcap > 0 else None, vocab_chunk=8192,
                    sequence_chunk=128)
    return time.perf_counter() - t0


def host_inputs(batch, seed=SEED):
    """Seeded bf16 inputs drawn on the host (for the reference arm, which has no GPU)."""
    gen = torch.Generator(device="cpu").manual_seed(seed + 1)
    W = (torch.randn((V, D), generator=gen) * 0.02).to(torch.bfloat16)
    gen_h = torch.Generator(device="cpu").manual_seed(seed + 2)
    H = torch.randn((batch, RESP, D), generator=gen_h).to(torch.bfloat16)
    return W, H


# --------------------------------------------------------------------------- reference arm
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    _, _, mask, ids, g = make_batch(args.batch)
    W, H = host_inputs(args.batch)
    Wf = W.float().numpy()
    Hf = H.float().numpy()
    sample = 64
    for _ in range(args.warmup):
        cpu_sample(Wf, Hf, ids, mask, g, sample, args.softcap)
    secs = [cpu_sample(Wf, Hf, ids, mask, g, sample, args.softcap) for _ in range(args.steps)]
    per = float(np.mean(secs))
    value = sample / per
    cores = blas_threads()
    n_valid = int(mask.sum())
    line = {
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": per * 1e3,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded)",
        "config": config_dict(args.batch, n_valid, args.gpus, args.softcap),
        "impl": "reference",
        "cpu_baseline": {
            "value": value,
            "unit": "tokens/s",
            "cores": cores,
            "kind": "port",
            "sample": f"{sample} valid response tokens per step (fwd+bwd over the full V=262144, d=2048), "
            "numpy float32 restatement of losses.py:72-147 + its recompute backward",
        },
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------------------- sampler head
def run_sampler_head(args):
    """Decode-time LM head (lp_head) on B rows: greedy (no logits written) and full logits.

    HBM-bound: per launch it must read W (V * d * 2 bytes) and, with logits, write B * V * 4.
    """
    from gemma4_posttrain_jax_b200 import _lib, ops

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    _lib.load()
    B = args.sampler_head
    softcap = args.softcap if args.softcap > 0 else None
    gen = torch.Generator(device=dev).manual_seed(SEED + 1)
    W = (torch.randn((V, D), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
    H = torch.randn((B, D), generator=gen, device=dev).to(torch.bfloat16)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # 256 MB > L2 between launches
    peaks, peak_src = load_peaks()
    out = {}
    for mode, want in (("greedy", False), ("logits", True)):
        for _ in range(args.warmup):
            ops.head(W, H, softcap, want_logits=want)
        torch.cuda.synchronize()
        _lib.profile_enable(True)
        for _ in range(args.steps):
            flush.zero_()
            ops.head(W, H, softcap, want_logits=want)
        torch.cuda.synchronize()
        prof = _lib.profile_read()
        _lib.profile_enable(False)
        ms = sum(v[0] for v in prof.values()) / args.steps
        gemm_ms = prof["head_gemm"][0] / args.steps
        nbytes = V * D * 2 + (B * V * 4 if want else 0)
        out[mode] = {"ms_per_call": ms, "rows_per_s": B / (ms / 1e3), "gemm_ms": gemm_ms,
                     "algorithmic_bytes": nbytes, "achieved_gbs": nbytes / (gemm_ms / 1e3) / 1e9,
                     "frac_of_hbm": nbytes / (gemm_ms / 1e3) / 1e9 / peaks["hbm_gbs"]}
    assert _lib.device_error(0) == 0
    line = {
        "metric": f"sampler LM head rows/s @V={V},d={D} (lp_head, {B} decode rows)",
        "value": out["greedy"]["rows_per_s"], "unit": "rows/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "higher_is_better": True, "dtype": "bf16", "data": "synthetic (seeded)",
        "config": {"workload": "rollout sampler head (forward_lm_head + _sample_token log-softmax / argmax)",
                   "rows": B, "hidden": D, "vocab": V, "softcap": softcap, "l2": "flushed (256 MB) per launch"},
        "roofline": {"bound": "hbm", "achieved": out["greedy"]["achieved_gbs"], "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": out["greedy"]["frac_of_hbm"], "peak_source": f"hbm_gbs ({peak_src})"},
        "modes": out,
    }
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------------------- CUDA arm
def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.sampler_head:
        return run_sampler_head(args)

    import torch.distributed as dist

    from gemma4_posttrain_jax_b200 import _lib, build
    from gemma4_posttrain_jax_b200.losses import completion_logps
    from gemma4_posttrain_jax_b200.sharding import VocabMesh

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if not _lib.LIB_PATH.exists():
        build.build()
    _lib.load()
    if args.cta_group:
        _lib.set_cta_group(args.cta_group)
    mesh = None
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
        mesh = VocabMesh(None)

    softcap = args.softcap if args.softcap > 0 else None
    chunk = args.token_chunk or None
    from gemma4_posttrain_jax_b200.losses import per_token_logps

    if args.config == 2:
        d_model = D
        prompt_len, resp_len, mask_np, ids_np, g_np = make_batch(args.batch)
        n_valid = int(mask_np.sum())
        # rows the backward computes: valid tokens with nonzero dlogp (zero-gradient rows are
        # skipped by the library, as the reference's Pallas backward skips all-zero blocks)
        n_bwd = int((g_np[mask_np] != 0).sum())
        vs = V // world
        # inputs: the same seeded draws on every rank; each rank keeps its W row block
        gen = torch.Generator(device=dev).manual_seed(SEED + 1)
        W_full = (torch.randn((V, D), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
        W = W_full[rank * vs : (rank + 1) * vs].clone().requires_grad_(True)
        del W_full
        gen_h = torch.Generator(device=dev).manual_seed(SEED + 2)
        H = torch.randn((args.batch, RESP, D), generator=gen_h, device=dev).to(torch.bfloat16).requires_grad_(True)
        ids = torch.from_numpy(ids_np).to(dev)
        mask = torch.from_numpy(mask_np).to(dev)
        g = torch.from_numpy(g_np).to(dev)
        inputs = [H.detach(), ids, mask, g]
        fwd_launch_flops = 2.0 * n_valid * D * vs
        bwd_launch_flops = {"bwd_dz_gemm": 2.0 * n_bwd * D * vs, "bwd_dh_gemm": 2.0 * n_bwd * D * vs,
                            "bwd_dw_gemm": 2.0 * n_bwd * D * vs}
        total_flops_needed = 2.0 * n_valid * D * V + 6.0 * n_bwd * D * V
        dense_flops = 8.0 * n_valid * D * V

        def step(Hx, idsx, maskx, gx):
            Hx = Hx.detach().requires_grad_(True)
            lp = completion_logps(W, Hx, idsx, maskx, prompt_width=1, softcap=softcap, mesh=mesh, token_chunk=chunk,
                                  num_valid=n_valid)
            dW, dH = torch.autograd.grad(lp, (W, Hx), gx)
            return lp, dW, dH
    else:
        T_cfg, d_model, frozen, second_pass = DENSE_CONFIGS[args.config]
        T_cfg = args.tokens or T_cfg
        n_valid = n_bwd = T_cfg
        vs = V // world
        gen = torch.Generator(device=dev).manual_seed(SEED + 1)
        W_full = (torch.randn((V, d_model), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
        W = W_full[rank * vs : (rank + 1) * vs].clone().requires_grad_(not frozen)
        W2 = None
        if second_pass:  # old / reference policy head: W + N(0, 1e-4)
            W2 = (W.detach().float() + torch.randn(W.shape, generator=gen, device=dev) * 1e-4).to(torch.bfloat16)
        del W_full
        gen_h = torch.Generator(device=dev).manual_seed(SEED + 2)
        Hd = torch.randn((T_cfg, d_model), generator=gen_h, device=dev).to(torch.bfloat16)
        Yd = torch.randint(0, V, (T_cfg,), generator=gen_h, device=dev, dtype=torch.int32)
        Gd = torch.randn((T_cfg,), generator=gen_h, device=dev)
        inputs = [Hd, Yd, Gd]
        fwd_launch_flops = 2.0 * T_cfg * d_model * vs
        bwd_launch_flops = {"bwd_dz_gemm": 2.0 * T_cfg * d_model * vs, "bwd_dh_gemm": 2.0 * T_cfg * d_model * vs}
        if not frozen:
            bwd_launch_flops["bwd_dw_gemm"] = 2.0 * T_cfg * d_model * vs
        total_flops_needed = (2.0 * (2 if second_pass else 1) + (4.0 if frozen else 6.0)) * T_cfg * d_model * V
        dense_flops = total_flops_needed

        def step(Hx, Yx, Gx):
            Hx = Hx.detach().requires_grad_(True)
            lp = per_token_logps(W, Hx, Yx, softcap=softcap, mesh=mesh, token_chunk=chunk)
            wrt = (Hx,) if frozen else (W, Hx)
            grads = torch.autograd.grad(lp, wrt, Gx)
            if W2 is not None:
                with torch.no_grad():
                    lp2 = per_token_logps(W2, Hx.detach(), Yx, softcap=softcap, mesh=mesh)
                return lp, lp2, grads
            return lp, grads

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---------------------------------------------------------------- device-resident timing
    for _ in range(args.warmup):
        step(*inputs)
    torch.cuda.synchronize()
    assert _lib.device_error(local) == 0, "device-side error during warm-up"
    barrier()
    torch.cuda.synchronize()
    from gemma4_posttrain_jax_b200 import phase_timer

    _lib.profile_enable(True)
    phase_timer.enable(True)
    launches0 = _lib.launch_count()
    try:
        torch.cuda.reset_peak_memory_stats(dev)
    except Exception:  # noqa: BLE001 - the peak is a reported extra, never a reason to fail
        pass
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    step_marks = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(list(range(world))) as clocks:
        start.record()
        for i in range(args.steps):
            step(*inputs)
            step_marks[i].record()
        stop.record()
        torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    launches = (_lib.launch_count() - launches0) // max(args.steps, 1)
    prof = _lib.profile_read()
    _lib.profile_enable(False)
    phases = phase_timer.read()
    phase_timer.enable(False)
    ms = max_over_ranks(start.elapsed_time(stop) / args.steps)
    value = n_valid / (ms / 1e3)
    # per-step device times and peak device memory of this rank (the reference's harness
    # reports the mean, the p50 and the peak device bytes, bench.py:42-63)
    try:
        marks = [start, *step_marks]
        per_step = [marks[i].elapsed_time(marks[i + 1]) for i in range(args.steps)]
        step_stats = {"rank": rank, "p50_ms": float(np.median(per_step)), "min_ms": float(min(per_step)),
                      "max_ms": float(max(per_step)), "peak_device_bytes": int(torch.cuda.max_memory_allocated(dev))}
    except Exception:  # noqa: BLE001
        step_stats = None
    clock_summary = clocks.summary() if rank == 0 else None
    assert _lib.device_error(local) == 0, "device-side error during the timed region"

    # ---------------------------------------------------------------- end-to-end (host buffers)
    e2e = None
    if not args.no_e2e:
        # Every step copies its inputs from pinned host memory and reads its logps back. The
        # inputs are double-buffered: step k+1's host->device copies run on a copy stream
        # (copy engines) while step k computes, as a data loader would feed the trainer.
        hosts = [x.detach().cpu().pin_memory() for x in inputs]
        bufs = [[torch.empty_like(x) for x in inputs] for _ in range(2)]
        out_shape = (args.batch, RESP) if args.config == 2 else (n_valid,)
        out_host = torch.empty(out_shape, dtype=torch.float32).pin_memory()
        h2d = sum(x.nbytes for x in hosts)
        d2h = out_host.nbytes
        copy_stream = torch.cuda.Stream(dev)
        compute_done = [torch.cuda.Event() for _ in range(2)]
        copied = [torch.cuda.Event() for _ in range(2)]
        for ev in compute_done:
            ev.record()

        def issue_copy(k):
            b = k % 2
            with torch.cuda.stream(copy_stream):
                copy_stream.wait_event(compute_done[b])  # step k-2 no longer reads buffer b
                for hx, dx in zip(hosts, bufs[b]):
                    dx.copy_(hx, non_blocking=True)
                copied[b].record(copy_stream)

        def e2e_run(nsteps):
            issue_copy(0)
            for k in range(nsteps):
                b = k % 2
                if k + 1 < nsteps:
                    issue_copy(k + 1)
                torch.cuda.current_stream().wait_event(copied[b])
                out = step(*bufs[b])
                compute_done[b].record()
                out_host.copy_(out[0].detach(), non_blocking=True)

        e2e_run(args.warmup)
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        e2e_run(args.steps)
        e1.record()
        torch.cuda.synchronize()
        barrier()
        ems = max_over_ranks(e0.elapsed_time(e1) / args.steps)
        e2e = {"value": n_valid / (ems / 1e3), "unit": "tokens/s", "ms_per_step": ems, "h2d_bytes_per_step": int(h2d),
               "d2h_bytes_per_step": int(d2h)}

    # ---------------------------------------------------------------- roofline of the dominant kernel
    peaks, peak_src = load_peaks()
    n_fwd_passes = 2 if (args.config == 3) else 1
    flops_per_step = {"fwd_lse_gemm": fwd_launch_flops * n_fwd_passes, **bwd_launch_flops}
    kernels = {}
    for name, (tot_ms, cnt) in prof.items():
        per_launch = tot_ms / max(cnt, 1)
        entry = {"launches_per_step": cnt / args.steps, "ms_per_step": tot_ms / args.steps, "ms_per_launch": per_launch}
        if name in flops_per_step:
            tf = flops_per_step[name] * args.steps / (tot_ms / 1e3) / 1e12
            entry["tflops"] = tf
            entry["frac_of_sustained_peak"] = tf / peaks["bf16_tflops_sustained"]
        kernels[name] = entry
    gemm_names = [k for k in kernels if k in flops_per_step]
    dom = max(gemm_names, key=lambda k: kernels[k]["ms_per_step"]) if gemm_names else None
    roofline = None
    if dom is not None:
        cnt = prof[dom][1]
        flop_per_launch = flops_per_step[dom] * args.steps / max(cnt, 1)
        achieved = flop_per_launch / (kernels[dom]["ms_per_launch"] / 1e3) / 1e12
        roofline = {
            "kernel": dom,
            "bound": "tensor",
            "achieved": achieved,
            "peak": peaks["bf16_tflops_sustained"],
            "unit": "TFLOP/s",
            "frac": achieved / peaks["bf16_tflops_sustained"],
            "traffic": (NCU_TRAFFIC_PER_LAUNCH_N1.get(dom)
                        if world == 1 and args.config == 2 and args.batch == B and args.softcap == SOFTCAP else None),
            "traffic_unit": "bytes per launch (ncu dram__bytes_read.sum + dram__bytes_write.sum)",
            "peak_source": f"bf16_tflops_sustained ({peak_src}); kernel runs inside a long step",
            "flop_per_launch": flop_per_launch,
        }
    step_tflops = total_flops_needed / (ms / 1e3) / 1e12  # the GEMM work one step needs
    dense_equiv_tflops = dense_flops / (ms / 1e3) / 1e12  # the 8*T*d*V roofline's count (config 2)

    # ---------------------------------------------------------------- CPU baseline (rank 0, N = 1)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.config == 2:
        Wf = W.detach().float().cpu().numpy()
        Hf = H.detach().float().cpu().numpy()
        sample = 64
        t = cpu_sample(Wf, Hf, ids_np, mask_np, g_np, sample, args.softcap)
        if t < 4.0:
            sample = 256
            t = cpu_sample(Wf, Hf, ids_np, mask_np, g_np, sample, args.softcap)
        cpu = {"value": sample / t, "unit": "tokens/s", "cores": blas_threads(), "kind": "port",
               "sample": f"{sample} valid response tokens of this workload, fwd+bwd over V=262144, d=2048 "
               f"({t:.1f} s), numpy float32 restatement of losses.py:72-147 + recompute backward"}

    if rank == 0:
        metric = METRIC if args.config == 2 else (
            f"logprob tokens/s @V=262144,d={d_model} (BASELINE config {args.config}, vocab-sharded)")
        cfg = config_dict(args.batch, n_valid, world, args.softcap) if args.config == 2 else {
            "workload": f"BASELINE config {args.config}: "
            + {1: "dense fwd+bwd", 3: "dense fwd+bwd + forward-only pass of W + N(0,1e-4)",
               4: "dense fwd + dH, frozen head"}[args.config],
            "tokens": n_valid, "hidden": d_model, "vocab": V, "vocab_per_gpu": vs,
            "softcap": args.softcap if args.softcap > 0 else None, "parallelism": f"vocab{world}",
            "l2": "no flush: W shard exceeds the 126 MB L2"}
        line = {
            "metric": metric,
            "value": value,
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) hidden, N(0,0.02) W, uniform targets)",
            "config": cfg,
            "clocks": clock_summary,
            "e2e": e2e,
            "gpu_launches": int(launches),
            "roofline": roofline,
            "cpu_baseline": cpu,
            "step_tflops": step_tflops,
            "step_frac_of_sustained_peak": step_tflops / world / peaks["bf16_tflops_sustained"],
            "dense_8Tdv_tflops": dense_equiv_tflops,
            "backward_rows": n_bwd,
            "kernels": kernels,
            "host_phases_ms_per_step": {k: v[0] / args.steps for k, v in phases.items()},
            "kernel_ms_per_step": sum(v["ms_per_step"] for v in kernels.values()),
            "step_stats": step_stats,
            "cta_group": cta_group_of_run(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
