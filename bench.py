#!/usr/bin/env python
"""Benchmark of the B200 logprob path (one JSON line on rank 0).

Workload (the metric's configuration): GRPO-shaped response-only
logprob, forward + backward, tied LM head V=262144, d=2048, bf16, softcap 30. 128
sequences of 2048 (512 prompt + 1536 response slots), response lengths uniform in
[64, 1536], so ~108k valid response tokens per step; only those are computed
(compaction). Upstream dlogp = per-sequence advantage ~ N(0,1) x Bernoulli(0.9) keep.
The vocabulary is sharded over the N ranks (strong scaling: the global batch is fixed);
hidden states / targets are replicated as at the reference's shard_map boundary, the
per-token (max, sum, target) triples are exchanged inside the forward and the dH partials
summed inside the dH GEMM (NVLink multicast), or by NCCL where that is unavailable.

A step = one call of the public API (``completion_logps``) + its backward on that batch:
compaction, fused LM-head GEMM + online LSE, combine, recompute backward into dZ, dH and dW
tensor-core GEMMs, scatter back. ``value`` has the inputs resident in HBM; ``e2e`` adds the
host->device copy of every step's inputs (pinned; double-buffered, so step k+1's copy runs
on the copy engines while step k computes) and the device->host read of the logps. With
N ranks each rank copies 1/N of the input bytes from host memory and pulls the other ranks'
parts over NVLink (``StepLoader``), so the whole job moves the inputs across PCIe once.

After the timed regions one more step is checked against a PyTorch float32 reference of
the same arithmetic computed on the GPUs (``parity``): the logp of every token, dH on 256
sampled rows and dW on 256 sampled vocabulary rows of every shard, at the bars of the
scope table (logp within 2e-3 absolute, dH / dW within 1e-2 relative L2). A failed check
still prints the line, then exits with status 3.

``--impl reference`` times the CPU restatement of the reference's native path
(``oracle/``; the reference itself is JAX-only and JAX is not installable here) on this
host's cores, on bounded samples of the same workload.
"""

from __future__ import annotations

import argparse
import datetime as _dt
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
# DRAM bytes (read + write) per launch of the forward GEMM on this workload at N=1: a stored
# constant, not measured by this run. It comes from an ncu capture of the batch-16 case of
# this workload (13,969 tokens: 2.766 GB read + 0.061 GB written by the forward launch, CTA
# pairs, of
# ``ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum,gpu__time_duration.sum
# --clock-control none -k regex:tc_gemm -s 39 -c 13 python bench.py --batch 16 --steps 1
# --warmup 3 --no-e2e --no-cpu-baseline --no-parity --token-chunk 4096``), scaled by the
# tokens of the full batch (the forward streams W once per 12,288-token block of hidden
# rows, so its traffic grows in proportion to the token count at a fixed vocabulary).
NCU_FWD_TRAFFIC_PER_TOKEN_N1 = (2.766e9 + 0.061e9) / 13969
NCU_TRAFFIC_NOTE = "stored constant: ncu DRAM bytes of the forward GEMM per token (batch-16 capture), x tokens"
# The same capture's dZ GEMM launches (4096-row chunks): 1.093 GB read (W once, the chunk's
# hidden rows) + 2.109 GB written (the chunk's bf16 dZ). A launch reads W once as long as its
# chunk is at most one 12,288-row block, so its traffic is that read plus its rows' writes.
NCU_DZ_READ_PER_LAUNCH_N1 = 1.093e9
NCU_DZ_WRITE_PER_ROW_N1 = 2.109e9 / 4096
NCU_DZ_TRAFFIC_NOTE = ("stored constant: ncu DRAM bytes of a dZ GEMM launch (batch-16 capture): W read once "
                       "+ dZ bytes written per row x rows per launch")
LOGP_ATOL, GRAD_RTOL = 2e-3, 1e-2

# Dense-token BASELINE configs: (tokens, hidden, frozen head, extra forward-only pass).
DENSE_CONFIGS = {1: (256, 2048, False, False), 3: (65536, 2560, False, True), 4: (32768, 3840, True, False),
                 5: (65536, 2048, False, False)}
DENSE_NAMES = {1: "dense fwd+bwd", 3: "dense fwd+bwd + forward-only pass of W + N(0,1e-4)",
               4: "dense fwd + dH, frozen head", 5: "dense fwd+bwd (T sweep)"}


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=("cuda", "reference"), default="cuda")
    p.add_argument("--softcap", type=float, default=SOFTCAP, help="<= 0 disables the softcap")
    p.add_argument("--batch", type=int, default=B, help="sequences (default: config 2's 128)")
    p.add_argument("--config", type=int, default=2, choices=(1, 2, 3, 4, 5),
                   help="BASELINE config: 2 = GRPO response tokens (the metric's workload, default); "
                        "1 = T=256 dense; 3 = T=65536, d=2560 + forward-only pass of a perturbed head; "
                        "4 = T=32768, d=3840, frozen head (forward + dH); 5 = dense d=2048 (T sweep)")
    p.add_argument("--tokens", type=str, default="",
                   help="T of configs 1 / 3 / 4 / 5; a comma-separated list runs each T in turn (one line each)")
    p.add_argument("--token-chunk", type=int, default=0, help="backward token chunk (0 = library default)")
    p.add_argument("--cta-group", type=int, default=0, choices=(0, 1, 2),
                   help="tensor-core CTA group of the GEMMs (0 = library default, per GEMM)")
    p.add_argument("--sampler-head", type=int, default=0, metavar="B",
                   help="instead: time the rollout sampler's LM head (lp_head) on B decode rows")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-parity", action="store_true", help="skip the float32 check of one step's results")
    p.add_argument("--vocab-per-gpu", type=int, default=0,
                   help="tuning only: vocabulary rows per GPU (default V / N); e.g. 32768 on one GPU runs the "
                        "per-GPU shard of an 8-GPU mesh without its collectives (the line's vocab says so)")
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


def make_batch(batch: int, seed: int = SEED, vocab: int = V):
    """Seeded synthetic GRPO batch (host numpy for masks / ids / advantages)."""
    rng = np.random.default_rng(seed)
    prompt_len = rng.integers(128, PROMPT + 1, size=batch)  # left-padded to 512: does not move the slice
    resp_len = rng.integers(64, RESP + 1, size=batch)
    mask = np.arange(RESP)[None, :] < resp_len[:, None]
    ids = rng.integers(0, vocab, size=(batch, RESP)).astype(np.int32)
    adv = rng.normal(size=(batch, 1)).astype(np.float32)
    keep = rng.random((batch, RESP)) < 0.9
    g = np.where(mask & keep, adv, 0.0).astype(np.float32)
    return prompt_len, resp_len, mask, ids, g


def config_dict(batch, n_valid, world, softcap, vocab=V):
    return {
        "workload": "grpo_response_logprob_fwd_bwd (BASELINE config 2)",
        "global_batch": batch,
        "seq_len": PROMPT + RESP,
        "prompt_width": PROMPT,
        "response_width": RESP,
        "valid_tokens": int(n_valid),
        "hidden": D,
        "vocab": vocab,
        "vocab_per_gpu": vocab // world,
        "softcap": softcap if softcap > 0 else None,
        "parallelism": f"vocab{world}",
        "l2": "no flush: W shard + hidden exceed the 126 MB L2 (>= 0.8 GB each)",
    }


def cta_group_of_run():
    from gemma4_posttrain_jax_b200 import _lib

    return _lib.cta_group()


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples (every 200 ms) of the GPUs' clocks and throttle reasons, started
    before the warm-up so that samples exist for short timed regions; ``summary`` keeps the
    samples that fall inside the marked windows."""

    FIELDS = (
        "timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, indices):
        self.indices = indices
        self.proc = None
        self.file = None

    def start(self):
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

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:  # noqa: BLE001
                self.proc.kill()
            self.proc = None
        if self.file is not None:
            self.file.close()
            os.unlink(self.file.name)
            self.file = None

    def _rows(self):
        if self.file is None:
            return []
        self.file.flush()
        out = []
        for line in Path(self.file.name).read_text().splitlines():
            r = [x.strip() for x in line.split(",")]
            if len(r) < 10:
                continue
            try:
                ts = _dt.datetime.strptime(r[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                out.append((ts, float(r[2]), float(r[3]), r[6:10]))
            except ValueError:
                continue
        return out

    def summary(self, windows, since):
        """Median SM clock and the active throttle reasons over the samples inside `windows`
        ((start, end) wall-clock pairs); with fewer than two such samples (timed regions
        shorter than the sampling period) over every sample since `since` (the warm-up)."""
        rows = self._rows()
        if not rows:
            return None
        inside = [r for r in rows if any(a - 0.1 <= r[0] <= b + 0.1 for a, b in windows)]
        window = "timed regions"
        if len(inside) < 2:
            inside = [r for r in rows if r[0] >= since]
            window = "warm-up + timed regions"
        if not inside:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in inside for n, v in zip(names, r[3]) if v.lower().startswith("active")})
        return {"sm_mhz": float(np.median([r[1] for r in inside])), "sm_max_mhz": float(max(r[2] for r in inside)),
                "reasons": reasons, "samples": len(inside), "window": window}


# --------------------------------------------------------------------------- CPU baseline
def use_all_host_cores() -> int:
    """Let numpy's BLAS use every core this process may run on (torchrun sets
    OMP_NUM_THREADS=1 for its ranks); returns the thread count in effect."""
    try:
        n = len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover - non-Linux
        n = os.cpu_count() or 1
    try:
        from threadpoolctl import threadpool_limits

        threadpool_limits(limits=n, user_api="blas")
    except Exception:  # noqa: BLE001
        pass
    torch.set_num_threads(n)
    return blas_threads(default=n)


def blas_threads(default: int | None = None) -> int:
    try:
        from threadpoolctl import threadpool_info

        n = [i.get("num_threads", 0) for i in threadpool_info() if i.get("user_api") == "blas"]
        if n:
            return int(max(n))
    except Exception:  # noqa: BLE001
        pass
    return default or os.cpu_count() or 1


CPU_SAMPLE_TOKENS = 256  # BASELINE config 1's T, taken from this workload's valid tokens


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
    cores = use_all_host_cores()
    _, _, mask, ids, g = make_batch(args.batch)
    W, H = host_inputs(args.batch)
    Wf = W.float().numpy()
    Hf = H.float().numpy()
    sample = CPU_SAMPLE_TOKENS
    for _ in range(args.warmup):
        cpu_sample(Wf, Hf, ids, mask, g, sample, args.softcap)
    secs = [cpu_sample(Wf, Hf, ids, mask, g, sample, args.softcap) for _ in range(args.steps)]
    per = float(np.mean(secs))
    value = sample / per
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
            "sample": f"{sample} valid response tokens of this workload per step (fwd+bwd over the full V=262144, "
            "d=2048, the arithmetic of BASELINE config 1), numpy float32 restatement of losses.py:72-147 + its "
            "recompute backward",
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


# --------------------------------------------------------------------------- float32 parity check
class Ranks:
    """The collectives of the check (no-ops on one GPU); every rank makes the same calls."""

    def __init__(self, world: int):
        self.world = world

    def all_reduce(self, t: torch.Tensor, op: str) -> torch.Tensor:
        if self.world > 1:
            import torch.distributed as dist

            dist.all_reduce(t, op={"sum": dist.ReduceOp.SUM, "max": dist.ReduceOp.MAX}[op])
        return t


def parity_check(W, Hv, yv, gv, lp_v, dW, dHv, *, softcap, rank, world, dev, seed=1234, rows=256):
    """Compare one step's results with a float32 PyTorch computation of the same math.

    W: this rank's shard bf16 [Vs, d]; Hv bf16 [T, d], yv int [T] global ids, gv f32 [T]:
    the tokens of the step; lp_v f32 [T], dW [Vs, d] (or None: frozen head), dHv [T, d]:
    what the library returned. The reference forms every logit in float32 (exact bf16
    products, float32 sums, as ``_matmul_f32``), the softcap, the log-sum-exp over every
    shard, and from them the softmax-minus-one-hot gradients of sampled dH rows (over every
    shard) and sampled dW rows (all tokens). Returns the error summary (same on every rank).
    """
    torch.set_float32_matmul_precision("highest")
    ranks = Ranks(world)
    T, d = Hv.shape
    Vs = W.shape[0]
    off = rank * Vs
    Wf = W.detach().float()
    cap = float(softcap) if softcap else None

    def capped(z):
        return cap * torch.tanh(z / cap) if cap else z

    def chain(zc):  # d softcap / dz, from the capped value
        return 1.0 - (zc / cap) ** 2 if cap else torch.ones_like(zc)

    y_local = yv.to(torch.int64) - off
    owned = (y_local >= 0) & (y_local < Vs)
    m = torch.empty(T, device=dev)
    s = torch.empty(T, device=dev)
    tgt = torch.zeros(T, device=dev)
    CH = max(256, min(8192, (1 << 30) // max(Vs, 1)))  # <= 4 GB of float32 logits per chunk
    for t0 in range(0, T, CH):
        t1 = min(T, t0 + CH)
        z = capped(Hv[t0:t1].float() @ Wf.T)
        mz = z.max(dim=1).values
        m[t0:t1] = mz
        s[t0:t1] = torch.exp(z - mz[:, None]).sum(dim=1)
        li = y_local[t0:t1].clamp(0, Vs - 1)
        tgt[t0:t1] = torch.where(owned[t0:t1], z.gather(1, li[:, None]).squeeze(1), torch.zeros_like(mz))
        del z
    m_g = ranks.all_reduce(m.clone(), "max")
    s_g = ranks.all_reduce(s * torch.exp(m - m_g), "sum")
    tgt_g = ranks.all_reduce(tgt, "sum")
    lse = m_g + torch.log(s_g)
    lp_ref = tgt_g - lse
    e_lp = float((lp_v.float() - lp_ref).abs().max()) if T else 0.0

    gen = torch.Generator(device=dev).manual_seed(seed)  # same draw on every rank
    nz = torch.nonzero(gv != 0).squeeze(1)
    R = nz[torch.randperm(nz.numel(), generator=gen, device=dev)[:rows]].sort().values
    zR = capped(Hv[R].float() @ Wf.T)
    oh = torch.zeros_like(zR)
    rr = torch.nonzero(owned[R]).squeeze(1)
    oh[rr, y_local[R][rr]] = 1.0
    dz = gv[R][:, None] * (oh - torch.exp(zR - lse[R][:, None])) * chain(zR)
    dH_ref = ranks.all_reduce(dz @ Wf, "sum")
    dH_got = dHv[R].float()
    e_dh = float(torch.linalg.norm(dH_got - dH_ref) / torch.linalg.norm(dH_ref)) if R.numel() else 0.0
    zero_rows = torch.nonzero(gv == 0).squeeze(1)[:1024]
    zero_ok = bool((dHv[zero_rows] == 0).all()) if zero_rows.numel() else True

    e_dw = 0.0
    if dW is not None:
        genr = torch.Generator(device=dev).manual_seed(seed + 1 + rank)
        tg = torch.unique(y_local[owned][:128])
        extra = torch.randperm(Vs, generator=genr, device=dev)[: max(0, rows - tg.numel())]
        C = torch.unique(torch.cat([tg, extra]))[:rows]
        Hf = Hv.float()
        zC = capped(Hf @ Wf[C].T)  # [T, |C|]
        ohC = (y_local[:, None] == C[None, :]).float()
        dzC = gv[:, None] * (ohC - torch.exp(zC - lse[:, None])) * chain(zC)
        dW_ref = dzC.T @ Hf
        e = torch.linalg.norm(dW[C].float() - dW_ref) / torch.linalg.norm(dW_ref)
        e_dw = float(ranks.all_reduce(e.reshape(1).clone(), "max")[0])
    e_lp = float(ranks.all_reduce(torch.tensor([e_lp], device=dev), "max")[0])
    e_dh = float(ranks.all_reduce(torch.tensor([e_dh], device=dev), "max")[0])
    ok = e_lp <= LOGP_ATOL and e_dh <= GRAD_RTOL and e_dw <= GRAD_RTOL and zero_ok
    return {"logp_max_abs": e_lp, "dh_rel_l2": e_dh, "dw_rel_l2": e_dw if dW is not None else None,
            "zero_grad_rows_zero": zero_ok, "tokens_checked": int(T), "dh_rows": int(R.numel()),
            "dw_rows_per_shard": int(rows) if dW is not None else 0,
            "bars": {"logp_abs": LOGP_ATOL, "grad_rel_l2": GRAD_RTOL},
            "reference": "PyTorch float32 on the GPUs (exact bf16 products, float32 sums), every shard", "ok": ok}


# --------------------------------------------------------------------------- workloads
class Workload:
    """One benchmark configuration: inputs, the step, FLOP counts and the parity view."""

    def __init__(self, **kw):
        self.__dict__.update(kw)


def grpo_workload(args, dev, rank, world, mesh, softcap, chunk):
    from gemma4_posttrain_jax_b200.losses import completion_logps

    vs = args.vocab_per_gpu or V // world
    vocab = vs * world
    prompt_len, resp_len, mask_np, ids_np, g_np = make_batch(args.batch, vocab=vocab)
    n_valid = int(mask_np.sum())
    # rows the backward computes: valid tokens with nonzero dlogp (zero-gradient rows are
    # skipped by the library, as the reference's Pallas backward skips all-zero blocks)
    n_bwd = int((g_np[mask_np] != 0).sum())
    # inputs: the same seeded draws on every rank; each rank keeps its W row block
    gen = torch.Generator(device=dev).manual_seed(SEED + 1)
    W_full = (torch.randn((vocab, D), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
    W = W_full[rank * vs : (rank + 1) * vs].clone().requires_grad_(True)
    del W_full
    gen_h = torch.Generator(device=dev).manual_seed(SEED + 2)
    H = torch.randn((args.batch, RESP, D), generator=gen_h, device=dev).to(torch.bfloat16)
    ids = torch.from_numpy(ids_np).to(dev)
    mask = torch.from_numpy(mask_np).to(dev)
    g = torch.from_numpy(g_np).to(dev)

    def step(Hx, idsx, maskx, gx):
        Hx = Hx.detach().requires_grad_(True)
        lp = completion_logps(W, Hx, idsx, maskx, prompt_width=1, softcap=softcap, mesh=mesh, token_chunk=chunk,
                              num_valid=n_valid)
        dW, dH = torch.autograd.grad(lp, (W, Hx), gx)
        return lp, dW, dH

    def parity_view(out):
        lp, dW, dH = out
        extra_ok = bool((lp[~mask] == 0).all()) and bool((dH[~mask] == 0).all())
        return dict(Hv=H[mask], yv=ids[mask], gv=g[mask], lp_v=lp[mask], dW=dW, dHv=dH[mask]), extra_ok

    bwd = 2.0 * n_bwd * D * vs
    return Workload(
        W=W, inputs=[H, ids, mask, g], step=step, parity_view=parity_view, n_valid=n_valid, n_bwd=n_bwd, d=D, vs=vs,
        flops={"fwd_lse_gemm": 2.0 * n_valid * D * vs, "bwd_dz_gemm": bwd, "bwd_dh_gemm": bwd, "bwd_dw_gemm": bwd},
        total_flops=2.0 * n_valid * D * vocab + 6.0 * n_bwd * D * vocab, dense_flops=8.0 * n_valid * D * vocab,
        out_shape=(args.batch, RESP), metric=METRIC if vocab == V else f"{METRIC} [tuning: vocab {vocab}]",
        config=config_dict(args.batch, n_valid, world, args.softcap, vocab),
        traffic_ok=world == 1 and vocab == V and args.batch == B and args.softcap == SOFTCAP)


def dense_workload(args, dev, rank, world, mesh, softcap, chunk, T_cfg):
    from gemma4_posttrain_jax_b200.losses import per_token_logps

    _, d_model, frozen, second_pass = DENSE_CONFIGS[args.config]
    vs = args.vocab_per_gpu or V // world
    vocab = vs * world
    gen = torch.Generator(device=dev).manual_seed(SEED + 1)
    W_full = (torch.randn((vocab, d_model), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
    W = W_full[rank * vs : (rank + 1) * vs].clone().requires_grad_(not frozen)
    W2 = None
    if second_pass:  # old / reference policy head: W + N(0, 1e-4)
        W2 = (W.detach().float() + torch.randn(W.shape, generator=gen, device=dev) * 1e-4).to(torch.bfloat16)
    del W_full
    gen_h = torch.Generator(device=dev).manual_seed(SEED + 2)
    Hd = torch.randn((T_cfg, d_model), generator=gen_h, device=dev).to(torch.bfloat16)
    Yd = torch.randint(0, vocab, (T_cfg,), generator=gen_h, device=dev, dtype=torch.int32)
    Gd = torch.randn((T_cfg,), generator=gen_h, device=dev)

    def step(Hx, Yx, Gx):
        Hx = Hx.detach().requires_grad_(True)
        lp = per_token_logps(W, Hx, Yx, softcap=softcap, mesh=mesh, token_chunk=chunk)
        if frozen:
            (dH,) = torch.autograd.grad(lp, (Hx,), Gx)
            dW = None
        else:
            dW, dH = torch.autograd.grad(lp, (W, Hx), Gx)
        if W2 is not None:
            with torch.no_grad():
                per_token_logps(W2, Hx.detach(), Yx, softcap=softcap, mesh=mesh)
        return lp, dW, dH

    def parity_view(out):
        lp, dW, dH = out
        return dict(Hv=Hd, yv=Yd, gv=Gd, lp_v=lp, dW=dW, dHv=dH), True

    flops = {"fwd_lse_gemm": 2.0 * T_cfg * d_model * vs * (2 if second_pass else 1),
             "bwd_dz_gemm": 2.0 * T_cfg * d_model * vs, "bwd_dh_gemm": 2.0 * T_cfg * d_model * vs}
    if not frozen:
        flops["bwd_dw_gemm"] = 2.0 * T_cfg * d_model * vs
    total = (2.0 * (2 if second_pass else 1) + (4.0 if frozen else 6.0)) * T_cfg * d_model * vocab
    cfg = {"workload": f"BASELINE config {args.config}: {DENSE_NAMES[args.config]}", "tokens": T_cfg,
           "hidden": d_model, "vocab": vocab, "vocab_per_gpu": vs, "softcap": args.softcap if args.softcap > 0 else None,
           "parallelism": f"vocab{world}", "l2": "no flush: W shard exceeds the 126 MB L2"}
    return Workload(
        W=W, inputs=[Hd, Yd, Gd], step=step, parity_view=parity_view, n_valid=T_cfg, n_bwd=T_cfg, d=d_model, vs=vs,
        flops=flops, total_flops=total, dense_flops=total, out_shape=(T_cfg,),
        metric=f"logprob tokens/s @V={vocab},d={d_model} (BASELINE config {args.config}, vocab-sharded)", config=cfg,
        traffic_ok=False)


# --------------------------------------------------------------------------- step-input loader
def byte_parts(total: int, world: int, align: int = 256) -> list[int]:
    """Bounds of ``world`` contiguous byte ranges covering ``total`` bytes, each starting on
    an ``align``-byte boundary (rank r copies [b[r], b[r+1]) from host memory)."""
    b = [min(total, -(-(total * r // world) // align) * align) for r in range(world)] + [total]
    return b


def pack_layout(inputs, align: int = 256):
    """Byte offset of each input in one packed buffer, and the buffer's size."""
    offs, pos = [], 0
    for x in inputs:
        pos = -(-pos // align) * align
        offs.append(pos)
        pos += x.nbytes
    return offs, -(-pos // align) * align


class StepLoader:
    """Feeds every step's inputs from pinned host memory to the GPUs, as a data loader does.

    The inputs are packed into one pinned host buffer and two device slots (double
    buffering: step k+1's copies run while step k computes). With N > 1 ranks every rank
    needs all of the inputs (they are replicated at the vocabulary-parallel boundary), but
    only 1/N of the bytes cross PCIe on each rank: rank r copies its byte range from host
    memory into its slot, and after a host barrier pulls the other ranks' ranges from their
    slots over NVLink (copy-engine peer copies from symmetric memory; no kernel waits on a
    peer). Without symmetric memory on every rank, every rank copies all bytes from host.

    A background thread does the copies, so the host barrier and the peer copies overlap the
    previous step's compute. Slot safety: step k's copies into slot k % 2 start once step
    k - 2 (its last reader on this rank) has finished, and every rank's pulls of step k - 2
    complete before the barrier of step k - 1, which comes before any rank overwrites its
    range of that slot.
    """

    def __init__(self, inputs, *, dev, rank, world, gloo_group=None):
        import torch.distributed as dist

        self.dev, self.rank, self.world = dev, rank, world
        self.offs, self.total = pack_layout(inputs)
        self.host = torch.empty(self.total, dtype=torch.uint8).pin_memory()
        for x, o in zip(inputs, self.offs):
            self.host[o:o + x.nbytes].copy_(x.detach().contiguous().view(-1).view(torch.uint8).cpu())
        self.sharded = False
        self.slots, self.peers = [], []
        if world > 1:
            try:
                import torch.distributed._symmetric_memory as symm_mem

                slots = [symm_mem.empty((self.total,), dtype=torch.uint8, device=dev) for _ in range(2)]
                ok = 1
            except (RuntimeError, ImportError):  # includes torch.OutOfMemoryError
                slots, ok = [], 0
            flag = torch.tensor([ok], dtype=torch.int32, device=dev)
            dist.all_reduce(flag, op=dist.ReduceOp.MIN)
            if int(flag.item()) == 1:
                for s in slots:
                    h = symm_mem.rendezvous(s, dist.group.WORLD)
                    self.peers.append([h.get_buffer(p, (self.total,), torch.uint8) for p in range(world)])
                self.slots, self.sharded = slots, True
        if not self.sharded:
            self.slots = [torch.empty(self.total, dtype=torch.uint8, device=dev) for _ in range(2)]
        self.gloo = gloo_group
        self.bounds = byte_parts(self.total, world) if self.sharded else [0, self.total]
        mine = (self.bounds[rank], self.bounds[rank + 1]) if self.sharded else (0, self.total)
        self.mine = mine
        self.views = [[s[o:o + x.nbytes].view(x.dtype).view(x.shape) for x, o in zip(inputs, self.offs)]
                      for s in self.slots]
        self.copy_stream = torch.cuda.Stream(dev)
        # one stream per peer, so the pulls run on several copy engines at once
        self.pull_streams = [torch.cuda.Stream(dev) for _ in range(world - 1)] if self.sharded else []
        self.compute_done = [torch.cuda.Event() for _ in range(2)]
        self.copied = [torch.cuda.Event() for _ in range(2)]
        for ev in self.compute_done:
            ev.record()

    @property
    def h2d_bytes(self) -> int:
        return self.mine[1] - self.mine[0]

    @property
    def peer_bytes(self) -> int:
        return self.total - self.h2d_bytes if self.sharded else 0

    def _produce(self, nsteps, state):
        import torch.distributed as dist

        try:
            torch.cuda.set_device(self.dev)
            cs = self.copy_stream
            lo, hi = self.mine
            for k in range(nsteps):
                s = k % 2
                with state["cv"]:
                    # the main thread has enqueued step k - 2 (recorded its compute_done)
                    if not state["cv"].wait_for(lambda: state["enqueued"] >= k - 1 or state["stop"], timeout=300):
                        raise TimeoutError(f"loader: step {k - 2} was never enqueued")
                    if state["stop"]:
                        return
                with torch.cuda.stream(cs):
                    cs.wait_event(self.compute_done[s])
                    if hi > lo:
                        self.slots[s][lo:hi].copy_(self.host[lo:hi], non_blocking=True)
                cs.synchronize()
                if self.sharded:
                    dist.barrier(group=self.gloo)
                    others = [p for p in range(self.world) if p != self.rank]
                    for p, ps in zip(others, self.pull_streams):
                        a, b = self.bounds[p], self.bounds[p + 1]
                        if b > a:
                            with torch.cuda.stream(ps):
                                self.slots[s][a:b].copy_(self.peers[s][p][a:b], non_blocking=True)
                        cs.wait_stream(ps)
                with torch.cuda.stream(cs):
                    self.copied[s].record(cs)
                cs.synchronize()
                with state["cv"]:
                    state["ready"] = k + 1
                    state["cv"].notify_all()
        except BaseException as e:  # surfaced by run()
            with state["cv"]:
                state["error"] = e
                state["cv"].notify_all()

    def run(self, nsteps, step, out_host):
        """``nsteps`` steps of ``step(*inputs)``, each fed by the loader; every step's logps
        (``out[0]``) are read back into ``out_host``."""
        import threading

        state = {"cv": threading.Condition(), "enqueued": 0, "ready": 0, "stop": False, "error": None}
        t = threading.Thread(target=self._produce, args=(nsteps, state), daemon=True)
        t.start()
        try:
            for k in range(nsteps):
                s = k % 2
                with state["cv"]:
                    state["cv"].wait_for(lambda: state["ready"] > k or state["error"] is not None, timeout=600)
                    if state["error"] is not None:
                        raise RuntimeError("step-input loader failed") from state["error"]
                    if state["ready"] <= k:
                        raise TimeoutError(f"loader: inputs of step {k} never arrived")
                torch.cuda.current_stream().wait_event(self.copied[s])
                out = step(*self.views[s])
                self.compute_done[s].record()
                out_host.copy_(out[0].detach(), non_blocking=True)
                with state["cv"]:
                    state["enqueued"] = k + 1
                    state["cv"].notify_all()
        finally:
            with state["cv"]:
                state["stop"] = True
                state["cv"].notify_all()
            t.join()


# --------------------------------------------------------------------------- CUDA arm
def measure(args, wl, *, dev, rank, world, local, clocks, gloo_group=None):
    """Warm-up, device-resident timing, end-to-end timing, parity, roofline; the JSON line."""
    import torch.distributed as dist

    from gemma4_posttrain_jax_b200 import _lib, phase_timer

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    windows = []
    t_warm = time.time()
    for _ in range(args.warmup):
        wl.step(*wl.inputs)
    torch.cuda.synchronize()
    assert _lib.device_error(local) == 0, "device-side error during warm-up"
    barrier()
    torch.cuda.synchronize()
    free0, total_mem = torch.cuda.mem_get_info(dev)

    # ---------------------------------------------------------------- device-resident timing
    _lib.profile_enable(True)
    phase_timer.enable(True)
    launches0 = _lib.launch_count()
    torch.cuda.reset_peak_memory_stats(dev)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    step_marks = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    t_wall0 = time.time()
    start.record()
    for i in range(args.steps):
        wl.step(*wl.inputs)
        step_marks[i].record()
    stop.record()
    torch.cuda.synchronize()
    windows.append((t_wall0, time.time()))
    free1, _ = torch.cuda.mem_get_info(dev)
    barrier()
    torch.cuda.synchronize()
    launches = (_lib.launch_count() - launches0) // max(args.steps, 1)
    prof = _lib.profile_read()
    _lib.profile_enable(False)
    phases = phase_timer.read()
    phase_timer.enable(False)
    ms = max_over_ranks(start.elapsed_time(stop) / args.steps)
    value = wl.n_valid / (ms / 1e3)
    # per-step device times and device memory of this rank (the reference's harness reports
    # the mean, the p50 and the peak device bytes, bench.py:42-63)
    marks = [start, *step_marks]
    per_step = [marks[i].elapsed_time(marks[i + 1]) for i in range(args.steps)]
    step_stats = {"rank": rank, "p50_ms": float(np.median(per_step)), "min_ms": float(min(per_step)),
                  "max_ms": float(max(per_step)),
                  "torch_peak_allocated_bytes": int(torch.cuda.max_memory_allocated(dev)),
                  "device_used_bytes": int(total_mem - min(free0, free1))}
    assert _lib.device_error(local) == 0, "device-side error during the timed region"

    # ---------------------------------------------------------------- end-to-end (host buffers)
    e2e = None
    if not args.no_e2e:
        # Every step copies its inputs from pinned host memory and reads its logps back
        # (StepLoader: double-buffered on the copy engines; with N ranks each rank copies 1/N
        # of the bytes from host and pulls the rest from its peers over NVLink).
        loader = StepLoader(wl.inputs, dev=dev, rank=rank, world=world, gloo_group=gloo_group)
        out_host = torch.empty(wl.out_shape, dtype=torch.float32).pin_memory()
        d2h = out_host.nbytes
        loader.run(args.warmup, wl.step, out_host)
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t_wall0 = time.time()
        e0.record()
        loader.run(args.steps, wl.step, out_host)
        e1.record()
        torch.cuda.synchronize()
        windows.append((t_wall0, time.time()))
        barrier()
        ems = max_over_ranks(e0.elapsed_time(e1) / args.steps)
        # the bytes every slot holds after the run are the step inputs (own range from host,
        # the rest from the peers), on every rank
        same = all(torch.equal(v, x) for s in range(2) for v, x in zip(loader.views[s], wl.inputs))
        inputs_ok = max_over_ranks(0.0 if same else 1.0) == 0.0
        e2e = {"value": wl.n_valid / (ems / 1e3), "unit": "tokens/s", "ms_per_step": ems,
               "h2d_bytes_per_step": int(loader.h2d_bytes), "d2h_bytes_per_step": int(d2h),
               "h2d_bytes_per_step_all_ranks": int(loader.total if loader.sharded else loader.total * world),
               "nvlink_bytes_per_step": int(loader.peer_bytes), "inputs_ok": bool(inputs_ok),
               "loader": ("each rank copies 1/N of the step inputs from pinned host memory and pulls the rest "
                          "from its peers over NVLink" if loader.sharded else
                          "every rank copies all step inputs from pinned host memory")}
        del loader
        torch.cuda.synchronize()
        barrier()

    # ---------------------------------------------------------------- parity of one step
    parity = None
    if not args.no_parity:
        out = wl.step(*wl.inputs)
        view, extra_ok = wl.parity_view(out)
        parity = parity_check(wl.W, softcap=args.softcap if args.softcap > 0 else None, rank=rank, world=world,
                              dev=dev, **view)
        parity["masked_slots_zero"] = extra_ok
        parity["ok"] = bool(parity["ok"] and extra_ok)
        del out, view
        torch.cuda.empty_cache()
        assert _lib.device_error(local) == 0, "device-side error in the parity step"

    # ---------------------------------------------------------------- roofline of the dominant kernel
    peaks, peak_src = load_peaks()
    kernels = {}
    for name, (tot_ms, cnt) in prof.items():
        per_launch = tot_ms / max(cnt, 1)
        entry = {"launches_per_step": cnt / args.steps, "ms_per_step": tot_ms / args.steps, "ms_per_launch": per_launch}
        if name in wl.flops:
            tf = wl.flops[name] * args.steps / (tot_ms / 1e3) / 1e12
            entry["tflops"] = tf
            entry["frac_of_sustained_peak"] = tf / peaks["bf16_tflops_sustained"]
        kernels[name] = entry
    gemm_names = [k for k in kernels if k in wl.flops]
    dom = max(gemm_names, key=lambda k: kernels[k]["ms_per_step"]) if gemm_names else None
    roofline = None
    if dom is not None:
        cnt = prof[dom][1]
        flop_per_launch = wl.flops[dom] * args.steps / max(cnt, 1)
        achieved = flop_per_launch / (kernels[dom]["ms_per_launch"] / 1e3) / 1e12
        traffic, traffic_note = None, None
        if wl.traffic_ok and dom == "fwd_lse_gemm":
            traffic, traffic_note = NCU_FWD_TRAFFIC_PER_TOKEN_N1 * wl.n_valid, NCU_TRAFFIC_NOTE
        elif wl.traffic_ok and dom == "bwd_dz_gemm":
            rows_per_launch = wl.n_bwd * args.steps / max(cnt, 1)
            if rows_per_launch <= 12288:
                traffic = NCU_DZ_READ_PER_LAUNCH_N1 + NCU_DZ_WRITE_PER_ROW_N1 * rows_per_launch
                traffic_note = NCU_DZ_TRAFFIC_NOTE
        roofline = {
            "kernel": dom,
            "bound": "tensor",
            "achieved": achieved,
            "peak": peaks["bf16_tflops_sustained"],
            "unit": "TFLOP/s",
            "frac": achieved / peaks["bf16_tflops_sustained"],
            "traffic": traffic,
            "traffic_unit": "bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum)",
            "traffic_source": traffic_note,
            "peak_source": f"bf16_tflops_sustained ({peak_src}); kernel runs inside a long step",
            "flop_per_launch": flop_per_launch,
        }
    step_tflops = wl.total_flops / (ms / 1e3) / 1e12  # the GEMM work one step needs
    dense_equiv_tflops = wl.dense_flops / (ms / 1e3) / 1e12

    # ---------------------------------------------------------------- exposed collective time
    def kms(name):
        return kernels[name]["ms_per_step"] if name in kernels else 0.0

    collective = None
    if world > 1:
        dh_over = 0.0
        if "bwd_dh_gemm" in kernels and "bwd_dw_gemm" in kernels:
            # the dH GEMM's time above the rate of this run's dW GEMM (same FLOPs, same CTA-pair
            # tiling, no collective): the cost of the dH sum inside it
            dw_rate = wl.flops["bwd_dw_gemm"] / kms("bwd_dw_gemm")
            dh_over = max(0.0, kms("bwd_dh_gemm") - wl.flops["bwd_dh_gemm"] / dw_rate)
        nccl = sum(v[0] for k, v in phases.items() if k in ("stats_all_gather", "dh_all_reduce")) / args.steps
        parts = {"fwd_exchange_ms": kms("fwd_finalize_mesh"), "peer_barrier_ms": kms("peer_barrier"),
                 "nccl_ms": nccl, "dh_sum_in_gemm_ms_est": dh_over}
        total = sum(parts.values())
        # every rank's own figure: the rank that waits least is normally the slowest GPU,
        # whose time sets the step; the others' waits are slack behind it
        lo, hi = -max_over_ranks(-total), max_over_ranks(total)
        collective = {**parts, "exposed_collective_ms": total, "frac_of_step": total / ms,
                      "exposed_collective_ms_min_over_ranks": lo, "exposed_collective_ms_max_over_ranks": hi,
                      "frac_of_step_min_over_ranks": lo / ms,
                      "note": "rank 0's kernel timings; fwd_exchange includes the wait for the slowest rank's "
                              "forward GEMM; min over ranks = the least-waiting rank (normally the slowest GPU)"}

    # ---------------------------------------------------------------- CPU baseline (rank 0, N = 1)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.config == 2:
        cores = use_all_host_cores()
        Wf = wl.W.detach().float().cpu().numpy()
        Hf = wl.inputs[0].float().cpu().numpy()
        mask_np = wl.inputs[2].cpu().numpy()
        ids_np = wl.inputs[1].cpu().numpy()
        g_np = wl.inputs[3].cpu().numpy()
        sample = CPU_SAMPLE_TOKENS
        t = cpu_sample(Wf, Hf, ids_np, mask_np, g_np, sample, args.softcap)
        cpu = {"value": sample / t, "unit": "tokens/s", "cores": cores, "kind": "port",
               "sample": f"{sample} valid response tokens of this workload, fwd+bwd over V=262144, d=2048 "
               f"({t:.1f} s), numpy float32 restatement of losses.py:72-147 + recompute backward"}
        del Wf, Hf

    clock_summary = None
    if rank == 0:
        clock_summary = clocks.summary(windows, t_warm)
    line = None
    if rank == 0:
        line = {
            "metric": wl.metric,
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
            "config": wl.config,
            "clocks": clock_summary,
            "sm_mcycles_per_step": (ms * clock_summary["sm_mhz"] / 1e3) if clock_summary else None,
            "e2e": e2e,
            "gpu_launches": int(launches),
            "roofline": roofline,
            "cpu_baseline": cpu,
            "parity": parity,
            "collective": collective,
            "step_tflops": step_tflops,
            "step_frac_of_sustained_peak": step_tflops / world / peaks["bf16_tflops_sustained"],
            "dense_8Tdv_tflops": dense_equiv_tflops,
            "backward_rows": wl.n_bwd,
            "kernels": kernels,
            "host_phases_ms_per_step": {k: v[0] / args.steps for k, v in phases.items()},
            "kernel_ms_per_step": sum(v["ms_per_step"] for v in kernels.values()),
            "step_stats": step_stats,
            "cta_group": cta_group_of_run(),
        }
        print(json.dumps(line), flush=True)
    return (parity is None or parity["ok"]) and (e2e is None or e2e["inputs_ok"])


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.sampler_head:
        return run_sampler_head(args)

    import torch.distributed as dist

    from gemma4_posttrain_jax_b200 import _lib, build
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
    gloo_group = None
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
        mesh = VocabMesh(None)
        # host-only barriers of the step-input loader (its background thread)
        gloo_group = dist.new_group(backend="gloo", timeout=timedelta(seconds=120))

    softcap = args.softcap if args.softcap > 0 else None
    chunk = args.token_chunk or None
    clocks = ClockSampler(list(range(world)))
    if rank == 0:
        clocks.start()
    ok = True
    try:
        if args.config == 2:
            ok = measure(args, grpo_workload(args, dev, rank, world, mesh, softcap, chunk), dev=dev, rank=rank,
                         world=world, local=local, clocks=clocks, gloo_group=gloo_group)
        else:
            tokens = [int(t) for t in args.tokens.split(",") if t.strip()] or [DENSE_CONFIGS[args.config][0]]
            for T_cfg in tokens:
                wl = dense_workload(args, dev, rank, world, mesh, softcap, chunk, T_cfg)
                ok = measure(args, wl, dev=dev, rank=rank, world=world, local=local, clocks=clocks,
                             gloo_group=gloo_group) and ok
                del wl
                torch.cuda.empty_cache()
    finally:
        clocks.stop()
    if world > 1:
        dist.destroy_process_group()
    return 0 if ok else 3


if __name__ == "__main__":
    sys.exit(main())
