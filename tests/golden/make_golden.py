"""Regenerate ``tests/golden/logprob_golden.npz`` (run from the repository root).

The reference (yixiaoer/gemma4-posttrain-jax) is JAX-only and cannot run in this image, so
these vectors come from the numpy oracle (``oracle/logprob_oracle.py``, float64 analytic
path) evaluated on the reference tests' own seeded inputs:

* ``losses_*``   shapes / scales / targets of ``tests/test_losses.py:25-28`` (the reference
                 draws them with ``jax.random.key(17)``, which numpy cannot reproduce; the
                 same shapes are drawn with ``np.random.default_rng(17)`` instead);
* ``stats_*``    ``tests/test_native_logprob_stats.py:22-32`` (``default_rng(20260925)``,
                 reproduced bit-for-bit);
* ``shard_*``    ``tests/test_sharding_tpu.py:51-61`` (``default_rng(7)`` with the planted
                 per-shard maxima, reproduced bit-for-bit).

The fixtures pin the oracle against regressions; the oracle itself is pinned by the
relations the reference tests assert (see ``tests/test_oracle.py``).
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import logprob_oracle as orc  # noqa: E402

OUT = Path(__file__).resolve().parent / "logprob_golden.npz"


def losses_inputs():
    rng = np.random.default_rng(17)
    embed = (rng.normal(size=(23, 7)) * 0.4).astype(np.float32)
    hidden = (rng.normal(size=(2, 5, 7)) * 0.7).astype(np.float32)
    targets = np.asarray([[0, 4, 22, 8, 2], [11, 3, 19, 1, 7]], np.int32)
    return embed, hidden, targets


def stats_inputs(scale: float):
    rng = np.random.default_rng(20260925)
    w = orc.bf16_round(rng.normal(size=(1036, 128)) * scale)
    h = orc.bf16_round(rng.normal(size=(513, 128)))
    token = np.resize(np.array([0, 258, 259, 517, 518, 776, 777, 1035], np.int32), 513)
    gradient = rng.normal(size=513).astype(np.float32)
    gradient[256:512] = 0
    return w, h, token, gradient


def shard_inputs():
    rng = np.random.default_rng(7)
    embed = rng.normal(0.0, 0.2, (96, 8)).astype(np.float32)
    hidden = rng.normal(0.0, 0.3, (4, 5, 8)).astype(np.float32)
    for shard, row in enumerate((3, 27, 51, 75)):
        embed[row, shard] = 30.0 + 10.0 * shard
        hidden[shard, :, shard] = 1.0
    targets = np.asarray(
        [[0, 23, 24, 47, 48], [71, 72, 95, 3, 27], [51, 75, 12, 36, 60], [84, 8, 32, 56, 80]], np.int32
    )
    weights = np.linspace(0.5, 1.5, targets.size, dtype=np.float32).reshape(targets.shape)
    return embed, hidden, targets, weights


def main() -> None:
    out: dict[str, np.ndarray] = {}
    e, h, t = losses_inputs()
    for name, cap in (("none", None), ("cap3", 3.0)):
        lp, dE, dH = orc.logps_grads_f64(e, h, t, np.ones(t.shape), cap)
        out[f"losses_{name}_logps"] = lp
        out[f"losses_{name}_dE"] = dE
        out[f"losses_{name}_dH"] = dH
    for scale in (0.04, 1.5):
        w, hh, tok, g = stats_inputs(scale)
        for name, cap in (("none", None), ("cap30", 30.0)):
            key = f"stats_s{scale}_{name}"
            lp, dW, dHs = orc.logps_grads_f64(w, hh, tok, g, cap)
            out[f"{key}_logps"] = lp
            out[f"{key}_norm"] = orc.dense_normalization(w, hh, cap)
            # gradients are large; keep per-row norms and a few full rows
            out[f"{key}_dW_rownorm"] = np.linalg.norm(dW, axis=1)
            out[f"{key}_dH_rownorm"] = np.linalg.norm(dHs, axis=1)
            out[f"{key}_dW_rows"] = dW[[0, 258, 259, 517, 518, 776, 777, 1035]]
            out[f"{key}_dH_rows"] = dHs[[0, 1, 255, 256, 511, 512]]
    e, h, t, wts = shard_inputs()
    lp, dE, dH = orc.logps_grads_f64(e, h, t, wts, 30.0)
    out["shard_logps"] = lp
    out["shard_dE"] = dE
    out["shard_dH"] = dH
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    main()
