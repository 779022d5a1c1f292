"""Optional CUDA-event timing of the host-side phases of the logprob path.

Kernels of liblp_b200 are timed inside the library (lp_profile_*); this module times what
happens between them on the host side — NCCL collectives, dtype casts, zero fills — by
recording CUDA events on the current stream around each phase. Disabled by default; a
disabled timer records nothing and costs one branch per phase.
"""

from __future__ import annotations

import contextlib
from collections import defaultdict

import torch

_enabled = False
_records: list[tuple[str, torch.cuda.Event, torch.cuda.Event]] = []


def enable(on: bool = True) -> None:
    """Start (or stop) recording; clears earlier records."""
    global _enabled
    _enabled = on
    _records.clear()


@contextlib.contextmanager
def phase(name: str):
    if not _enabled:
        yield
        return
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    start.record()
    try:
        yield
    finally:
        stop.record()
        _records.append((name, start, stop))


def read() -> dict[str, tuple[float, int]]:
    """{phase: (total ms, count)} of the recorded phases (synchronises on the events)."""
    out: dict[str, list] = defaultdict(lambda: [0.0, 0])
    for name, start, stop in _records:
        stop.synchronize()
        out[name][0] += start.elapsed_time(stop)
        out[name][1] += 1
    return {k: (v[0], v[1]) for k, v in out.items()}
