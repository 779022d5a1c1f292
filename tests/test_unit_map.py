"""The GEMM work-unit map (lpk::get_unit, host-callable) covers every tile and K block
exactly once in each unit order, and the cross-rank dH sum's reduce items follow all tiles
of their row block. Compiled with nvcc as a host program and run on the CPU."""

from __future__ import annotations

import subprocess
from pathlib import Path

import pytest

from gemma4_posttrain_jax_b200 import build

SRC = Path(__file__).resolve().parent / "sched" / "unit_map_check.cu"


def test_unit_map_covers_every_tile_once(tmp_path):
    try:
        nvcc = build.nvcc_path()
    except RuntimeError:
        pytest.skip("nvcc not available")
    exe = tmp_path / "unit_map_check"
    cc = subprocess.run([nvcc, "-std=c++17", "--expt-relaxed-constexpr", "-gencode", "arch=compute_100a,code=sm_100a",
                         "-o", str(exe), str(SRC)], capture_output=True, text=True)
    assert cc.returncode == 0, cc.stderr[-3000:]
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout[-3000:]
    assert "unit map: ok" in run.stdout
