"""The library's launch planning (lp_plan.cuh: backward token chunks, split-K choices, the
forward's vocabulary groups and their widening for the fixed-scratch forward), compiled with
nvcc as a host program and run on the CPU."""

from __future__ import annotations

import os
import subprocess
from pathlib import Path

import pytest

from gemma4_posttrain_jax_b200 import build

SRC = Path(__file__).resolve().parent / "sched" / "plan_check.cu"


def test_launch_plans(tmp_path):
    try:
        nvcc = build.nvcc_path()
    except RuntimeError:
        pytest.skip("nvcc not available")
    exe = tmp_path / "plan_check"
    cc = subprocess.run([nvcc, "-std=c++17", "--expt-relaxed-constexpr", "-gencode", "arch=compute_100a,code=sm_100a",
                         "-o", str(exe), str(SRC)], capture_output=True, text=True)
    assert cc.returncode == 0, cc.stderr[-3000:]
    env = {k: v for k, v in os.environ.items() if not k.startswith("LP_B200_")}  # the default plans
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120, env=env)
    assert run.returncode == 0, run.stdout[-3000:]
    assert "plan: ok" in run.stdout
