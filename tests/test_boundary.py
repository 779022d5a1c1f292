"""The C-ABI library without a GPU: it loads, exports every declared symbol, and rejects
bad arguments with LP_EINVAL before touching the device."""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from gemma4_posttrain_jax_b200 import _lib, build

HEADER = Path(__file__).resolve().parents[1] / "include" / "lp_logprob.h"


@pytest.fixture(scope="module")
def lib():
    if not _lib.LIB_PATH.exists():
        build.build()
    return _lib.load()


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"^LP_API [^(]*?\b(lp_\w+)\(", text, flags=re.M)


def test_header_declarations_match_binding():
    names = declared_symbols()
    assert len(names) == len(set(names)) >= 10
    assert set(names) == set(_lib.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (lp_\w+)$", out, flags=re.M))
    assert set(declared_symbols()) <= exported


def test_library_links_no_torch_or_python(lib):
    out = subprocess.run(["ldd", str(_lib.LIB_PATH)], capture_output=True, text=True).stdout
    assert "torch" not in out and "python" not in out and "libcudart" not in out


def test_version_and_error_string(lib):
    assert lib.lp_version() >= 100
    assert isinstance(lib.lp_last_error(), bytes)


def _einval(rc, lib, fragment):
    assert rc == _lib.LP_EINVAL
    assert fragment in lib.lp_last_error().decode()


def test_fwd_rejects_bad_shapes_before_device_work(lib):
    P = ctypes.c_void_p
    fake = P(16)
    rc = lib.lp_fwd(None, fake, 4, 7, 7, fake, 10, 0, fake, 0.0, fake, fake, fake, 1 << 20)
    _einval(rc, lib, "multiple of 8")
    rc = lib.lp_fwd(None, fake, 4, 8, 4, fake, 10, 0, fake, 0.0, fake, fake, fake, 1 << 20)
    _einval(rc, lib, "ldh")
    rc = lib.lp_fwd(None, None, 4, 8, 8, fake, 10, 0, fake, 0.0, fake, fake, fake, 1 << 20)
    _einval(rc, lib, "null")
    rc = lib.lp_fwd(None, fake, -1, 8, 8, fake, 10, 0, fake, 0.0, fake, fake, fake, 1 << 20)
    _einval(rc, lib, "bad sizes")


def test_bwd_requires_outputs(lib):
    P = ctypes.c_void_p
    fake = P(16)
    rc = lib.lp_bwd(None, fake, 4, 8, 8, fake, 10, 0, fake, 0.0, fake, fake, None, 8, fake, 0, 0, fake, 1 << 20)
    _einval(rc, lib, "dH")
    rc = lib.lp_bwd(None, fake, 4, 8, 8, fake, 10, 0, fake, 0.0, fake, fake, fake, 8, None, 0, 0, fake, 1 << 20)
    _einval(rc, lib, "dW")


def test_small_entry_points_validate(lib):
    P = ctypes.c_void_p
    fake = P(16)
    _einval(lib.lp_combine(None, fake, 0, 5, fake, fake), lib, "bad P")
    _einval(lib.lp_scatter_rows(None, fake, 1, fake, 4, 1, 3, fake, 1, 4, 4, 3), lib, "elem_bytes")
    _einval(lib.lp_scatter_rows(None, fake, 1, fake, 4, 1, 2, fake, 1, 4, 4, 4), lib, "out_elem_bytes")
    _einval(lib.lp_scatter_rows(None, fake, 1, fake, 4, 1, 4, fake, 1, 0, 4, 4), lib, "rows_per_group")
    _einval(lib.lp_compact(None, None, 2, 3, None, 0, 0, 0, 0, None, None, None, fake, fake, fake, fake, 1024), lib,
            "null mask")
    _einval(lib.lp_gemm_bf16(None, fake, 0, 8, 8, 0, fake, 8, 8, 0, fake, 8), lib, "sizes")
    # sampler head: logits row stride and flag checks run before any device work
    _einval(lib.lp_head(None, fake, 4, 8, 8, fake, 10, 0.0, fake, 9, 0, fake, fake, fake, fake, 1024), lib,
            "ld_logits")
    _einval(lib.lp_head(None, fake, 4, 8, 8, fake, 10, 0.0, None, 12, 1, fake, fake, fake, fake, 1024), lib,
            "LP_HEAD_LOGPROBS")
    _einval(lib.lp_head(None, fake, 4, 8, 8, fake, 10, 0.0, fake, 12, 4, fake, fake, fake, fake, 1024), lib,
            "flags")
    # mesh forward: rank / epoch / exchange checks
    _einval(lib.lp_fwd_sum(None, fake, 4, 8, 8, fake, 10, 0, fake, 0.0, fake, fake, 4, fake, fake, fake, 1, 2, 2,
                           100, fake, fake, fake, 1 << 20), lib, "rank")
    _einval(lib.lp_fwd_sum(None, fake, 4, 8, 8, fake, 10, 0, fake, 0.0, fake, fake, 4, fake, fake, fake, 0, 0, 2,
                           100, fake, fake, fake, 1 << 20), lib, "epoch")
    _einval(lib.lp_fwd_sum(None, fake, 4, 8, 8, fake, 10, 0, fake, 0.0, fake, fake, 2, fake, fake, fake, 1, 0, 2,
                           100, fake, fake, fake, 1 << 20), lib, "ld_exchange")


def test_loader_fails_loudly_when_library_missing(tmp_path):
    with pytest.raises(_lib.LogprobLibraryError, match="no CPU fallback"):
        _lib.load(tmp_path / "liblp_b200.so")


def test_plain_c_caller_links_and_gets_error_codes(lib, tmp_path):
    """A C program compiled against include/lp_logprob.h and linked to the library (what a
    cgo / JNI binding does) gets sizes and LP_EINVAL codes with messages, without a GPU."""
    src = Path(__file__).resolve().parent / "c_abi" / "abi_smoke.c"
    exe = tmp_path / "abi_smoke"
    libdir = _lib.LIB_PATH.parent
    cc = subprocess.run(
        ["gcc", "-std=c11", "-Wall", "-Werror", f"-I{HEADER.parent}", str(src), f"-L{libdir}", "-llp_b200",
         f"-Wl,-rpath,{libdir}", "-o", str(exe)],
        capture_output=True, text=True,
    )
    assert cc.returncode == 0, cc.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "c abi smoke: ok" in run.stdout
