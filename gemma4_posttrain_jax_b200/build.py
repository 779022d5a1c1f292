"""Build liblp_b200.so in-tree with nvcc for sm_100a (no JIT cache, no torch extension).

``python -m gemma4_posttrain_jax_b200.build`` compiles ``csrc/lp_capi.cu`` (which includes
the kernel headers) into ``gemma4_posttrain_jax_b200/liblp_b200.so``. The library links the
CUDA runtime statically and resolves ``cuTensorMapEncodeTiled`` from the driver at run
time, so it has no dependency on torch, Python or libcuda at link time.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
LIB_PATH = PKG_DIR / "liblp_b200.so"
SOURCES = [CSRC / "lp_capi.cu"]
HEADERS = sorted(CSRC.glob("*.cuh")) + [PKG_DIR.parent / "include" / "lp_logprob.h"]

NVCC_FLAGS = [
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden",
    "-shared",
    "-cudart",
    "static",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the B200 logprob library must be built with CUDA 12.8+")


def needs_rebuild() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    return any(p.stat().st_mtime > built for p in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    """Compile the library if any source is newer than it; returns the .so path."""
    if not force and not needs_rebuild():
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc_path(), *NVCC_FLAGS, *(extra_flags or []), "-o", str(tmp), *map(str, SOURCES)]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout, res.stderr, file=sys.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


XLA_FFI_SOURCE = CSRC / "lp_xla_ffi.cc"
XLA_FFI_LIB = PKG_DIR / "liblp_b200_xla.so"


def build_xla_ffi(force: bool = False) -> Path:
    """Compile the XLA FFI handlers against jaxlib's headers (needs an installed ``jax``)."""
    import jax.ffi  # noqa: PLC0415 - only where JAX exists

    lib = build()
    if not force and XLA_FFI_LIB.exists() and XLA_FFI_LIB.stat().st_mtime > max(
        XLA_FFI_SOURCE.stat().st_mtime, lib.stat().st_mtime
    ):
        return XLA_FFI_LIB
    cmd = [
        os.environ.get("CXX", "g++"), "-std=c++17", "-O2", "-shared", "-fPIC",
        f"-I{jax.ffi.include_dir()}", "-I/usr/local/cuda/include", str(XLA_FFI_SOURCE),
        f"-L{PKG_DIR}", "-llp_b200", "-Wl,-rpath,$ORIGIN", "-o", str(XLA_FFI_LIB),
    ]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"building the XLA FFI handlers failed:\n{res.stdout}\n{res.stderr}")
    return XLA_FFI_LIB


if __name__ == "__main__":
    flags = [a for a in sys.argv[1:] if a.startswith("-X") or a.startswith("--")]
    print(build(force=True, verbose=True, extra_flags=flags))
