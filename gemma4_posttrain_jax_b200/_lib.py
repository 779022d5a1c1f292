"""ctypes binding of liblp_b200.so (the C ABI declared in include/lp_logprob.h).

The shared library is built in-tree (``python -m gemma4_posttrain_jax_b200.build``).
There is no fallback: if the library is missing or fails to load, every call raises
``LogprobLibraryError``.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "liblp_b200.so"

LP_OK = 0
LP_EINVAL = -1
LP_ECUDA = -2
LP_EWORKSPACE = -3
LP_EDEVICE = -4
LP_EUNSUPPORTED = -5

LP_BWD_DH_F32 = 1
LP_BWD_DW_BF16 = 2
LP_BWD_NO_DW = 4
LP_BWD_NO_DH = 8
LP_HEAD_LOGPROBS = 1

# Every symbol include/lp_logprob.h declares, with its ctypes signature.
_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_SIG = {
    "lp_version": (ctypes.c_int, []),
    "lp_last_error": (ctypes.c_char_p, []),
    "lp_launch_count": (ctypes.c_longlong, []),
    "lp_device_error": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_int)]),
    "lp_device_error_poll": (ctypes.c_int, [ctypes.c_int]),
    "lp_set_cta_group": (ctypes.c_int, [ctypes.c_int]),
    "lp_get_cta_group": (ctypes.c_int, []),
    "lp_device_pairs": (ctypes.c_int, []),
    "lp_debug_enable": (ctypes.c_int, [ctypes.c_int]),
    "lp_debug_read": (ctypes.c_int, [ctypes.POINTER(ctypes.c_ulonglong)]),
    "lp_profile_enable": (ctypes.c_int, [ctypes.c_int]),
    "lp_profile_read": (
        ctypes.c_int,
        [ctypes.c_int, ctypes.c_char_p, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_longlong),
         ctypes.POINTER(ctypes.c_int)],
    ),
    "lp_fwd_workspace_bytes": (ctypes.c_size_t, [_I64, _I64]),
    "lp_fwd": (ctypes.c_int, [_P, _P, _I64, _I64, _I64, _P, _I64, _I64, _P, ctypes.c_float, _P, _P, _P, ctypes.c_size_t]),
    "lp_fwd_noalloc": (ctypes.c_int, [_P, _P, _I64, _I64, _I64, _P, _I64, _I64, _P, ctypes.c_float, _P, _P]),
    "lp_combine": (ctypes.c_int, [_P, _P, ctypes.c_int, _I64, _P, _P]),
    "lp_fwd_sum": (
        ctypes.c_int,
        [_P, _P, _I64, _I64, _I64, _P, _I64, _I64, _P, ctypes.c_float, _P, _P, _I64, _P, _P, _P, ctypes.c_uint,
         ctypes.c_int, ctypes.c_int, ctypes.c_int, _P, _P, _P, ctypes.c_size_t],
    ),
    "lp_bwd_workspace_bytes": (ctypes.c_size_t, [_I64, _I64, _I64, _I64, ctypes.c_int]),
    "lp_bwd": (
        ctypes.c_int,
        [_P, _P, _I64, _I64, _I64, _P, _I64, _I64, _P, ctypes.c_float, _P, _P, _P, _I64, _P, ctypes.c_int, _I64, _P,
         ctypes.c_size_t],
    ),
    "lp_bwd_sum_counters": (ctypes.c_size_t, [_I64]),
    "lp_bwd_sum": (
        ctypes.c_int,
        [_P, _P, _I64, _I64, _I64, _P, _I64, _I64, _P, ctypes.c_float, _P, _P, _P, _P, _I64, _P, _P, ctypes.c_int,
         ctypes.c_int, ctypes.c_int, _P, ctypes.c_int, _I64, _P, ctypes.c_size_t],
    ),
    "lp_head_workspace_bytes": (ctypes.c_size_t, [_I64, _I64]),
    "lp_head": (
        ctypes.c_int,
        [_P, _P, _I64, _I64, _I64, _P, _I64, ctypes.c_float, _P, _I64, ctypes.c_int, _P, _P, _P, _P, ctypes.c_size_t],
    ),
    "lp_compact_workspace_bytes": (ctypes.c_size_t, [_I64, _I64]),
    "lp_compact": (
        ctypes.c_int,
        [_P, _P, _I64, _I64, _P, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P, _P, ctypes.c_size_t],
    ),
    "lp_gemm_bf16": (ctypes.c_int, [_P, _P, _I64, _I64, _I64, ctypes.c_int, _P, _I64, _I64, ctypes.c_int, _P, _I64]),
    "lp_scatter_rows": (
        ctypes.c_int, [_P, _P, _I64, _P, _I64, _I64, ctypes.c_int, _P, _I64, _I64, _I64, ctypes.c_int]
    ),
    "lp_peer_barrier": (ctypes.c_int, [_P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]),
}
EXPORTED_SYMBOLS = tuple(_SIG)


class LogprobLibraryError(RuntimeError):
    """The CUDA library is missing, failed to load, or returned an error code."""


_lib: ctypes.CDLL | None = None


def load(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Load (once) and return the library with every declared symbol typed."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise LogprobLibraryError(
            f"{p} is missing; build it with `python -m gemma4_posttrain_jax_b200.build` (nvcc, sm_100a). "
            "The cuda logprob backend has no CPU fallback."
        )
    try:
        lib = ctypes.CDLL(str(p))
    except OSError as exc:  # pragma: no cover - depends on the host
        raise LogprobLibraryError(f"cannot load {p}: {exc}") from exc
    for name, (res, args) in _SIG.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def check(rc: int, what: str) -> None:
    """Raise ``ValueError`` for argument errors and ``LogprobLibraryError`` otherwise."""
    if rc == LP_OK:
        return
    msg = (load().lp_last_error() or b"").decode(errors="replace")
    if rc == LP_EINVAL:
        raise ValueError(f"{what}: {msg}")
    raise LogprobLibraryError(f"{what} failed ({rc}): {msg}")


def device_error(device: int) -> int:
    """Read and clear the device-side error code of the library on ``device`` (syncs it)."""
    code = ctypes.c_int(0)
    check(load().lp_device_error(device, ctypes.byref(code)), "lp_device_error")
    return code.value


# Device-side error codes (lp_ptx.cuh): which bounded wait gave up.
DEVICE_ERROR_NAMES = {
    1: "DEV_TIMEOUT_PRODUCER (a GEMM's TMA producer waited too long for a free stage)",
    2: "DEV_TIMEOUT_MMA (a GEMM's MMA issuer waited too long for its operands)",
    3: "DEV_TIMEOUT_EPILOGUE (a GEMM's epilogue waited too long for its accumulator)",
    4: "DEV_TIMEOUT_DRAIN (a GEMM could not drain its loads or MMAs)",
    5: "DEV_TIMEOUT_PEER (another rank of the vocabulary mesh did not arrive in time)",
}


class DeviceTimeoutError(LogprobLibraryError):
    """A kernel of the library gave up a bounded wait; its outputs are not valid."""


def device_error_poll(device: int) -> int:
    """The device-side error code of ``device`` without a CUDA call or synchronisation
    (covers the kernels that have completed; 0 = none since the last ``device_error``)."""
    return int(load().lp_device_error_poll(int(device)))


def raise_on_device_error(device: int, where: str) -> None:
    """Raise ``DeviceTimeoutError`` if a kernel recorded a device-side error on ``device``.

    Reads the host-mapped copy of the code (no synchronisation): call it after waiting for
    the stream whose kernels it should cover. The code stays set until ``device_error``
    clears it, so every later check raises too."""
    code = device_error_poll(device)
    if code:
        raise DeviceTimeoutError(
            f"{where}: a kernel on cuda:{device} recorded device error {code}: "
            f"{DEVICE_ERROR_NAMES.get(code, 'unknown code')}; its outputs are not valid "
            "(read and clear the code with _lib.device_error before retrying)"
        )


def profile_enable(on: bool = True) -> None:
    """Start (or stop) recording per-kernel CUDA-event timings; clears earlier records."""
    check(load().lp_profile_enable(1 if on else 0), "lp_profile_enable")


def profile_read(max_tags: int = 32) -> dict[str, tuple[float, int]]:
    """{kernel name: (total device ms, launches)} of the launches recorded since enabling."""
    names = ctypes.create_string_buffer(32 * max_tags)
    ms = (ctypes.c_double * max_tags)()
    cnt = (ctypes.c_longlong * max_tags)()
    n = ctypes.c_int(0)
    check(load().lp_profile_read(max_tags, names, ms, cnt, ctypes.byref(n)), "lp_profile_read")
    raw = names.raw
    out = {}
    for k in range(n.value):
        name = raw[32 * k : 32 * k + 32].split(b"\0", 1)[0].decode()
        out[name] = (float(ms[k]), int(cnt[k]))
    return out


def set_cta_group(cg: int) -> None:
    """Force pair (2) or single-CTA (1) tensor-core GEMMs for later calls; 0 = per-GEMM default."""
    check(load().lp_set_cta_group(int(cg)), "lp_set_cta_group")


def cta_group() -> int:
    return int(load().lp_get_cta_group())


DEBUG_KINDS = ("fwd", "dz", "dh", "dw", "other")
DEBUG_FIELDS = ("prod_wait", "mma_wait_load", "mma_wait_acc", "epi_wait", "mma_cycles", "kblocks", "epi_busy", "tiles")


def debug_enable(on: bool = True) -> None:
    """Zero (and switch on / off) the GEMM pipeline counters of the current device."""
    check(load().lp_debug_enable(1 if on else 0), "lp_debug_enable")


def debug_read() -> dict[str, dict[str, int]]:
    """{gemm kind: {counter: total over CTAs}} of the counters since debug_enable."""
    out = (ctypes.c_ulonglong * 40)()
    check(load().lp_debug_read(out), "lp_debug_read")
    return {k: {f: int(out[i * 8 + j]) for j, f in enumerate(DEBUG_FIELDS)} for i, k in enumerate(DEBUG_KINDS)}


def launch_count() -> int:
    """Kernels launched by the library in this process so far."""
    return int(load().lp_launch_count())
