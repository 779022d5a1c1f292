"""jax.ffi binding of liblp_b200: the ``backend="cuda"`` a JAX caller of the reference uses.

This is the binding the reference's backend switch (``gemma4_posttrain_jax/losses.py:307-343``)
would import, in the same place it imports the Pallas backend (``:329-342``). It registers
the XLA FFI handlers of ``csrc/lp_xla_ffi.cc`` (typed FFI, CUDA platform) and wraps them in
a ``jax.custom_vjp`` inside ``jax.shard_map`` over the mesh axis "d", mirroring the
reference's vocab-parallel structure (``losses.py:172-260``): per-shard forward,
``all_gather`` of the (max, sum, owned target) triples + ``lp_combine``, per-shard backward
and a ``psum`` of the dH partials.

Status: JAX is not installed in the image this repository is built and tested in, so this
module and ``lp_xla_ffi.cc`` have not been compiled or run here; the torch binding
(``losses.py``) exercises the same C ABI and is what the tests and the benchmark use.
Targets outside a shard are handled by shifting them by the shard offset in JAX
(``y - axis_index * Vs``) and calling the C ABI with ``v_off = 0``: ids outside
``[0, Vs)`` are simply not owned, so no traced value has to become an FFI attribute.
"""

from __future__ import annotations

import ctypes
import math

import numpy as np

from . import _lib

_REGISTERED = False


def register() -> None:
    """Build (if needed) and register the lp_fwd / lp_combine / lp_bwd FFI targets."""
    global _REGISTERED
    if _REGISTERED:
        return
    import jax

    from .build import build_xla_ffi

    lib = ctypes.cdll.LoadLibrary(str(build_xla_ffi()))
    for target, symbol in (("lp_fwd", "LpFwd"), ("lp_combine", "LpCombine"), ("lp_bwd", "LpBwd")):
        jax.ffi.register_ffi_target(target, jax.ffi.pycapsule(getattr(lib, symbol)), platform="CUDA")
    _REGISTERED = True


def _fwd_call(w, h, y, cap):
    import jax
    import jax.numpy as jnp

    T = h.shape[0]
    ws = int(_lib.load().lp_fwd_workspace_bytes(T, w.shape[0]))
    stats, logp, _ = jax.ffi.ffi_call(
        "lp_fwd",
        (
            jax.ShapeDtypeStruct((3, T), jnp.float32),
            jax.ShapeDtypeStruct((T,), jnp.float32),
            jax.ShapeDtypeStruct((ws,), jnp.uint8),
        ),
    )(h, w, y, softcap=np.float32(cap), v_off=np.int64(0))
    return stats, logp


def _combine_call(all_stats):
    import jax
    import jax.numpy as jnp

    T = all_stats.shape[-1]
    return jax.ffi.ffi_call(
        "lp_combine",
        (jax.ShapeDtypeStruct((T,), jnp.float32), jax.ShapeDtypeStruct((2, T), jnp.float32)),
    )(all_stats)


def _bwd_call(w, h, y, norm, g, cap, token_chunk):
    import jax
    import jax.numpy as jnp

    T, d = h.shape
    ws = int(_lib.load().lp_bwd_workspace_bytes(T, d, w.shape[0], token_chunk, 0))
    dh, dw, _ = jax.ffi.ffi_call(
        "lp_bwd",
        (
            jax.ShapeDtypeStruct((T, d), jnp.bfloat16),
            jax.ShapeDtypeStruct(w.shape, jnp.float32),
            jax.ShapeDtypeStruct((ws,), jnp.uint8),
        ),
    )(h, w, y, norm, g, softcap=np.float32(cap), v_off=np.int64(0), token_chunk=np.int64(token_chunk))
    return dh, dw


def _local_logps(cap, sharded, token_chunk):
    """custom_vjp over one device's (W shard, replicated H, shifted targets)."""
    import jax
    import jax.numpy as jnp
    from jax import lax

    @jax.custom_vjp
    def f(w, h, y):
        return fwd(w, h, y)[0]

    def fwd(w, h, y):
        stats, logp = _fwd_call(w, h, y, cap)
        if sharded:
            logp, norm = _combine_call(lax.all_gather(stats, "d"))
        else:
            norm = stats[:2]
        return logp, (w, h, y, norm)

    def bwd(res, g):
        w, h, y, norm = res
        dh, dw = _bwd_call(w, h, y, norm, g.astype(jnp.float32), cap, token_chunk)
        if sharded:
            # the bf16 partials are summed in bf16, as the reference's psum of the bf16 hidden
            # cotangent (losses.py:253-259 transposed) and the torch binding's default do
            dh = lax.psum(dh.astype(h.dtype), "d")
        return dw.astype(w.dtype), dh, None

    f.defvjp(fwd, bwd)
    return f


def per_token_logps(
    embed_tokens,
    hidden,
    targets,
    *,
    softcap: float | None,
    vocab_chunk: int = 8192,
    sequence_chunk: int = 256,
    mesh=None,
    token_chunk: int = 0,
):
    """``per_token_logps`` (``losses.py:307-343``) on the B200 kernels, for JAX arrays.

    Same validation messages as the reference; bf16 embedding and hidden states. With a
    multi-device ``mesh`` the embedding is vocabulary-sharded ``P("d", None)`` and hidden /
    targets replicated, exactly as ``_vocab_parallel_logps`` expects.
    """
    import jax
    import jax.numpy as jnp
    from jax import lax
    from jax.sharding import PartitionSpec as P

    if hidden.shape[:-1] != targets.shape:
        raise ValueError(f"hidden prefix {hidden.shape[:-1]} does not match targets {targets.shape}")
    if embed_tokens.ndim != 2 or hidden.shape[-1] != embed_tokens.shape[-1]:
        raise ValueError(f"incompatible embedding {embed_tokens.shape} and hidden {hidden.shape}")
    if vocab_chunk <= 0 or sequence_chunk <= 0:
        raise ValueError("vocab_chunk and sequence_chunk must be positive")
    if softcap is not None and (not math.isfinite(softcap) or softcap <= 0):
        raise ValueError("softcap must be finite and positive, or None")
    if embed_tokens.dtype != jnp.bfloat16 or hidden.dtype != jnp.bfloat16:
        raise ValueError("the cuda logprob backend requires BF16 weights and hidden states")
    register()
    cap = 0.0 if softcap is None else float(softcap)
    out_shape = targets.shape
    h2 = hidden.reshape(-1, hidden.shape[-1])
    y = targets.reshape(-1).astype(jnp.int32)
    if mesh is None or mesh.size == 1:
        return _local_logps(cap, False, token_chunk)(embed_tokens, h2, y).reshape(out_shape)
    if "d" not in mesh.axis_names:
        raise ValueError(f"vocab-parallel mesh needs axis 'd': {mesh.axis_names}")
    if embed_tokens.shape[0] % mesh.shape["d"]:
        raise ValueError(f"vocab size {embed_tokens.shape[0]} must be divisible by mesh axis {mesh.shape['d']}")
    f = _local_logps(cap, True, token_chunk)

    def local(w, h, t):
        shifted = t - lax.axis_index("d") * w.shape[0]
        return f(w, h, shifted)

    mapped = jax.shard_map(local, mesh=mesh, in_specs=(P("d", None), P(), P()), out_specs=P(), axis_names={"d"})
    return mapped(embed_tokens, h2, y).reshape(out_shape)
