"""Host-side behaviour of the Python mirror, no GPU needed: argument validation (same
messages as the reference), no silent fallback, checkpoint identity (mirrors
``tests/test_logprob_backends.py`` of the reference)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from gemma4_posttrain_jax_b200 import logprob_protocol as proto
from gemma4_posttrain_jax_b200 import ops
from gemma4_posttrain_jax_b200.losses import completion_logps, per_token_logps, sft_token_logps


def test_shape_mismatch_message_matches_reference():
    with pytest.raises(ValueError, match="does not match"):
        per_token_logps(torch.ones((7, 3)), torch.ones((2, 4, 3)), torch.ones((2, 3), dtype=torch.int32), softcap=None)


def test_incompatible_embedding_and_chunk_checks():
    with pytest.raises(ValueError, match="incompatible embedding"):
        per_token_logps(torch.ones((7, 3)), torch.ones((2, 4)), torch.ones((2,), dtype=torch.int32), softcap=None)
    with pytest.raises(ValueError, match="must be positive"):
        per_token_logps(torch.ones((7, 3)), torch.ones((2, 3)), torch.ones((2,), dtype=torch.int32), softcap=None,
                        vocab_chunk=0)
    with pytest.raises(ValueError, match="softcap must be finite"):
        per_token_logps(torch.ones((7, 3)), torch.ones((2, 3)), torch.ones((2,), dtype=torch.int32), softcap=-1.0)


@pytest.mark.parametrize("backend,message", [("unknown", "unknown logprob"), ("jax", "backend='cuda'"),
                                             ("pallas", "backend='cuda'")])
def test_invalid_backend_never_silently_falls_back(backend, message):
    w = torch.ones((8, 8), dtype=torch.bfloat16)
    h = torch.ones((2, 8), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match=message):
        per_token_logps(w, h, torch.zeros((2,), dtype=torch.int32), softcap=30.0, backend=backend)


def test_cpu_tensors_are_refused_not_computed():
    w = torch.ones((8, 8), dtype=torch.bfloat16)
    h = torch.ones((2, 8), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="no CPU fallback"):
        per_token_logps(w, h, torch.zeros((2,), dtype=torch.int32), softcap=30.0)
    with pytest.raises(ValueError, match="no CPU fallback"):
        ops.shard_forward(w, h, torch.zeros((2,), dtype=torch.int32), None)
    with pytest.raises(ValueError, match="no CPU fallback"):
        ops.compact(torch.ones((2, 3), dtype=torch.bool))


def test_caller_shape_checks():
    with pytest.raises(ValueError, match="prompt_width"):
        completion_logps(torch.ones((8, 8)), torch.ones((2, 4, 8)), torch.zeros((2, 4), dtype=torch.int32),
                         torch.ones((2, 4), dtype=torch.bool), prompt_width=2, softcap=None)
    with pytest.raises(ValueError, match="at least two tokens"):
        sft_token_logps(torch.ones((8, 8)), torch.ones((2, 1, 8)), torch.zeros((2, 1), dtype=torch.int64), softcap=None)


def test_legacy_checkpoint_keeps_native_backend():
    saved = {"mode": "gsm8k", "seed": 7}
    proto.validate_logprob_resume(saved, {**saved, "logprob_backend": "jax"})
    with pytest.raises(ValueError, match="logprob_backend"):
        proto.validate_logprob_resume(saved, {**saved, **proto.logprob_run_metadata("cuda")})


def test_cuda_checkpoint_identity_and_changes_refused():
    meta = proto.logprob_run_metadata("cuda")
    assert meta == {"logprob_backend": "cuda", "logprob_protocol": proto.CUDA_LOGPROB_PROTOCOL}
    saved = {"mode": "overfit", **meta}
    proto.validate_logprob_resume(saved, dict(saved))
    with pytest.raises(ValueError, match="logprob_backend"):
        proto.validate_logprob_resume(saved, {**saved, **proto.logprob_run_metadata("pallas")})
    with pytest.raises(ValueError, match="logprob_protocol"):
        proto.validate_logprob_resume({**saved, "logprob_protocol": "older"}, saved)


def test_native_metadata_is_empty_and_unknown_rejected():
    assert proto.logprob_run_metadata("jax") == {}
    assert proto.logprob_run_metadata("pallas")["logprob_protocol"] == proto.PALLAS_LOGPROB_PROTOCOL
    with pytest.raises(ValueError, match="unknown logprob"):
        proto.logprob_run_metadata("unknown")


def test_dh_reduce_mode_single_shard_and_override(monkeypatch):
    from gemma4_posttrain_jax_b200 import sharding

    assert sharding.dh_reduce_mode(None) == "none"
    assert sharding.dh_reduce_mode(sharding.make_mesh()) == "none"  # no process group: one shard
    assert sharding.stats_exchange_mode(None) == "none"
    assert sharding.stats_exchange_mode(sharding.make_mesh()) == "none"
    monkeypatch.setenv("LP_B200_PEER_TIMEOUT_MS", "250")
    assert sharding.peer_timeout_ms() == 250
    monkeypatch.setenv("LP_B200_PEER_TIMEOUT_MS", "0")
    assert sharding.peer_timeout_ms() == 1


def test_stats_exchange_alternates_buffers_and_counts_epochs():
    """lp_fwd_sum's bookkeeping: calls alternate between the two exchange buffers (so a rank
    never overwrites a slot a peer may still read), and call k of a buffer waits for k * world
    on a counter that is never reset."""
    from gemma4_posttrain_jax_b200.sharding import StatsExchange

    x = object.__new__(StatsExchange)  # the bookkeeping only; no symmetric memory on CPU
    x.slot_bytes, x.base, x.base_mc, x.calls = 1 << 20, 0x10000000, 0x70000000, 0
    calls = [x.next_call() for _ in range(5)]
    xch = [c[0] for c in calls]
    assert xch == [x.base, x.base + x.slot_bytes] * 2 + [x.base]
    assert [c[1] - c[0] for c in calls] == [x.base_mc - x.base] * 5  # multicast twin of each buffer
    assert [c[5] for c in calls] == [1, 1, 2, 2, 3]  # epoch per buffer
    counters = {c[2] for c in calls}
    assert len(counters) == 2 and all(c >= x.base + 2 * x.slot_bytes for c in counters)
    assert len({c[4] for c in calls}) == 1  # one local arrival counter


def test_mesh_forward_routes_to_the_nvlink_exchange_or_the_all_gather(monkeypatch):
    """With a multicast exchange buffer the forward of a vocabulary mesh is one lp_fwd_sum
    call; without one it is lp_fwd + all-gather + lp_combine (the fallback never computes on
    the host: the device calls are stubbed here and only the routing is checked)."""
    import torch

    from gemma4_posttrain_jax_b200 import losses

    calls = []
    H, y = torch.zeros(5, 8), torch.zeros(5, dtype=torch.int32)
    W = torch.zeros(6, 8)
    mesh = object()
    logp, norm = torch.full((5,), -1.0), torch.ones(2, 5)

    def fwd_sum(embed, hidden, targets, softcap, xch, *, vocab_offset, timeout_ms):
        calls.append(("lp_fwd_sum", xch, vocab_offset, timeout_ms))
        return logp, norm

    def shard_forward(embed, hidden, targets, softcap, *, vocab_offset=0, want_logp=True):
        calls.append(("lp_fwd", vocab_offset, want_logp))
        return torch.zeros(3, 5), None

    def gather(stats, m):
        calls.append(("all_gather", m))
        return torch.stack([stats, stats])

    def combine(gathered):
        calls.append(("lp_combine", tuple(gathered.shape)))
        return logp, norm

    monkeypatch.setattr(losses.ops, "shard_forward_sum", fwd_sum)
    monkeypatch.setattr(losses.ops, "shard_forward", shard_forward)
    monkeypatch.setattr(losses.ops, "combine", combine)
    monkeypatch.setattr(losses, "all_gather_stats", gather)
    monkeypatch.setenv("LP_B200_PEER_TIMEOUT_MS", "1234")
    monkeypatch.setattr(losses, "stats_exchange", lambda m, rows, dev: "xch")
    # after the exchange the call waits for its stream and raises on a recorded peer timeout
    monkeypatch.setattr(losses, "_check_mesh_call", lambda dev, m, where: calls.append(("check", where.split()[0])))
    assert losses._mesh_forward(W, H, y, 30.0, mesh, 6) == (logp, norm)
    assert calls == [("lp_fwd_sum", "xch", 6, 1234), ("check", "lp_fwd_sum")]
    calls.clear()
    monkeypatch.setattr(losses, "stats_exchange", lambda m, rows, dev: None)
    assert losses._mesh_forward(W, H, y, 30.0, mesh, 6) == (logp, norm)
    assert calls == [("lp_fwd", 6, False), ("all_gather", mesh), ("lp_combine", (2, 3, 5))]


def test_mesh_backward_routes_the_dh_sum(monkeypatch):
    """The backward of a vocabulary mesh: with a multicast dH buffer, the fused lp_bwd_sum
    backward, the counters zeroed again for the next call, one peer barrier (dH shared with
    the buffer) and the host-side check for a peer timeout;
    without one, the plain backward and an all-reduce of dH. Device calls are stubbed; only
    the routing and its order are checked."""
    import torch

    from gemma4_posttrain_jax_b200 import losses

    calls = []
    T, d, Vs = 6, 8, 10
    H, y, g = torch.zeros(T, d), torch.zeros(T, dtype=torch.int32), torch.ones(T)
    W, norm = torch.zeros(Vs, d), torch.ones(2, T)

    class FakeMesh:
        size = 2

    class FakeBuf:
        counters = torch.full((16,), 7, dtype=torch.int32)

    def shard_backward(embed, Hz, yz, softcap, nz, gz, *, vocab_offset, need_dh, need_dw, dh_dtype, dw_dtype,
                       token_chunk, dh_mesh_sum=None):
        calls.append(("lp_bwd_sum" if dh_mesh_sum is not None else "lp_bwd", vocab_offset, dh_dtype))
        return torch.zeros(T, d, dtype=dh_dtype), torch.zeros(Vs, d)

    monkeypatch.setattr(losses.ops, "shard_backward", shard_backward)
    monkeypatch.setattr(losses.ops, "bwd_sum_counters", lambda rows: 4)
    monkeypatch.setattr(losses.ops, "peer_barrier", lambda buf, t: calls.append(("barrier", t)))
    monkeypatch.setattr(losses, "all_reduce_sum", lambda t, m: calls.append(("all_reduce", t.dtype, tuple(t.shape))) or t)
    monkeypatch.setattr(losses, "_check_mesh_call", lambda dev, m, where: calls.append(("check", where.split()[0])))
    monkeypatch.setenv("LP_B200_PEER_TIMEOUT_MS", "777")
    kw = dict(mesh=FakeMesh(), vocab_offset=10, need_dh=True, need_dw=True, dh_dtype=torch.bfloat16,
              dw_dtype=torch.float32, token_chunk=None, skip_zero_grad=False)

    buf = FakeBuf()
    monkeypatch.setattr(losses, "dh_sum_buffer", lambda m, rows, dd, dev: buf)
    dH, dW, pos, shared = losses._backward_rows(W, H, y, 30.0, norm, g, **kw)
    assert shared and pos is None
    # ... and the host waits for the stream, raising on a recorded peer timeout
    assert calls == [("lp_bwd_sum", 10, torch.bfloat16), ("barrier", 777), ("check", "lp_bwd_sum")]
    assert buf.counters[:4].eq(0).all() and buf.counters[4:].eq(7).all()  # the used counters are zeroed

    calls.clear()
    monkeypatch.setattr(losses, "dh_sum_buffer", lambda m, rows, dd, dev: None)
    dH, dW, pos, shared = losses._backward_rows(W, H, y, 30.0, norm, g, **kw)
    assert not shared
    # the only collective over tensor data is the [T, d] dH sum: the vocabulary-sharded
    # embedding (and its gradient) never leaves its rank, as the reference asserts of its
    # compiled program (tests/test_sharding_tpu.py:97-101)
    assert calls == [("lp_bwd", 10, torch.bfloat16), ("all_reduce", torch.bfloat16, (T, d))]


@pytest.mark.parametrize(
    "temperature,top_k,top_p",
    [(1.0, 0, 1.0), (0.7, 0, 1.0), (0.8, 3, 1.0), (0.8, 0, 0.85), (0.8, 4, 0.7), (0.8, 0, 1e-50)],
)
def test_sampling_logic_matches_transformers_warpers_on_cpu(monkeypatch, temperature, top_k, top_p):
    """sample_token's temperature / top-k / top-p / draw on top of the head, with the head
    (lp_head) stubbed by exact logits so the logic runs on the CPU: frequencies match
    transformers' warpers (the reference's test, tests/test_sampler.py:175-205) and the
    recorded logp is the untempered log-softmax."""
    import torch
    from transformers.generation.logits_process import TemperatureLogitsWarper, TopKLogitsWarper, TopPLogitsWarper

    from gemma4_posttrain_jax_b200 import sampler

    logits = torch.tensor([1.1, -0.7, 0.3, 2.0, -2.0])
    count = 20000

    def head(embed, hidden, softcap, *, want_logits=True, log_probs=False):
        z = logits.expand(hidden.shape[0], -1).clone()
        m = z.max(dim=-1).values
        norm = torch.stack([m, torch.exp(z - m[:, None]).sum(dim=-1)])
        top = z.argmax(dim=-1).to(torch.int32)
        return z, norm, top, z.max(dim=-1).values - (m + torch.log(norm[1]))

    monkeypatch.setattr(sampler.ops, "head", head)
    gen = torch.Generator().manual_seed(7)
    tok, logp = sampler.sample_token(torch.zeros(5, 8), torch.zeros(count, 8), None, temperature=temperature,
                                     top_k=top_k, top_p=top_p, generator=gen)
    scores = TemperatureLogitsWarper(temperature)(None, logits[None])
    if top_k:
        scores = TopKLogitsWarper(top_k)(None, scores)
    if top_p < 1:
        scores = TopPLogitsWarper(top_p)(None, scores)
    expected = torch.softmax(scores, dim=-1)[0].numpy()
    t = tok.numpy()
    assert (expected[t] > 0).all()
    np.testing.assert_allclose(np.bincount(t, minlength=5) / count, expected, atol=0.02)
    np.testing.assert_allclose(logp.numpy(), torch.log_softmax(logits, -1).numpy()[t], atol=1e-6)
