"""CUDA path vs the CPU oracle, through the C ABI (via the torch-facing wrappers).

Inputs follow the reference tests' own seeded generators
(``tests/test_native_logprob_stats.py:22-32``, ``tests/test_pallas_logprob_tpuv4.py:37-51``,
``tests/test_sharding_tpu.py:51-61``). Tolerances: the north-star bars (per-token logp
within 2e-3 absolute; dH and dW within 1e-2 relative L2 against the f64-accumulated
oracle), with tighter diagnostics printed.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import logprob_oracle as orc

pytestmark = pytest.mark.gpu

LOGP_ATOL = 2e-3
GRAD_REL_L2 = 1e-2


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / den) if den else float(np.linalg.norm(a - b))


def to_bf16(x: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(orc.bf16_round(x)).to(dev).to(torch.bfloat16)


@pytest.fixture(params=[0, 2, 1], ids=["default", "pair", "single"])
def cta_group(request, cuda_device):
    """Run a test with the per-GEMM default, all-pair and all-single tensor-core GEMMs."""
    from gemma4_posttrain_jax_b200 import _lib

    before = _lib.cta_group()
    _lib.set_cta_group(request.param)
    yield request.param
    _lib.set_cta_group(before)


def _stats_case(scale, seed=20260925, V=1036, T=513, d=128):
    rng = np.random.default_rng(seed)
    w = orc.bf16_round(rng.normal(size=(V, d)) * scale)
    h = orc.bf16_round(rng.normal(size=(T, d)))
    y = np.resize(np.array([0, 258, 259, 517, 518, 776, 777, 1035], np.int32), T)
    g = rng.normal(size=T).astype(np.float32)
    g[256:512] = 0
    return w, h, y, g


# --------------------------------------------------------------------------- GEMM core
@pytest.mark.parametrize("a_mn,b_mn", [(0, 0), (0, 1), (1, 1), (1, 0)])
@pytest.mark.parametrize("M,N,K", [(200, 300, 160), (128, 256, 64), (513, 1036, 136)])
def test_gemm_core_matches_f32(cuda_device, cta_group, a_mn, b_mn, M, N, K):
    import ctypes

    from gemma4_posttrain_jax_b200 import _lib
    from gemma4_posttrain_jax_b200.ops import _ptr, _stream

    N4 = (N + 3) // 4 * 4
    rng = np.random.default_rng(M * 7 + N * 3 + K)
    a = orc.bf16_round(rng.normal(size=(M, K)))
    b = orc.bf16_round(rng.normal(size=(N4, K)))
    ta = torch.from_numpy(a.T.copy() if a_mn else a).to(cuda_device).to(torch.bfloat16)
    tb = torch.from_numpy(b.T.copy() if b_mn else b).to(cuda_device).to(torch.bfloat16)
    # pad leading dims to multiples of 8 elements (16-byte rows)
    def pad_cols(t):
        c = t.shape[1]
        c8 = (c + 7) // 8 * 8
        if c8 == c:
            return t
        out = torch.zeros((t.shape[0], c8), dtype=t.dtype, device=t.device)
        out[:, :c] = t
        return out

    ta, tb = pad_cols(ta), pad_cols(tb)
    D = torch.full((M, N4), float("nan"), dtype=torch.float32, device=cuda_device)
    lib = _lib.load()
    rc = lib.lp_gemm_bf16(
        _stream(cuda_device), _ptr(ta), M, K, ta.stride(0), a_mn, _ptr(tb), N4, tb.stride(0), b_mn, _ptr(D), D.stride(0)
    )
    _lib.check(rc, "lp_gemm_bf16")
    torch.cuda.synchronize()
    assert _lib.device_error(0) == 0
    ref = a.astype(np.float64) @ b.astype(np.float64).T
    got = D.cpu().numpy()
    assert np.isfinite(got).all()
    err = np.abs(got - ref).max() / max(1.0, np.abs(ref).max())
    print(f"gemm cg={cta_group} a_mn={a_mn} b_mn={b_mn} M={M} N={N4} K={K}: max rel err {err:.2e}")
    assert err < 1e-5


# --------------------------------------------------------------------------- forward
@pytest.mark.parametrize("softcap", [None, 30.0])
@pytest.mark.parametrize("scale", [0.04, 1.5])
def test_forward_stats_and_logps(cuda_device, cta_group, softcap, scale):
    from gemma4_posttrain_jax_b200 import ops

    w, h, y, _ = _stats_case(scale)
    stats, logp = ops.shard_forward(to_bf16(w, cuda_device), to_bf16(h, cuda_device),
                                    torch.from_numpy(y).to(cuda_device), softcap)
    torch.cuda.synchronize()
    ref = orc.single_partition_logps(w, h, y, softcap=softcap, vocab_chunk=128, sequence_chunk=256)
    dense = orc.dense_normalization(w, h, softcap)
    got = logp.cpu().numpy()
    st = stats.cpu().numpy()
    print(f"softcap={softcap} scale={scale}: logp max abs err {np.abs(got - ref).max():.2e}")
    assert np.abs(got - ref).max() <= LOGP_ATOL
    np.testing.assert_allclose(st[0], dense[0], atol=2e-4, rtol=2e-5)
    np.testing.assert_allclose(st[1], dense[1], rtol=1e-4)
    assert np.isfinite(st).all() and (st[1] > 0).all()


def test_forward_tails_repeated_targets_3d(cuda_device):
    """Pallas test shapes: W[1036,160], H[3,171,160] (token, vocab and hidden tails)."""
    from gemma4_posttrain_jax_b200.losses import per_token_logps

    rng = np.random.default_rng(20260925)
    w = orc.bf16_round(rng.normal(size=(1036, 160)) * 1.5)
    h = orc.bf16_round(rng.normal(size=(3, 171, 160)))
    t = np.resize(np.array([0, 258, 259, 517, 518, 776, 777, 1035], np.int32), 513).reshape(3, 171)
    for softcap in (None, 30.0):
        got = per_token_logps(to_bf16(w, cuda_device), to_bf16(h, cuda_device), torch.from_numpy(t).to(cuda_device),
                              softcap=softcap).cpu().numpy()
        ref = orc.dense_logps(w, h, t, softcap)
        assert got.shape == (3, 171)
        assert np.abs(got - ref).max() <= LOGP_ATOL


# --------------------------------------------------------------------------- backward
@pytest.mark.parametrize("softcap", [None, 30.0])
@pytest.mark.parametrize("scale", [0.04, 1.5])
def test_backward_matches_analytic_vjp(cuda_device, cta_group, softcap, scale):
    from gemma4_posttrain_jax_b200 import ops

    w, h, y, g = _stats_case(scale)
    W, H = to_bf16(w, cuda_device), to_bf16(h, cuda_device)
    Y = torch.from_numpy(y).to(cuda_device)
    stats, _ = ops.shard_forward(W, H, Y, softcap)
    dH, dW = ops.shard_backward(W, H, Y, softcap, stats[:2], torch.from_numpy(g).to(cuda_device),
                                dh_dtype=torch.float32, dw_dtype=torch.float32)
    torch.cuda.synchronize()
    _, dW_ref, dH_ref = orc.logps_grads_f64(w, h, y, g, softcap)
    eh, ew = rel_l2(dH.cpu().numpy(), dH_ref), rel_l2(dW.cpu().numpy(), dW_ref)
    print(f"softcap={softcap} scale={scale}: dH rel-L2 {eh:.2e}, dW rel-L2 {ew:.2e}")
    assert eh <= GRAD_REL_L2 and ew <= GRAD_REL_L2
    # rows whose upstream gradient is zero get an exactly zero dH
    assert (dH[256:512] == 0).all()


@pytest.mark.parametrize("token_chunk", [128, 256, None])
def test_backward_token_chunks_and_bf16_outputs(cuda_device, cta_group, token_chunk):
    from gemma4_posttrain_jax_b200 import ops

    w, h, y, g = _stats_case(0.04)
    W, H = to_bf16(w, cuda_device), to_bf16(h, cuda_device)
    Y = torch.from_numpy(y).to(cuda_device)
    G = torch.from_numpy(g).to(cuda_device)
    stats, _ = ops.shard_forward(W, H, Y, 30.0)
    dH32, dW32 = ops.shard_backward(W, H, Y, 30.0, stats[:2], G, dh_dtype=torch.float32, dw_dtype=torch.float32)
    dH16, dW16 = ops.shard_backward(W, H, Y, 30.0, stats[:2], G, dh_dtype=torch.bfloat16, dw_dtype=torch.bfloat16,
                                    token_chunk=token_chunk)
    dHc, dWc = ops.shard_backward(W, H, Y, 30.0, stats[:2], G, dh_dtype=torch.float32, dw_dtype=torch.float32,
                                  token_chunk=token_chunk)
    torch.cuda.synchronize()
    assert rel_l2(dH16.float().cpu(), dH32.cpu()) < 5e-3
    assert rel_l2(dW16.float().cpu(), dW32.cpu()) < 5e-3
    # chunking changes only the f32 summation order of dW
    assert rel_l2(dWc.cpu(), dW32.cpu()) < 1e-5
    # ... and the split-K plan (summation order) of dH
    assert rel_l2(dHc.cpu(), dH32.cpu()) < 1e-5


def test_frozen_head_skips_dw(cuda_device):
    from gemma4_posttrain_jax_b200 import ops

    w, h, y, g = _stats_case(0.04)
    W, H = to_bf16(w, cuda_device), to_bf16(h, cuda_device)
    Y = torch.from_numpy(y).to(cuda_device)
    stats, _ = ops.shard_forward(W, H, Y, None)
    dH, dW = ops.shard_backward(W, H, Y, None, stats[:2], torch.from_numpy(g).to(cuda_device), need_dw=False,
                                dh_dtype=torch.float32)
    assert dW is None
    _, _, dH_ref = orc.logps_grads_f64(w, h, y, g, None)
    assert rel_l2(dH.cpu().numpy(), dH_ref) <= GRAD_REL_L2


# --------------------------------------------------------------------------- vocab parallel
@pytest.mark.parametrize("shards", [2, 4])
def test_vocab_parallel_shards_on_one_gpu(cuda_device, cta_group, shards):
    """Each shard through lp_fwd / lp_bwd, merged by lp_combine, equals the unsharded result.

    Planted per-shard maxima as in ``tests/test_sharding_tpu.py:51-61`` (seed 7), scaled to
    a vocabulary the 4 shards split evenly.
    """
    from gemma4_posttrain_jax_b200 import ops

    rng = np.random.default_rng(7)
    V, d = 1024, 64
    w = rng.normal(0.0, 0.2, (V, d)).astype(np.float32)
    h = rng.normal(0.0, 0.3, (4, 37, d)).astype(np.float32)
    vs = V // 4
    for shard in range(4):
        w[shard * vs + 3 + 8 * shard, shard] = 30.0 + 10.0 * shard
        h[shard, :, shard] = 1.0
    w, h = orc.bf16_round(w), orc.bf16_round(h)
    t = rng.integers(0, V, size=(4, 37)).astype(np.int32)
    t[0, :4] = [0, vs - 1, vs, V - 1]
    g = np.linspace(0.5, 1.5, t.size, dtype=np.float32)
    W, H, Y, G = to_bf16(w, cuda_device), to_bf16(h.reshape(-1, d), cuda_device), torch.from_numpy(t.reshape(-1)).to(
        cuda_device), torch.from_numpy(g).to(cuda_device)
    step = V // shards
    parts = [ops.shard_forward(W[r * step:(r + 1) * step], H, Y, 30.0, vocab_offset=r * step, want_logp=False)[0]
             for r in range(shards)]
    logp, norm = ops.combine(torch.stack(parts))
    ref = orc.vocab_parallel_logps_and_normalization(w, h, t, num_shards=shards, softcap=30.0, vocab_chunk=17,
                                                     sequence_chunk=6)
    assert np.abs(logp.cpu().numpy() - ref[0].reshape(-1)).max() <= LOGP_ATOL
    np.testing.assert_allclose(norm.cpu().numpy(), ref[1].reshape(2, -1), rtol=1e-4, atol=1e-4)
    dHs, dWs = [], []
    for r in range(shards):
        dH, dW = ops.shard_backward(W[r * step:(r + 1) * step], H, Y, 30.0, norm, G, vocab_offset=r * step,
                                    dh_dtype=torch.float32, dw_dtype=torch.float32)
        dHs.append(dH)
        dWs.append(dW)
    dH = torch.stack(dHs).sum(0).cpu().numpy()
    dW = torch.cat(dWs).cpu().numpy()
    _, dW_ref, dH_ref = orc.logps_grads_f64(w, h, t, g, 30.0)
    assert rel_l2(dH, dH_ref.reshape(-1, d)) <= GRAD_REL_L2
    assert rel_l2(dW, dW_ref) <= GRAD_REL_L2


# --------------------------------------------------------------------------- compaction / callers
def test_compaction_gather_and_scatter(cuda_device):
    from gemma4_posttrain_jax_b200 import ops

    rng = np.random.default_rng(3)
    B, S, N, d, pw = 5, 40, 29, 24, 12
    lens = np.array([0, 1, 29, 17, 5])
    mask = np.arange(N)[None, :] < lens[:, None]
    hidden = orc.bf16_round(rng.normal(size=(B, S, d)))
    ids = rng.integers(0, 1000, size=(B, N)).astype(np.int32)
    Hc, yc, idx, pos, count = ops.compact(torch.from_numpy(mask).to(cuda_device), to_bf16(hidden, cuda_device),
                                          torch.from_numpy(ids).to(cuda_device), row_offset=pw - 1)
    n = int(count.item())
    ref_idx = orc.compact_response(mask)
    assert n == ref_idx.size == lens.sum()
    np.testing.assert_array_equal(idx[:n].cpu().numpy(), ref_idx)
    ref_pos = np.full(B * N, -1)
    ref_pos[ref_idx] = np.arange(n)
    np.testing.assert_array_equal(pos.cpu().numpy(), ref_pos)
    b, j = ref_idx // N, ref_idx % N
    np.testing.assert_array_equal(Hc[:n].float().cpu().numpy(), hidden[b, j + pw - 1])
    np.testing.assert_array_equal(yc[:n].cpu().numpy(), ids[b, j])
    # scatter back into a strided response slice of a [B, S, d] buffer
    out = torch.full((B, S, d), 7.0, dtype=torch.bfloat16, device=cuda_device)
    ops.scatter_rows(Hc[:n], pos, out[:, pw - 1: pw - 1 + N])
    o = out.float().cpu().numpy()
    exp = np.zeros((B, N, d), np.float32)
    exp[b, j] = hidden[b, j + pw - 1]
    np.testing.assert_array_equal(o[:, pw - 1: pw - 1 + N], exp)
    assert (o[:, : pw - 1] == 7.0).all() and (o[:, pw - 1 + N:] == 7.0).all()
    # f32 rows scattered into a bf16 slice are rounded on the way
    src32 = torch.from_numpy(rng.normal(size=(n, d)).astype(np.float32)).to(cuda_device)
    out16 = torch.full((B, S, d), 7.0, dtype=torch.bfloat16, device=cuda_device)
    ops.scatter_rows(src32, pos, out16[:, pw - 1: pw - 1 + N])
    exp16 = torch.zeros((B, N, d), dtype=torch.bfloat16)
    exp16[torch.from_numpy(b), torch.from_numpy(j)] = src32.cpu().to(torch.bfloat16)
    assert torch.equal(out16[:, pw - 1: pw - 1 + N].cpu(), exp16)


def test_completion_logps_autograd_matches_oracle(cuda_device):
    from gemma4_posttrain_jax_b200.losses import completion_logps

    rng = np.random.default_rng(11)
    B, Pw, N, d, V = 4, 9, 23, 64, 1000
    S = Pw + N
    w = orc.bf16_round(rng.normal(size=(V, d)) * 0.2)
    hidden = orc.bf16_round(rng.normal(size=(B, S, d)))
    ids = rng.integers(0, V, size=(B, N)).astype(np.int32)
    mask = np.arange(N)[None, :] < np.array([23, 5, 0, 14])[:, None]
    adv = rng.normal(size=(B, 1)).astype(np.float32) * (rng.random((B, N)) < 0.9)
    W = to_bf16(w, cuda_device).requires_grad_(True)
    Hd = to_bf16(hidden, cuda_device).requires_grad_(True)
    out = completion_logps(W, Hd, torch.from_numpy(ids).to(cuda_device), torch.from_numpy(mask).to(cuda_device),
                           prompt_width=Pw, softcap=30.0)
    (out * torch.from_numpy(adv).to(cuda_device)).sum().backward()
    # oracle on the un-compacted response slice, masked afterwards (losses.py:667-682)
    resp = hidden[:, Pw - 1: Pw - 1 + N]
    safe = np.where(mask, ids, 0)
    ref = orc.dense_logps(w, resp, safe, 30.0)
    got = out.detach().cpu().numpy()
    assert np.abs(got[mask] - ref[mask]).max() <= LOGP_ATOL
    assert (got[~mask] == 0).all()
    gm = np.where(mask, adv, 0).astype(np.float32)
    _, dW_ref, dR_ref = orc.logps_grads_f64(w, resp, safe, gm, 30.0)
    dH_ref = np.zeros_like(hidden, dtype=np.float64)
    dH_ref[:, Pw - 1: Pw - 1 + N] = dR_ref
    assert rel_l2(W.grad.float().cpu().numpy(), dW_ref) <= GRAD_REL_L2
    assert rel_l2(Hd.grad.float().cpu().numpy(), dH_ref) <= GRAD_REL_L2


def test_per_token_logps_autograd_and_sft(cuda_device):
    from gemma4_posttrain_jax_b200.losses import per_token_logps, sft_token_logps

    rng = np.random.default_rng(5)
    B, S, d, V = 3, 41, 72, 777
    w = orc.bf16_round(rng.normal(size=(V, d)) * 0.3)
    hidden = orc.bf16_round(rng.normal(size=(B, S, d)))
    labels = rng.integers(0, V, size=(B, S)).astype(np.int64)
    labels[:, :3] = -100
    W = to_bf16(w, cuda_device).requires_grad_(True)
    Hd = to_bf16(hidden, cuda_device).requires_grad_(True)
    logps, mask = sft_token_logps(W, Hd, torch.from_numpy(labels).to(cuda_device), softcap=None)
    loss = -torch.where(mask, logps, torch.zeros_like(logps)).sum() / mask.sum().clamp(min=1)
    loss.backward()
    tgt = labels[:, 1:]
    m = tgt != -100
    safe = np.where(m, tgt, 0)
    ref = orc.dense_logps(w, hidden[:, :-1], safe, None)
    assert np.abs(logps.detach().cpu().numpy() - ref).max() <= LOGP_ATOL
    g = -m.astype(np.float64) / max(m.sum(), 1)
    _, dW_ref, dHs_ref = orc.logps_grads_f64(w, hidden[:, :-1], safe, g, None)
    dH_ref = np.zeros_like(hidden, dtype=np.float64)
    dH_ref[:, :-1] = dHs_ref
    assert rel_l2(W.grad.float().cpu().numpy(), dW_ref) <= GRAD_REL_L2
    assert rel_l2(Hd.grad.float().cpu().numpy(), dH_ref) <= GRAD_REL_L2
    # plain per_token_logps on [B, S-1] equals the SFT logps
    again = per_token_logps(W.detach(), Hd.detach()[:, :-1], torch.from_numpy(safe).to(cuda_device), softcap=None)
    assert torch.equal(again, logps.detach())


def test_config1_shape_fwd_bwd(cuda_device, cta_group):
    """BASELINE config 1 at full size: T=256, d=2048, V=262144, softcap 30, seed 0."""
    from gemma4_posttrain_jax_b200 import ops

    T, d, V = 256, 2048, 262144
    gen = torch.Generator(device="cpu").manual_seed(0)
    h = torch.randn((T, d), generator=gen).to(torch.bfloat16)
    w = (torch.randn((V, d), generator=gen) * 0.02).to(torch.bfloat16)
    y = torch.randint(0, V, (T,), generator=gen, dtype=torch.int32)
    g = torch.randn((T,), generator=gen)
    W, H, Y, G = w.to(cuda_device), h.to(cuda_device), y.to(cuda_device), g.to(cuda_device)
    stats, logp = ops.shard_forward(W, H, Y, 30.0)
    dH, dW = ops.shard_backward(W, H, Y, 30.0, stats[:2], G, dh_dtype=torch.float32, dw_dtype=torch.float32)
    torch.cuda.synchronize()
    wn, hn = w.float().numpy(), h.float().numpy()
    lp_ref, dW_ref, dH_ref = orc.fwd_bwd_f32(wn, hn, y.numpy(), g.numpy(), softcap=30.0, vocab_chunk=8192,
                                            sequence_chunk=128)
    assert np.abs(logp.cpu().numpy() - lp_ref).max() <= LOGP_ATOL
    assert rel_l2(dH.cpu().numpy(), dH_ref) <= GRAD_REL_L2
    assert rel_l2(dW.cpu().numpy(), dW_ref) <= GRAD_REL_L2


def test_zero_gradient_rows_are_skipped_without_changing_results(cuda_device):
    """The backward runs only on rows with nonzero upstream gradient; dH rows of the others
    are exactly zero and every other result equals the dense backward's up to f32 order."""
    from gemma4_posttrain_jax_b200.losses import completion_logps, per_token_logps

    rng = np.random.default_rng(29)
    T, d, V = 700, 96, 3000
    w = orc.bf16_round(rng.normal(size=(V, d)) * 0.3)
    h = orc.bf16_round(rng.normal(size=(T, d)))
    y = rng.integers(0, V, size=T).astype(np.int32)
    g = rng.normal(size=T).astype(np.float32) * (rng.random(T) < 0.6)
    grads = []
    for skip in (True, False):
        W = to_bf16(w, cuda_device).requires_grad_(True)
        H = to_bf16(h, cuda_device).requires_grad_(True)
        lp = per_token_logps(W, H, torch.from_numpy(y).to(cuda_device), softcap=30.0, skip_zero_grad=skip)
        (lp * torch.from_numpy(g).to(cuda_device)).sum().backward()
        grads.append((W.grad.float().cpu().numpy(), H.grad.float().cpu().numpy()))
    # dW / dH come back in bf16: a different f32 summation order flips a few roundings
    assert rel_l2(grads[0][0], grads[1][0]) < 1e-3
    assert rel_l2(grads[0][1], grads[1][1]) < 1e-3
    assert (grads[0][1][g == 0] == 0).all()
    _, dW_ref, dH_ref = orc.logps_grads_f64(w, h, y, g, 30.0)
    assert rel_l2(grads[0][0], dW_ref) <= GRAD_REL_L2 and rel_l2(grads[0][1], dH_ref) <= GRAD_REL_L2
    # all-zero upstream gradient: zero dW and dH
    W = to_bf16(w, cuda_device).requires_grad_(True)
    H = to_bf16(h, cuda_device).requires_grad_(True)
    lp = per_token_logps(W, H, torch.from_numpy(y).to(cuda_device), softcap=30.0)
    (lp * 0.0).sum().backward()
    assert (W.grad == 0).all() and (H.grad == 0).all()
    # GRPO caller with zero-advantage sequences
    B, Pw, N = 4, 3, 50
    hid = orc.bf16_round(rng.normal(size=(B, Pw + N, d)))
    ids = rng.integers(0, V, size=(B, N)).astype(np.int32)
    mask = np.arange(N)[None, :] < np.array([50, 20, 0, 33])[:, None]
    adv = np.array([[0.7], [0.0], [1.0], [-0.4]], np.float32) * (rng.random((B, N)) < 0.8)
    outs = []
    for skip in (True, False):
        W = to_bf16(w, cuda_device).requires_grad_(True)
        Hd = to_bf16(hid, cuda_device).requires_grad_(True)
        out = completion_logps(W, Hd, torch.from_numpy(ids).to(cuda_device), torch.from_numpy(mask).to(cuda_device),
                               prompt_width=Pw, softcap=30.0, skip_zero_grad=skip)
        (out * torch.from_numpy(adv).to(cuda_device)).sum().backward()
        outs.append((W.grad.float().cpu().numpy(), Hd.grad.float().cpu().numpy()))
    assert rel_l2(outs[0][0], outs[1][0]) < 1e-3
    assert rel_l2(outs[0][1], outs[1][1]) < 1e-3


@pytest.mark.parametrize("d,frozen_head", [(2560, False), (3840, True)])
def test_config3_and_config4_hidden_sizes(cuda_device, d, frozen_head):
    """BASELINE config 3 (d=2560, fwd+bwd plus a forward-only pass over W + N(0, 1e-4)) and
    config 4 (d=3840, frozen head: forward + dH only) at the full V=262144, on 256 tokens."""
    from gemma4_posttrain_jax_b200 import ops

    T, V = 256, 262144
    gen = torch.Generator(device="cpu").manual_seed(d)
    h = torch.randn((T, d), generator=gen).to(torch.bfloat16)
    w = (torch.randn((V, d), generator=gen) * 0.02).to(torch.bfloat16)
    y = torch.randint(0, V, (T,), generator=gen, dtype=torch.int32)
    g = torch.randn((T,), generator=gen)
    W, H, Y, G = w.to(cuda_device), h.to(cuda_device), y.to(cuda_device), g.to(cuda_device)
    stats, logp = ops.shard_forward(W, H, Y, 30.0)
    dH, dW = ops.shard_backward(W, H, Y, 30.0, stats[:2], G, need_dw=not frozen_head, dh_dtype=torch.float32)
    torch.cuda.synchronize()
    wn, hn = w.float().numpy(), h.float().numpy()
    lp_ref, dW_ref, dH_ref = orc.fwd_bwd_f32(wn, hn, y.numpy(), g.numpy(), softcap=30.0, vocab_chunk=8192,
                                            sequence_chunk=128)
    assert np.abs(logp.cpu().numpy() - lp_ref).max() <= LOGP_ATOL
    assert rel_l2(dH.cpu().numpy(), dH_ref) <= GRAD_REL_L2
    if frozen_head:
        assert dW is None
    else:
        assert rel_l2(dW.float().cpu().numpy(), dW_ref) <= GRAD_REL_L2
        # the second, forward-only pass of config 3 over a perturbed head (old / reference policy)
        w2 = (w.float() + torch.randn((V, d), generator=gen) * 1e-4).to(torch.bfloat16)
        _, logp2 = ops.shard_forward(w2.to(cuda_device), H, Y, 30.0)
        lp2_ref = orc.single_partition_logps(w2.float().numpy(), hn, y.numpy(), softcap=30.0, vocab_chunk=8192,
                                             sequence_chunk=128)
        assert np.abs(logp2.cpu().numpy() - lp2_ref).max() <= LOGP_ATOL


def test_microbatched_completion_logps_match_the_full_batch(cuda_device):
    """The reference's microbatch invariance (``tests/test_grpo.py:311-317``, atol / rtol
    3e-6): completion logps of a batch equal those of its 2-row microbatches, and so do the
    hidden-state gradients; dW summed over the microbatches matches the full batch's."""
    from gemma4_posttrain_jax_b200.losses import completion_logps

    rng = np.random.default_rng(5)
    B, Pw, N, d, V = 6, 7, 150, 128, 3000
    w = orc.bf16_round(rng.normal(size=(V, d)) * 0.3)
    hidden = orc.bf16_round(rng.normal(size=(B, Pw + N, d)))
    ids = rng.integers(0, V, size=(B, N)).astype(np.int32)
    mask = np.arange(N)[None, :] < np.array([150, 40, 0, 77, 150, 3])[:, None]
    adv = (rng.normal(size=(B, 1)) * (rng.random((B, N)) < 0.9)).astype(np.float32)
    W = to_bf16(w, cuda_device).requires_grad_(True)
    Hd = to_bf16(hidden, cuda_device).requires_grad_(True)
    Y, M, G = (torch.from_numpy(x).to(cuda_device) for x in (ids, mask, adv))
    full = completion_logps(W, Hd, Y, M, prompt_width=Pw, softcap=30.0)
    (full * G).sum().backward()
    dW_full, dH_full = W.grad.float().clone(), Hd.grad.float().clone()
    W.grad = None
    parts, dH_parts = [], []
    for b0 in range(0, B, 2):
        Hb = Hd.detach()[b0 : b0 + 2].clone().requires_grad_(True)
        out = completion_logps(W, Hb, Y[b0 : b0 + 2], M[b0 : b0 + 2], prompt_width=Pw, softcap=30.0)
        (out * G[b0 : b0 + 2]).sum().backward()
        parts.append(out.detach())
        dH_parts.append(Hb.grad.float())
    split = torch.cat(parts).cpu().numpy()
    np.testing.assert_allclose(split, full.detach().cpu().numpy(), atol=3e-6, rtol=3e-6)
    assert rel_l2(torch.cat(dH_parts).cpu().numpy(), dH_full.cpu().numpy()) <= 5e-3
    assert rel_l2(W.grad.float().cpu().numpy(), dW_full.cpu().numpy()) <= 1e-2
