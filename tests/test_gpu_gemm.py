"""GPU parity of the tcgen05 prefill GEMM (csrc/gemm.cuh) against the model
oracle (oracle/model_np.py), whose GEMM and SwiGLU rounding points are pinned
to the reference's own kernels (tests/test_oracle.py), and of the fused
QKV + RMSNorm + RoPE + KV-append epilogue against the oracle and against
the two-kernel path it replaces.

Tolerance: every BF16 output within one BF16 ulp of the oracle's (an FP32
sum against an FP64 one can land on the other side of a rounding boundary)
and at most 2% of elements differing; FP32 outputs within 1e-5 of the
largest; RoPE outputs within the reference's 3.2e-2 (test_engine.py:75-77)."""
from __future__ import annotations

import importlib

import numpy as np
import pytest
import torch

from conftest import bf16f, u16

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def G():
    return importlib.import_module("roofline-inference_b200.gemm")


def _ulp_close(got_u16, want_u16, frac=0.02):
    g, w = bf16f(got_u16).astype(np.float64), bf16f(want_u16).astype(np.float64)
    # one BF16 ulp of the value, plus FP32 summation noise of the matrix's scale
    tol = np.maximum(np.abs(w), np.abs(g)) * 2.0 ** -7 + 1e-5 * np.abs(w).max() + 1e-30
    bad = np.abs(g - w) > tol
    assert not bad.any(), (np.abs(g - w)[bad].max(), int(bad.sum()))
    assert (got_u16 != want_u16).mean() <= frac, (got_u16 != want_u16).mean()


def _inputs(wl, M, N, K, seed):
    A = wl.randn_bf16((M, K), seed=seed, device="cuda")
    W = wl.randn_bf16((N, K), seed=seed + 1, device="cuda", scale=0.02)
    return A, W


@pytest.mark.parametrize("M,N,K", [(37, 256, 1024), (300, 4096, 1024), (513, 1024, 2048), (128, 384, 384),
                                   (1, 128, 64), (2049, 6144, 1024), (70, 1000, 256)])
def test_gemm_bf16_matches_oracle(G, wl, M, N, K):
    from oracle import model_np
    A, W = _inputs(wl, M, N, K, seed=M + N)
    C = G.gemm(A, W)
    torch.cuda.synchronize()
    assert tuple(C.shape) == (M, N)
    rows = slice(None) if M <= 600 else np.r_[0:64, M // 2:M // 2 + 64, M - 64:M]
    want = model_np.matmul(u16(A)[rows], u16(W))
    _ulp_close(u16(C)[rows], want)


def test_gemm_qwen3_shapes_4096(G, wl):
    """The four projections of a 4096-token prefill (QKV, O, gate/up, down),
    sampled rows against the oracle."""
    from oracle import model_np
    for N, K in ((4096, 1024), (1024, 2048), (6144, 1024), (1024, 3072)):
        A, W = _inputs(wl, 4096, N, K, seed=N + K)
        C = G.gemm(A, W)
        torch.cuda.synchronize()
        rows = np.r_[0:32, 2000:2032, 4064:4096]
        _ulp_close(u16(C)[rows], model_np.matmul(u16(A)[rows], u16(W)))


@pytest.mark.parametrize("M", [1, 16, 37, 64])
@pytest.mark.parametrize("N,K,epi", [(4096, 1024, "bf16"), (1024, 2048, "bf16"), (1024, 3072, "bf16"),
                                     (6144, 1024, "swiglu"), (256, 64, "bf16"), (512, 128, "swiglu")])
def test_gemm_few_rows_matches_oracle(G, wl, M, N, K, epi):
    """The few-row GEMM (rib_gemm_small: weights as the 128-row operand, K
    split over the GPU, partials summed in split order) against the oracle,
    at the Qwen3 projection shapes of a 64-sequence batched decode step; two
    calls in a row on the shared partials buffer give the same bits."""
    from oracle import model_np
    A, W = _inputs(wl, M, N, K, seed=M * 7 + N + K)
    y = G.gemm(A, W, epi=epi, small=True)
    y2 = G.gemm(A, W, epi=epi, small=True)
    torch.cuda.synchronize()
    assert torch.equal(y, y2)
    want = model_np.matmul(u16(A), u16(W))
    if epi == "swiglu":
        want = model_np.swiglu(want)
        d = np.abs(bf16f(u16(y)) - bf16f(want))
        assert d.max() <= 6.25e-2, d.max()
        assert (u16(y) != want).mean() <= 0.02
        assert torch.equal(y, importlib.import_module("roofline-inference_b200").swiglu(G.gemm(A, W, small=True)))
    else:
        _ulp_close(u16(y), want)


def test_gemm_few_rows_routing(G, wl):
    """gemm() takes the few-row kernel by default up to 64 rows where its
    shape rules hold, and refuses it explicitly where they do not."""
    assert G.small_ok(64, 4096, 1024, "bf16") and G.small_ok(1, 6144, 1024, "swiglu")
    assert not G.small_ok(65, 4096, 1024, "bf16")
    assert not G.small_ok(16, 1000, 1024, "bf16")
    assert not G.small_ok(16, 4096, 1024, "f32")
    A, W = _inputs(wl, 16, 1000, 256, seed=3)
    with pytest.raises(ValueError):
        G.gemm(A, W, small=True)


@pytest.mark.parametrize("M,N,K", [(200, 512, 3072), (33, 1000, 256)])
def test_gemm_f32(G, wl, M, N, K):
    A, W = _inputs(wl, M, N, K, seed=5)
    C = G.gemm(A, W, epi="f32")
    torch.cuda.synchronize()
    ref = bf16f(u16(A)).astype(np.float64) @ bf16f(u16(W)).astype(np.float64).T
    err = np.abs(C.cpu().numpy() - ref).max()
    assert err <= 1e-5 * np.abs(ref).max(), err


@pytest.mark.parametrize("M,F,K", [(64, 3072, 1024), (4096, 3072, 1024), (130, 384, 128)])
def test_gemm_swiglu_matches_oracle(G, wl, M, F, K):
    from oracle import model_np
    A, W = _inputs(wl, M, 2 * F, K, seed=F + K)
    y = G.gemm(A, W, epi="swiglu")
    torch.cuda.synchronize()
    assert tuple(y.shape) == (M, F)
    rows = slice(None) if M <= 600 else np.r_[0:64, M - 64:M]
    want = model_np.swiglu(model_np.matmul(u16(A)[rows], u16(W)))
    # five BF16 rounding points compound: the reference test's SwiGLU bound,
    # <= 1 BF16 ulp at |y| < 16 (agent-test/v2/test_engine.py:40)
    d = np.abs(bf16f(u16(y)[rows]) - bf16f(want))
    assert d.max() <= 6.25e-2, d.max()
    assert (u16(y)[rows] != want).mean() <= 0.02
    # bit-identical to the unfused path on the same BF16 products
    ref2 = importlib.import_module("roofline-inference_b200").swiglu(G.gemm(A, W))
    assert torch.equal(y, ref2)


@pytest.mark.parametrize("M,pos0,nkv", [(37, 0, 8), (300, 500, 8), (4096, 0, 8), (129, 32000, 4), (1, 7, 1)])
def test_gemm_qkv_rope(G, rib, wl, oracle, M, pos0, nkv):
    nq = 2 * nkv
    K = 1024
    A, W = _inputs(wl, M, (nq + 2 * nkv) * 128, K, seed=M + pos0)
    qw, kw = wl.norm_weights(3, "cuda"), wl.norm_weights(4, "cuda")
    cap = wl.round_cap(pos0 + M + 5)
    cache = wl.randn_bf16((2, nkv, cap, 128), seed=9, device="cuda")
    before = cache.clone()
    Lp = (M + 31) // 32 * 32
    table = G.rope_table(pos0, M, 1e6, "cuda")
    Q = G.gemm_qkv_rope(A, W, qw, kw, table, pos0, nq, nkv, cache, Lp)
    torch.cuda.synchronize()
    # exact write rows: nothing outside [pos0, pos0 + M) changed; pad rows zero
    keep = np.ones(cap, bool)
    keep[pos0:pos0 + M] = False
    assert np.array_equal(u16(cache)[:, :, keep], u16(before)[:, :, keep])
    assert not Q[:, M:].any()
    # bit-identical to the two-kernel path on the same BF16 projection (the
    # tiled GEMM's: the few-row kernel sums K in another order)
    qkv = G.gemm(A, W, small=False)
    cache2 = before.clone()
    Q2 = rib.qk_norm_rope_append(qkv, qw, kw, pos0, nq, nkv, 1e6, cache2, Lp)
    torch.cuda.synchronize()
    assert torch.equal(Q, Q2)
    assert torch.equal(cache, cache2)
    # against the oracle: oracle GEMM (FP64 sums) then the oracle's norm + RoPE
    from oracle import model_np
    rows = slice(None) if M <= 600 else np.r_[0:64, M - 64:M]
    qkv_o = model_np.matmul(u16(A)[rows], u16(W))
    Qo, KVo = oracle.qk_norm_rope(qkv_o, u16(qw), u16(kw), 0, nq, nkv, 1e6)
    if isinstance(rows, slice):
        pos_rows = np.arange(pos0, pos0 + M)
        q_rows = np.arange(M)
    else:
        pos_rows, q_rows = pos0 + rows, rows
    # the oracle was run at offset 0 over the sampled rows: redo its RoPE at the true positions
    Qo, KVo = _oracle_at_positions(oracle, qkv_o, qw, kw, nq, nkv, pos_rows)
    got_q = u16(Q)[:, q_rows]
    d = np.abs(bf16f(got_q) - bf16f(Qo))
    assert d.max() <= 3.2e-2 and (got_q != Qo).sum() <= max(8, 0.02 * got_q.size)
    got_k = u16(cache)[0][:, pos_rows]
    assert np.abs(bf16f(got_k) - bf16f(KVo[0])).max() <= 3.2e-2
    _ulp_close(u16(cache)[1][:, pos_rows], KVo[1])


def _oracle_at_positions(oracle, qkv_rows, qw, kw, nq, nkv, positions):
    """Oracle norm + RoPE of each row at its own position (rows need not be
    consecutive)."""
    Qs, Ks, Vs = [], [], []
    for r, pos in enumerate(positions):
        Q, KV = oracle.qk_norm_rope(qkv_rows[r:r + 1], u16(qw), u16(kw), int(pos), nq, nkv, 1e6)
        Qs.append(Q[:, 0])
        Ks.append(KV[0, :, 0])
        Vs.append(KV[1, :, 0])
    return np.stack(Qs, axis=1), np.stack([np.stack(Ks, axis=1), np.stack(Vs, axis=1)])


def test_gemm_argument_checks(G, wl):
    A, W = _inputs(wl, 16, 128, 64, seed=1)
    with pytest.raises(ValueError):
        G.gemm(A, W[:, :32].contiguous())          # K mismatch
    with pytest.raises(ValueError):
        G.gemm(A[:, :32].contiguous(), W[:, :32].contiguous())  # K not a multiple of 64
    with pytest.raises(ValueError):
        G.gemm(A, wl.randn_bf16((100, 64), seed=2, device="cuda"))  # N not a multiple of 8
    with pytest.raises(ValueError):
        G.gemm(A, W, epi="swiglu", small=False)    # F = 64 is not a multiple of 128 (tiled GEMM)
