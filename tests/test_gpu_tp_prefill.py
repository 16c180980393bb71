"""GPU: the tensor-parallel prefill exchange (rib_gemm_tp_partial, then
rib_tp_reduce_add_rms) against the oracle.

With one rank every row is owned locally and every signal is the rank's own,
so the whole protocol -- the owner-slot epilogue of the tcgen05 GEMM, the
rank-order reduction, the gather-buffer stores, both flag rounds and the
residual add + RMSNorm -- runs on one GPU.  The expected values are the
oracle's: the FP32 partial sums of the ranks added in rank order, rounded
once to BF16, then add_rms (agent-test/v2/kernels.py:227-268) or the plain
residual add of the last layer.  The same calls on two GPUs are in
test_gpu_multi.py.
"""
from __future__ import annotations

import ctypes
import importlib

import numpy as np
import pytest
import torch

from conftest import bf16f, u16

pytestmark = pytest.mark.gpu


def expected(parts_in, h, nw):
    """The oracle's row-parallel projection + add_rms (u16 in and out)."""
    from oracle import model_np
    return model_np.row_parallel_add_rms(parts_in, h, nw)


def close_bf16(got, want, what):
    g, w = bf16f(got).astype(np.float64), bf16f(want).astype(np.float64)
    # FP32 tensor-core sums against FP64 ones: the BF16 rounding of the sum
    # may land one step apart -- a step of the sum's own size, which a
    # residual add that nearly cancels keeps -- and the RMSNorm carries it
    scale = np.abs(w).max(axis=-1, keepdims=True)
    assert np.all(np.abs(g - w) <= 2.0 ** -6 * np.abs(w) + 2.0 ** -7 * scale), \
        f"{what}: max abs diff {np.abs(g - w).max()}"
    assert np.mean(g == w) >= 0.98, f"{what}: only {np.mean(g == w):.4f} of the elements bit-equal"


@pytest.fixture(scope="module")
def tpx():
    rib = importlib.import_module("roofline-inference_b200")
    T = importlib.import_module("roofline-inference_b200.tp")
    L = rib.load_library()
    T._bind(L)
    return rib, T, L


def one_rank_exchange(T, L, rows_cap, H):
    nb = int(L.rib_tp_prefill_buffer_bytes(1, rows_cap, H))
    assert nb > 0
    buf = torch.zeros(nb, dtype=torch.uint8, device="cuda")
    s = T._PrefillExchangeStruct()
    s.world, s.rank, s.rows_cap, s.hidden = 1, 0, rows_cap, H
    s.buf[0] = buf.data_ptr()
    return buf, s


@pytest.mark.parametrize("M,K,H,norm", [(1, 1024, 1024, True), (37, 256, 256, True), (300, 1024, 1024, False),
                                        (4096, 2048, 1024, True), (129, 3072, 1024, True), (64, 64, 2048, True)])
def test_prefill_exchange_one_rank(tpx, wl, M, K, H, norm):
    rib, T, L = tpx
    from oracle import model_np
    buf, ex = one_rank_exchange(T, L, max(M, 512), H)
    st = torch.cuda.current_stream().cuda_stream
    epoch = 0
    # three pairs on the same buffers (epochs 1, 2, 3): the flags and the CTA
    # counter carry over correctly from call to call
    for rep in range(3):
        A = wl.randn_bf16((M, K), seed=100 + rep, device="cuda")
        W = wl.randn_bf16((H, K), seed=200 + rep, device="cuda", scale=K ** -0.5)
        h = wl.randn_bf16((M, H), seed=300 + rep, device="cuda")
        nw = wl.randn_bf16((H,), seed=400 + rep, device="cuda", scale=0.1) + 1.0 if norm else None
        nw = nw.to(torch.bfloat16) if nw is not None else None
        h0 = u16(h)
        out = torch.empty_like(h) if norm else None
        epoch += 1
        assert L.rib_gemm_tp_partial(A.data_ptr(), M, K, W.data_ptr(), ctypes.byref(ex), st) == 0
        assert L.rib_tp_reduce_add_rms(ctypes.byref(ex), M, epoch, h.data_ptr(),
                                       None if nw is None else nw.data_ptr(),
                                       None if out is None else out.data_ptr(), st) == 0
        torch.cuda.synchronize()
        res, x = expected([(u16(A), u16(W))], h0, None if nw is None else u16(nw))
        close_bf16(h, res, f"residual rep {rep}")
        if norm:
            close_bf16(out, x, f"normalised rep {rep}")
            # the normalisation of the kernel's own residual (the FP32 sum of
            # squares adds in another order than the oracle's)
            close_bf16(out, model_np.rms_norm(u16(h), u16(nw)), f"norm of the residual rep {rep}")
    assert importlib.import_module("roofline-inference_b200._lib").take_device_status() == 0
    del buf


def test_prefill_exchange_matches_gemm_and_add_rms(tpx, wl):
    """One rank: the exchange's output is bit-identical to the plain FP32
    tcgen05 GEMM followed by the BF16 rounding and rib_add_rms."""
    rib, T, L = tpx
    M, K, H = 1000, 1024, 1024
    buf, ex = one_rank_exchange(T, L, M, H)
    A = wl.randn_bf16((M, K), seed=1, device="cuda")
    W = wl.randn_bf16((H, K), seed=2, device="cuda", scale=K ** -0.5)
    h = wl.randn_bf16((M, H), seed=3, device="cuda")
    nw = (wl.randn_bf16((H,), seed=4, device="cuda", scale=0.1) + 1.0).to(torch.bfloat16)
    G = importlib.import_module("roofline-inference_b200.gemm")
    part = G.gemm(A, W, epi="f32", small=False)
    want_h, want_x = rib.add_rms(h, part.to(torch.bfloat16), nw)
    out = torch.empty_like(h)
    st = torch.cuda.current_stream().cuda_stream
    assert L.rib_gemm_tp_partial(A.data_ptr(), M, K, W.data_ptr(), ctypes.byref(ex), st) == 0
    assert L.rib_tp_reduce_add_rms(ctypes.byref(ex), M, 1, h.data_ptr(), nw.data_ptr(), out.data_ptr(), st) == 0
    torch.cuda.synchronize()
    assert torch.equal(h, want_h)
    assert torch.equal(out, want_x)
