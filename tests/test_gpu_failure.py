"""Failure detection on one GPU without a GPU fault: bounded device-side waits
made to run out.

Every wait of the library's kernels is bounded (rib_set_wait_limit_ns, 2 s
by default).  Each test lowers the limit to 20 ms, launches a kernel whose
peer never arrives -- the "peer" is a second buffer in this GPU's own memory
that nothing writes -- and checks that the launch returns, that the device
status word reads RIB_ETIMEOUT, that what the kernel produced before the
wait is intact, and that the next ordinary call is correct.  No fault, trap
or unbounded loop is involved.  The reference's analogue is the v3
harness's per-unit timeout and exclusion record (agent-test/v3/run.py:238-261).
"""
from __future__ import annotations

import ctypes
import importlib
import time

import numpy as np
import pytest
import torch

from conftest import bf16f, u16

pytestmark = pytest.mark.gpu
LIMIT_NS = 20_000_000  # 20 ms


@pytest.fixture()
def lib():
    m = importlib.import_module("roofline-inference_b200._lib")
    assert m.take_device_status() == 0
    yield m
    m.set_wait_limit_ns(m.DEFAULT_WAIT_LIMIT_NS)
    assert m.wait_limit_ns() == m.DEFAULT_WAIT_LIMIT_NS


def test_wait_limit_range(lib):
    with pytest.raises(ValueError):
        lib.set_wait_limit_ns(10)
    with pytest.raises(ValueError):
        lib.set_wait_limit_ns(61_000_000_000)
    lib.set_wait_limit_ns(LIMIT_NS)
    assert lib.wait_limit_ns() == LIMIT_NS


def test_gather_epoch_wait_times_out(lib, rib, wl, oracle):
    """The fused decode + NVLink all-gather with world = 2, where rank 1's
    buffer is local memory and rank 1 never publishes its epoch: the last
    unit's bounded wait for the peer runs out."""
    ng = importlib.import_module("roofline-inference_b200.nvlink_gather")
    L = lib.load()
    ng._bind(L)
    n = 4096
    st = wl.decode_step(n, seed=3, device="cuda")        # cache rows [0, 4096) filled
    cap = st.cache.shape[2]
    q = wl.randn_bf16((1, 16, 128), seed=4, device="cuda")
    ptrs = torch.tensor([st.cache.data_ptr()], dtype=torch.int64, device="cuda")
    lens = torch.tensor([n], dtype=torch.int32, device="cuda")
    nbytes = int(L.rib_peer_buffer_bytes(1, 32))         # batch 1, 2 ranks x 16 heads
    region = (nbytes - 256) // 2
    bufs = [torch.zeros(nbytes, dtype=torch.uint8, device="cuda") for _ in range(2)]
    g = ng._PeerGatherStruct()
    g.world, g.rank, g.region_bytes = 2, 0, region
    for r in range(2):
        g.out[r] = bufs[r].data_ptr()
        g.sig[r] = bufs[r].data_ptr() + 2 * region
    ws = torch.zeros(int(L.rib_decode_workspace_bytes(1, n, 8)), dtype=torch.uint8, device="cuda")
    epoch = 1
    lib.set_wait_limit_ns(LIMIT_NS)
    t0 = time.perf_counter()
    s = L.rib_decode_attention_gather(q.data_ptr(), ptrs.data_ptr(), lens.data_ptr(), 1, n, cap, 16, 8,
                                      wl.SCALE, ctypes.byref(g), epoch, ws.data_ptr(), ws.numel(),
                                      torch.cuda.current_stream().cuda_stream)
    assert s == 0
    status = lib.take_device_status()                     # synchronises the device
    elapsed = time.perf_counter() - t0
    assert status == lib.RIB_ETIMEOUT, status
    assert elapsed < 1.5, elapsed
    # this rank's 16 head outputs went to both ranks' regions before the wait
    of, _ = oracle.decode_attention(u16(q[0]), u16(st.cache), n, wl.SCALE)
    off = (epoch & 1) * region
    for r in range(2):
        heads = bufs[r][off:off + 32 * 128 * 2].view(torch.bfloat16).reshape(32, 128)[:16]
        err = np.abs(bf16f(heads) - of)
        assert err.max() <= 2e-2 and err.mean() <= 2e-3, err.max()
    # and our epoch reached the stand-in peer's slot for rank 0
    assert int(bufs[1][2 * region:2 * region + 8].view(torch.int64).item()) == epoch
    # the library recovers: an ordinary decode is right and the status stays clean
    lib.set_wait_limit_ns(lib.DEFAULT_WAIT_LIMIT_NS)
    out = rib.decode_attention(q.reshape(1, 16, 1, 128), st.cache, n, wl.SCALE)
    err = np.abs(bf16f(out.reshape(16, 128)) - of)
    assert err.max() <= 2e-2 and err.mean() <= 2e-3
    assert lib.take_device_status() == 0


def test_tensor_parallel_partial_wait_times_out(lib, rib, wl):
    """A tensor-parallel GEMV whose input is the residual plus every rank's
    published partial sums (in_sum), with world = 2 and exchange buffers that
    never carry the awaited epoch: the tagged-word polls run out."""
    tp = importlib.import_module("roofline-inference_b200.tp")
    from oracle import model_np
    L = lib.load()
    tp._bind(L)
    N, K, slot = 256, 1024, 1024
    nb = int(L.rib_tp_buffer_bytes(2, slot))
    bufs = [torch.zeros(nb, dtype=torch.uint8, device="cuda") for _ in range(2)]
    epoch = torch.tensor([6], dtype=torch.int64, device="cuda")  # words carry tag 0, never 6
    done = torch.zeros(1, dtype=torch.int32, device="cuda")
    ex = tp._TpExchangeStruct()
    ex.world, ex.rank, ex.slot = 2, 0, slot
    ex.buf[0], ex.buf[1] = bufs[0].data_ptr(), bufs[1].data_ptr()
    ex.epoch, ex.done = epoch.data_ptr(), done.data_ptr()
    W = wl.randn_bf16((N, K), seed=7, device="cuda", scale=0.02)
    x = wl.randn_bf16((K,), seed=8, device="cuda")
    y = torch.empty(N, dtype=torch.bfloat16, device="cuda")
    x_out = torch.empty(K, dtype=torch.bfloat16, device="cuda")
    lib.set_wait_limit_ns(LIMIT_NS)
    t0 = time.perf_counter()
    s = L.rib_gemv_tp(W.data_ptr(), N, K, x.data_ptr(), None, 0, 0, y.data_ptr(), ctypes.byref(ex), 1,
                      x_out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert s == 0
    status = lib.take_device_status()
    elapsed = time.perf_counter() - t0
    assert status == lib.RIB_ETIMEOUT, status
    assert elapsed < 1.5, elapsed
    assert int(epoch.item()) == 6  # an input-side wait publishes nothing
    lib.set_wait_limit_ns(lib.DEFAULT_WAIT_LIMIT_NS)
    got = rib.gemv(W, x)
    want = model_np.gemv(u16(W), u16(x))
    assert np.abs(bf16f(got) - bf16f(want)).max() <= np.abs(bf16f(want)).max() * 2.0 ** -7
    assert lib.take_device_status() == 0


def test_tp_prefill_exchange_wait_times_out(lib, rib, wl):
    """The tensor-parallel prefill exchange with world = 2, where "rank 1" is
    a second buffer in this GPU's memory that no kernel signals: the owner-slot
    GEMM stores its partials, the reduce kernel publishes this rank's signal
    to both buffers and its wait for rank 1's runs out; the residual is left
    untouched, and the next exchange on fresh buffers is correct."""
    tp = importlib.import_module("roofline-inference_b200.tp")
    from oracle import model_np
    L = lib.load()
    tp._bind(L)
    M, K, H = 64, 256, 256
    nb = int(L.rib_tp_prefill_buffer_bytes(2, M, H))
    bufs = [torch.zeros(nb, dtype=torch.uint8, device="cuda") for _ in range(2)]
    ex = tp._PrefillExchangeStruct()
    ex.world, ex.rank, ex.rows_cap, ex.hidden = 2, 0, M, H
    ex.buf[0], ex.buf[1] = bufs[0].data_ptr(), bufs[1].data_ptr()
    A = wl.randn_bf16((M, K), seed=21, device="cuda")
    W = wl.randn_bf16((H, K), seed=22, device="cuda", scale=K ** -0.5)
    h = wl.randn_bf16((M, H), seed=23, device="cuda")
    h_before = h.clone()
    st = torch.cuda.current_stream().cuda_stream
    lib.set_wait_limit_ns(LIMIT_NS)
    t0 = time.perf_counter()
    assert L.rib_gemm_tp_partial(A.data_ptr(), M, K, W.data_ptr(), ctypes.byref(ex), st) == 0
    assert L.rib_tp_reduce_add_rms(ctypes.byref(ex), M, 1, h.data_ptr(), None, None, st) == 0
    status = lib.take_device_status()
    elapsed = time.perf_counter() - t0
    assert status == lib.RIB_ETIMEOUT, status
    assert elapsed < 1.5, elapsed
    assert torch.equal(h, h_before)
    f0, f1 = bufs[0][:128].view(torch.int64).cpu(), bufs[1][:128].view(torch.int64).cpu()
    assert int(f0[0]) == 1 and int(f1[0]) == 1       # rank 0's "partials in place" reached both
    assert int(f0[1]) == 0 and int(f0[8]) == 0       # nothing from rank 1; no "rows in place"
    lib.set_wait_limit_ns(lib.DEFAULT_WAIT_LIMIT_NS)
    one = torch.zeros(int(L.rib_tp_prefill_buffer_bytes(1, M, H)), dtype=torch.uint8, device="cuda")
    ex1 = tp._PrefillExchangeStruct()
    ex1.world, ex1.rank, ex1.rows_cap, ex1.hidden = 1, 0, M, H
    ex1.buf[0] = one.data_ptr()
    assert L.rib_gemm_tp_partial(A.data_ptr(), M, K, W.data_ptr(), ctypes.byref(ex1), st) == 0
    assert L.rib_tp_reduce_add_rms(ctypes.byref(ex1), M, 1, h.data_ptr(), None, None, st) == 0
    torch.cuda.synchronize()
    r = model_np.matmul(u16(A), u16(W))
    want = model_np.add_rms(u16(h_before), r, np.full(H, 0x3F80, np.uint16))[0]  # the residual bf16(h + r)
    assert np.abs(bf16f(h) - bf16f(want)).max() <= np.abs(bf16f(want)).max() * 2.0 ** -7
    assert lib.take_device_status() == 0
