"""CPU: the C-ABI library loads, exports every entry point the header
declares, and rejects bad arguments on the host (before any launch) with the
documented status codes.  No call here reaches a kernel launch."""
from __future__ import annotations

import ctypes
import re

import pytest

from conftest import ROOT

HEADER = ROOT / "include" / "rib_attention.h"
FAKE = 0x10000  # 16-byte aligned dummy address; never dereferenced
MISALIGNED = 0x10008


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(rib_\w+)\s*\(", text)))


def test_header_declares_expected_entry_points():
    names = declared_functions()
    for n in ["rib_qk_norm_rope", "rib_qk_norm_rope_prefill", "rib_qk_norm_rope_append",
              "rib_decode_attention", "rib_decode_attention_batched", "rib_prefill_attention",
              "rib_decode_workspace_bytes", "rib_version", "rib_status_string",
              "rib_take_device_status"]:
        assert n in names


def test_library_exports_every_declared_symbol(rib):
    L = rib.load_library()
    for name in declared_functions():
        assert hasattr(L, name), name


def test_status_strings(rib):
    L = rib.load_library()
    assert L.rib_status_string(0) == b"ok"
    assert L.rib_status_string(2) == b"KV capacity exceeded"
    assert L.rib_version() >> 16 == 1


def test_workspace_bytes(rib):
    L = rib.load_library()
    a = L.rib_decode_workspace_bytes(1, 513, 8)
    b = L.rib_decode_workspace_bytes(1, 32769, 8)
    c = L.rib_decode_workspace_bytes(64, 32768, 8)
    assert 0 < a <= b < c
    assert L.rib_decode_workspace_bytes(0, 10, 8) == 0


def test_workspace_init_rejects_bad_arguments(rib):
    L = rib.load_library()
    assert L.rib_decode_workspace_init(None, 1 << 20, None) == 1
    assert L.rib_decode_workspace_init(FAKE, 4096, None) == 1
    assert L.rib_decode_workspace_init(MISALIGNED, 1 << 20, None) == 3


def test_decode_rejects_bad_arguments(rib):
    L = rib.load_library()
    ws = L.rib_decode_workspace_bytes(1, 100, 8)
    # GQA factor must be 2
    assert L.rib_decode_attention(FAKE, FAKE, 256, 100, 15, 8, 0.088, FAKE, FAKE, ws, None) == 1
    # n beyond capacity
    assert L.rib_decode_attention(FAKE, FAKE, 256, 300, 16, 8, 0.088, FAKE, FAKE, ws, None) == 2
    # misaligned pointer
    assert L.rib_decode_attention(MISALIGNED, FAKE, 256, 100, 16, 8, 0.088, FAKE, FAKE, ws,
                                  None) == 3
    # null pointers
    assert L.rib_decode_attention(None, FAKE, 256, 100, 16, 8, 0.088, FAKE, FAKE, ws, None) == 1
    assert L.rib_decode_attention_batched(FAKE, None, FAKE, 2, 100, 256, 16, 8, 0.088, FAKE,
                                          FAKE, ws, None) == 1
    assert L.rib_decode_attention_batched(FAKE, FAKE, FAKE, 2, 300, 256, 16, 8, 0.088, FAKE,
                                          FAKE, ws, None) == 2


def test_rope_rejects_bad_arguments(rib):
    L = rib.load_library()
    # offset + L beyond the cache capacity -> "KV capacity exceeded"
    assert L.rib_qk_norm_rope_append(FAKE, 37, FAKE, FAKE, 240, 16, 8, 1e6, 37, FAKE, FAKE, 256,
                                     None) == 2
    # Lp < L
    assert L.rib_qk_norm_rope_prefill(FAKE, 37, FAKE, FAKE, 0, 16, 8, 1e6, 32, FAKE, FAKE,
                                      None) == 1
    # misaligned
    assert L.rib_qk_norm_rope(MISALIGNED, FAKE, FAKE, 0, 16, 8, 1e6, FAKE, FAKE, None) == 3
    # too many heads per token
    assert L.rib_qk_norm_rope(FAKE, FAKE, FAKE, 0, 60, 8, 1e6, FAKE, FAKE, None) == 1


def test_prefill_rejects_bad_arguments(rib):
    L = rib.load_library()
    ws = L.rib_prefill_workspace_bytes(64, 8)
    assert ws == 8 * 64 * 128 * 2 and L.rib_prefill_workspace_bytes(0, 8) == 0
    # H != 2 * nkv
    assert L.rib_prefill_attention(FAKE, FAKE, FAKE, 64, 64, 64, 256, 12, 8, 0.088, FAKE,
                                   FAKE, ws, None) == 1
    # kL < qL
    assert L.rib_prefill_attention(FAKE, FAKE, FAKE, 64, 32, 64, 256, 16, 8, 0.088, FAKE,
                                   FAKE, ws, None) == 1
    # kL beyond cap
    assert L.rib_prefill_attention(FAKE, FAKE, FAKE, 64, 300, 64, 256, 16, 8, 0.088, FAKE,
                                   FAKE, ws, None) == 2
    # workspace too small, or missing
    assert L.rib_prefill_attention(FAKE, FAKE, FAKE, 64, 64, 64, 256, 16, 8, 0.088, FAKE,
                                   FAKE, ws - 16, None) == 1
    assert L.rib_prefill_attention(FAKE, FAKE, FAKE, 64, 64, 64, 256, 16, 8, 0.088, FAKE,
                                   None, ws, None) == 1
    # misaligned
    assert L.rib_prefill_attention(MISALIGNED, FAKE, FAKE, 64, 64, 64, 256, 16, 8, 0.088, FAKE,
                                   FAKE, ws, None) == 3
    assert L.rib_prefill_attention(FAKE, FAKE, FAKE, 64, 64, 64, 256, 16, 8, 0.088, FAKE,
                                   MISALIGNED, ws, None) == 3


def test_gemm_rejects_bad_arguments(rib):
    import importlib
    G = importlib.import_module("roofline-inference_b200.gemm")
    L = G._L()
    # K not a multiple of 64, N not a multiple of 8, unknown epilogue
    assert L.rib_gemm(FAKE, 64, 96, FAKE, 128, 0, FAKE, 128, None) == 1
    assert L.rib_gemm(FAKE, 64, 128, FAKE, 100, 0, FAKE, 100, None) == 1
    assert L.rib_gemm(FAKE, 64, 128, FAKE, 128, 7, FAKE, 128, None) == 1
    # SwiGLU needs F = N / 2 a multiple of 128
    assert L.rib_gemm(FAKE, 64, 128, FAKE, 192, 2, FAKE, 96, None) == 1
    # misaligned operands
    assert L.rib_gemm(MISALIGNED, 64, 128, FAKE, 128, 0, FAKE, 128, None) == 3
    assert L.rib_gemm(FAKE, 64, 128, FAKE, 128, 0, MISALIGNED, 128, None) == 3
    # QKV + RoPE + append beyond the cache capacity (engine.py:45-46)
    assert L.rib_gemm_qkv_rope(FAKE, 64, 128, FAKE, 16, 8, FAKE, FAKE, FAKE, 250, FAKE, 64, FAKE, 256,
                               None) == 2
    assert L.rib_rope_table(0, 0, 1e6, FAKE, None) == 1


def test_gemm_few_rows_rejects_bad_arguments(rib):
    """rib_gemm_small: 1-64 rows, K a multiple of 64, N of 128, BF16 or SwiGLU
    epilogue, a workspace of the stated size; checked before any launch."""
    import importlib
    G = importlib.import_module("roofline-inference_b200.gemm")
    L = G._L()
    ws = int(L.rib_gemm_small_workspace_bytes(64, 4096, 1024))
    assert ws > 0
    assert L.rib_gemm_small_workspace_bytes(65, 4096, 1024) == 0
    assert L.rib_gemm_small_workspace_bytes(64, 4000, 1024) == 0

    def call(M=64, K=1024, N=4096, epi=0, ldc=4096, nbytes=ws, A=FAKE, C=FAKE, wsp=FAKE):
        return L.rib_gemm_small(A, M, K, FAKE, N, epi, C, ldc, wsp, nbytes, None)
    assert call(M=0) == 1
    assert call(M=65) == 1
    assert call(K=96) == 1
    assert call(N=4000, ldc=4000) == 1
    assert call(epi=1) == 1               # FP32 output is not offered
    assert call(ldc=100) == 1
    assert call(nbytes=ws - 16) == 1
    assert call(wsp=None) == 1
    assert call(A=MISALIGNED) == 3
    assert call(C=MISALIGNED) == 3


def test_wait_limit_range_checked_on_host(rib):
    L = rib.load_library()
    assert L.rib_set_wait_limit_ns(10) == 1
    assert L.rib_set_wait_limit_ns(61_000_000_000) == 1
    assert L.rib_get_wait_limit_ns(None) == 1


def test_tp_prefill_exchange_rejects_bad_arguments(rib):
    """rib_tp_prefill_buffer_bytes / rib_gemm_tp_partial /
    rib_tp_reduce_add_rms: the buffer layout (flags, receive slots of
    ceil(rows / world) rows per source, BF16 gather rows) and the host-side
    checks, before any launch."""
    import importlib
    T = importlib.import_module("roofline-inference_b200.tp")
    L = rib.load_library()
    T._bind(L)
    H, rows, world = 1024, 4096, 2
    nbytes = int(L.rib_tp_prefill_buffer_bytes(world, rows, H))
    recv = world * ((rows + world - 1) // world) * H * 4
    assert nbytes == (256 + recv + 255) // 256 * 256 + rows * H * 2
    assert L.rib_tp_prefill_buffer_bytes(3, 37, 256) == (256 + 3 * 13 * 256 * 4 + 255) // 256 * 256 + 37 * 256 * 2
    for bad in [(0, rows, H), (9, rows, H), (world, 0, H), (world, rows, 768), (world, rows, 128),
                (world, rows, 4096)]:
        assert L.rib_tp_prefill_buffer_bytes(*bad) == 0, bad

    def ex(world=2, rank=0, rows_cap=rows, hidden=H, bufs=(FAKE * 16, FAKE * 32)):
        s = T._PrefillExchangeStruct()
        s.world, s.rank, s.rows_cap, s.hidden = world, rank, rows_cap, hidden
        for r, b in enumerate(bufs):
            s.buf[r] = b
        return ctypes.byref(s)

    assert L.rib_gemm_tp_partial(FAKE, rows + 1, 1024, FAKE, ex(), None) == 1       # more rows than the buffers
    assert L.rib_gemm_tp_partial(FAKE, 0, 1024, FAKE, ex(), None) == 1
    assert L.rib_gemm_tp_partial(FAKE, 64, 1024, FAKE, ex(rank=2), None) == 1
    assert L.rib_gemm_tp_partial(FAKE, 64, 1024, FAKE, ex(bufs=(FAKE * 16, 0)), None) == 1
    assert L.rib_gemm_tp_partial(FAKE, 64, 1024, FAKE, ex(bufs=(FAKE * 16, FAKE * 16 + 128)), None) == 3
    assert L.rib_gemm_tp_partial(FAKE, 64, 1024, FAKE, ex(hidden=768), None) == 1
    assert L.rib_gemm_tp_partial(FAKE, 64, 96, FAKE, ex(), None) == 1              # K not a multiple of 64
    assert L.rib_gemm_tp_partial(MISALIGNED, 64, 1024, FAKE, ex(), None) == 3
    assert L.rib_gemm_tp_partial(FAKE, 64, 1024, FAKE, None, None) == 1
    assert L.rib_tp_reduce_add_rms(ex(), 64, 0, FAKE, FAKE, FAKE, None) == 1          # epoch 0 is never valid
    assert L.rib_tp_reduce_add_rms(ex(), 64, 1, None, FAKE, FAKE, None) == 1
    assert L.rib_tp_reduce_add_rms(ex(), 64, 1, FAKE, FAKE, None, None) == 1          # a norm needs an output
    assert L.rib_tp_reduce_add_rms(ex(), rows + 1, 1, FAKE, None, None, None) == 1
    assert L.rib_tp_reduce_add_rms(ex(), 64, 1, MISALIGNED, None, None, None) == 3
    assert L.rib_tp_reduce_add_rms(ex(), 64, 1, FAKE, FAKE, MISALIGNED, None) == 3
