"""CPU: host logic of the Qwen3 forward (config checks, weight layout, C-ABI
argument checks of the model kernels) and self-consistency of the numpy
model oracle.  No kernel is launched here."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import ROOT  # noqa: F401  (puts the repository on sys.path)

FAKE = 0x10000        # 16-byte aligned dummy device address; never dereferenced
MISALIGNED = 0x10008


@pytest.fixture(scope="module")
def mnp():
    from oracle import model_np
    return model_np


def tiny_config(rib, layers=2):
    return rib.Qwen3Config(num_layers=layers, hidden_size=256, num_heads=2, num_kv_heads=1,
                           intermediate_size=512, vocab_size=1000)


# ------------------------------------------------------------------ config / weights
def test_config_preconditions(rib):
    rib.QWEN3_0_6B.validate()
    assert rib.QWEN3_0_6B.q_dim == 2048 and rib.QWEN3_0_6B.kv_dim == 1024
    with pytest.raises(ValueError):
        rib.Qwen3Config(num_heads=16, num_kv_heads=4).validate()   # GQA factor must be 2
    with pytest.raises(ValueError):
        rib.Qwen3Config(hidden_size=1000).validate()               # GEMV K % 256
    with pytest.raises(ValueError):
        rib.Qwen3Config(head_dim=64).validate()


def test_random_weights_layout(rib):
    cfg = tiny_config(rib)
    w = rib.random_weights(cfg, seed=3)
    l0 = w.layers[0]
    assert tuple(l0["qkv"].shape) == (cfg.q_dim + 2 * cfg.kv_dim, cfg.hidden_size)
    assert tuple(l0["o"].shape) == (cfg.hidden_size, cfg.q_dim)
    assert tuple(l0["gu"].shape) == (2 * cfg.intermediate_size, cfg.hidden_size)
    assert tuple(l0["down"].shape) == (cfg.hidden_size, cfg.intermediate_size)
    assert tuple(w.embed.shape) == (cfg.vocab_size, cfg.hidden_size)
    assert all(t.dtype == torch.bfloat16 for t in l0.values())
    assert abs(float(l0["qkv"].float().std()) - 0.02) < 2e-3
    w2 = rib.random_weights(cfg, seed=3)
    assert torch.equal(w.layers[1]["down"], w2.layers[1]["down"])   # seeded


def test_engine_requires_cuda_weights(rib):
    w = rib.random_weights(tiny_config(rib), seed=0)
    with pytest.raises(ValueError):
        rib.Engine(w)


# ------------------------------------------------------------------ C-ABI checks
def test_model_entry_points_reject_bad_arguments(rib):
    L = rib.load_library()
    # gemv: K not a multiple of 256; residual epilogue without res; swiglu with odd N;
    # misaligned x
    assert L.rib_gemv(FAKE, 64, 100, FAKE, None, None, 0, 0, FAKE, None) == 1
    assert L.rib_gemv(FAKE, 64, 256, FAKE, None, None, 1, 0, FAKE, None) == 1
    assert L.rib_gemv(FAKE, 63, 256, FAKE, None, None, 2, 0, FAKE, None) == 1
    assert L.rib_gemv(FAKE, 64, 256, FAKE, None, FAKE, 1, 1, FAKE, None) == 1
    assert L.rib_gemv(FAKE, 64, 256, MISALIGNED, None, None, 0, 0, FAKE, None) == 3
    assert L.rib_gemv(FAKE, 64, 256, FAKE, None, None, 7, 0, FAKE, None) == 1
    # row kernels
    assert L.rib_add_rms(FAKE, FAKE, FAKE, 0, 1024, FAKE, FAKE, None) == 1
    assert L.rib_add_rms(FAKE, FAKE, FAKE, 4, 1020, FAKE, FAKE, None) == 1
    assert L.rib_rms_norm(FAKE, MISALIGNED, 4, 1024, FAKE, None) == 3
    assert L.rib_swiglu(FAKE, 4, 12, FAKE, None) == 1
    assert L.rib_embed(FAKE, 100, 1024, FAKE, 0, FAKE, None) == 1
    assert L.rib_embed(FAKE, 100, 1024, 0x10002, 3, FAKE, None) == 3
    # argmax and the device-offset append
    assert L.rib_argmax_workspace_bytes() >= 16
    assert L.rib_argmax_f32(FAKE, 0, FAKE, FAKE, None) == 1
    assert L.rib_argmax_f32(FAKE, 10, FAKE, 0x10004, None) == 3
    assert L.rib_qk_norm_rope_append_dev(FAKE, 1, FAKE, FAKE, None, 16, 8, 1e6, 1, FAKE, FAKE, 256,
                                         None) == 1
    assert L.rib_qk_norm_rope_append_dev(FAKE, 1, FAKE, FAKE, 0x10002, 16, 8, 1e6, 1, FAKE, FAKE, 256,
                                         None) == 3


# ------------------------------------------------------------------ oracle
def _u16(rng, shape, scale=1.0):
    from oracle.reference_np import f32_to_bf16
    return f32_to_bf16((rng.standard_normal(shape) * scale).astype(np.float32))


def test_oracle_rms_norm_closed_form(mnp):
    from oracle.reference_np import bf16_to_f32, f32_to_bf16
    x = f32_to_bf16(np.full(256, 2.0, np.float32))
    w = f32_to_bf16(np.full(256, 0.5, np.float32))
    # mean(x^2) = 4, inv = 1/2 (eps negligible at BF16), x*inv = 1, w*1 = 0.5
    np.testing.assert_array_equal(bf16_to_f32(mnp.rms_norm(x, w)), np.full(256, 0.5, np.float32))


def test_oracle_gemv_epilogues_compose(mnp):
    from oracle.reference_np import bf16_to_f32, f32_to_bf16
    rng = np.random.default_rng(0)
    W, x, nw, res = _u16(rng, (64, 256), 0.05), _u16(rng, 256), _u16(rng, 256, 0.1), _u16(rng, 64)
    plain = mnp.gemv(W, x, nw=nw)
    np.testing.assert_array_equal(plain, mnp.matmul(mnp.rms_norm(x, nw)[None], W)[0])
    r = mnp.gemv(W, x, res=res)
    np.testing.assert_array_equal(r, f32_to_bf16(bf16_to_f32(res) + bf16_to_f32(mnp.gemv(W, x))))
    s = mnp.gemv(W, x, swiglu_epi=True)
    np.testing.assert_array_equal(s, mnp.swiglu(mnp.gemv(W, x)))
    lg = mnp.gemv(W, x, out_float=True)
    assert lg.dtype == np.float32 and mnp.argmax(lg) == int(np.argmax(lg))


def test_oracle_add_rms(mnp):
    rng = np.random.default_rng(1)
    a, b, w = _u16(rng, (3, 256)), _u16(rng, (3, 256)), _u16(rng, 256)
    r, n = mnp.add_rms(a, b, w)
    from oracle.reference_np import bf16_to_f32, f32_to_bf16
    np.testing.assert_array_equal(r, f32_to_bf16(bf16_to_f32(a) + bf16_to_f32(b)))
    np.testing.assert_array_equal(n, mnp.rms_norm(r, w))


def test_oracle_decode_continues_prefill(rib, mnp):
    """Prefill of n tokens then one decode step gives the logits of a prefill
    of n+1 tokens: the cache, positions and causal structure agree."""
    cfg = tiny_config(rib)
    w = mnp.weights_to_numpy(rib.random_weights(cfg, seed=5))
    toks = np.random.default_rng(2).integers(0, cfg.vocab_size, 19)
    a = mnp.Qwen3Oracle(w, cfg, 64)
    a.prefill(toks[:18])
    la = a.decode(toks[18])
    b = mnp.Qwen3Oracle(w, cfg, 64)
    lb = b.prefill(toks)
    assert a.offset == b.offset == 19
    np.testing.assert_allclose(la, lb, atol=2e-2 * np.abs(lb).max())
    assert np.abs(la - lb).mean() < 2e-3 * np.abs(lb).max()


def test_batched_entry_points_reject_bad_arguments(rib):
    L = rib.load_library()
    # GQA factor, misaligned caps, null pointers, empty batch
    assert L.rib_decode_attention_ragged(FAKE, FAKE, FAKE, FAKE, 2, 100, 15, 8, 0.09, FAKE, FAKE, 1 << 20,
                                         None) == 1
    assert L.rib_decode_attention_ragged(FAKE, FAKE, 0x10002, FAKE, 2, 100, 16, 8, 0.09, FAKE, FAKE, 1 << 20,
                                         None) == 3
    assert L.rib_qk_norm_rope_append_batched(FAKE, FAKE, FAKE, None, FAKE, FAKE, 2, 16, 8, 1e6, FAKE,
                                             None) == 1
    assert L.rib_qk_norm_rope_append_batched(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 0, 16, 8, 1e6, FAKE,
                                             None) == 1
    assert L.rib_argmax_rows_f32(FAKE, 0, 10, FAKE, None) == 1
    assert L.rib_argmax_rows_f32(0x10002, 2, 10, FAKE, None) == 3


# ------------------------------------------------------------------ tensor-parallel weight split
@pytest.mark.parametrize("world", [2, 4])
def test_tp_shard_layer_reconstructs_products(rib, world):
    """The per-rank slices of shard_layer rebuild every projection: row
    slices concatenate to the full output, column slices sum to it."""
    import importlib
    tp = importlib.import_module("roofline-inference_b200.tp")
    sharding = importlib.import_module("roofline-inference_b200.sharding")
    cfg = rib.Qwen3Config(num_layers=1, hidden_size=256, num_heads=8, num_kv_heads=4,
                          intermediate_size=1024, vocab_size=1000)
    layer = {k: v.double() for k, v in rib.random_weights(cfg, seed=9).layers[0].items()}
    F = cfg.intermediate_size
    g = torch.Generator().manual_seed(1)
    o_in = torch.randn(cfg.q_dim, generator=g, dtype=torch.float64)
    a_in = torch.randn(F, generator=g, dtype=torch.float64)
    x = torch.randn(cfg.hidden_size, generator=g, dtype=torch.float64)
    o_sum, d_sum, gates, ups = 0, 0, [], []
    for r in range(world):
        h0, h1 = sharding.head_range(r, world, cfg.num_kv_heads)
        f0, f1 = tp.split_range(F, r, world)
        s = tp.shard_layer(layer, h0, h1, f0, f1, cfg.num_heads, cfg.num_kv_heads)
        o_sum = o_sum + s["o"] @ o_in[2 * h0 * 128:2 * h1 * 128]
        d_sum = d_sum + s["down"] @ a_in[f0:f1]
        gu = s["gu"] @ x
        gates.append(gu[:f1 - f0])
        ups.append(gu[f1 - f0:])
    torch.testing.assert_close(o_sum, layer["o"] @ o_in)
    torch.testing.assert_close(d_sum, layer["down"] @ a_in)
    full = layer["gu"] @ x
    torch.testing.assert_close(torch.cat(gates), full[:F])
    torch.testing.assert_close(torch.cat(ups), full[F:])
    with pytest.raises(ValueError):
        tp.split_range(1000, 0, 3)


def test_tp_entry_points_reject_bad_arguments(rib):
    import ctypes
    import importlib
    tp = importlib.import_module("roofline-inference_b200.tp")
    L = rib.load_library()
    tp._bind(L)
    assert L.rib_tp_buffer_bytes(2, 256) == 2 * 2 * 256 * 8
    assert L.rib_tp_buffer_bytes(9, 256) == 0 and L.rib_tp_buffer_bytes(2, 6) == 0
    ex = tp._TpExchangeStruct()
    ex.world, ex.rank, ex.slot = 2, 0, 256
    ex.buf[0], ex.buf[1], ex.epoch, ex.done = 0x10000, 0x20000, 0x30000, 0x30008
    # partial epilogue wider than the slot; in_sum without x_out; misaligned peer buffer; bad rank
    assert L.rib_gemv_tp(FAKE, 512, 256, FAKE, None, 3, 0, None, ctypes.byref(ex), 0, None, None) == 1
    assert L.rib_gemv_tp(FAKE, 64, 256, FAKE, None, 0, 0, FAKE, ctypes.byref(ex), 1, None, None) == 1
    ex.buf[1] = 0x20010
    assert L.rib_gemv_tp(FAKE, 64, 256, FAKE, None, 3, 0, None, ctypes.byref(ex), 0, None, None) == 3
    ex.buf[1], ex.rank = 0x20000, 2
    assert L.rib_argmax_f32_tp(FAKE, 100, 0, FAKE, FAKE, ctypes.byref(ex), None) == 1
    # a residual epilogue has no tensor-parallel form
    ex.rank = 0
    assert L.rib_gemv_tp(FAKE, 64, 256, FAKE, None, 1, 0, FAKE, ctypes.byref(ex), 0, None, None) == 1


def test_gemv_wide_flag_keeps_the_argument_checks(rib):
    """RIB_GEMV_WIDE is a launch hint OR-ed into epi: the epilogue under it is
    checked as without it."""
    L = rib.load_library()
    wide = 0x100
    assert L.rib_gemv(FAKE, 64, 256, FAKE, None, None, 7 | wide, 0, FAKE, None) == 1   # unknown epilogue
    assert L.rib_gemv(FAKE, 64, 256, FAKE, None, None, 1 | wide, 0, FAKE, None) == 1   # residual without res
    assert L.rib_gemv(FAKE, 63, 256, FAKE, None, None, 2 | wide, 0, FAKE, None) == 1   # odd N for SwiGLU


def test_fused_decode_entry_rejects_bad_arguments(rib):
    """rib_decode_attention_qkv argument checks (no launch): GQA factor, null
    pointers, non-positive base, misaligned qkv, capacity below max_n."""
    L = rib.load_library()
    args = dict(qkv=FAKE, qw=FAKE, kw=FAKE, base=1e6, ptrs=FAKE, lens=FAKE, B=1, max_n=100, cap=256, nq=16,
                nkv=8, scale=0.09, out=FAKE, ws=FAKE, wsb=1 << 20)

    def call(**kw):
        a = dict(args, **kw)
        return L.rib_decode_attention_qkv(a["qkv"], a["qw"], a["kw"], a["base"], a["ptrs"], a["lens"], a["B"],
                                          a["max_n"], a["cap"], a["nq"], a["nkv"], a["scale"], a["out"], a["ws"],
                                          a["wsb"], None)
    assert call(nq=15) == 1
    assert call(qkv=None) == 1
    assert call(base=0.0) == 1
    assert call(B=0) == 1
    assert call(qkv=MISALIGNED) == 3
    assert call(lens=0x10002) == 3
    assert call(max_n=300) == 2          # RIB_ECAPACITY: max_n above the capacity


def test_fused_decode_wrapper_checks_shapes(rib):
    """decode_attention_qkv refuses CPU tensors and a qkv width that does not
    match the caches' KV heads before any launch."""
    qkv = torch.zeros((1, 32 * 128), dtype=torch.bfloat16)
    w = torch.ones(128, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        rib.decode_attention_qkv(qkv, w, w, 1e6, torch.zeros((1, 2, 8, 256, 128), dtype=torch.bfloat16), [5],
                                 0.09)


def test_local_prefill_exchange_checks_its_geometry():
    """tp.PrefillExchange(local=True) needs no process group, and a geometry
    the kernels do not take (hidden not 256/512/1024/2048, no rows) is refused
    on the host before any buffer is made."""
    import importlib
    T = importlib.import_module("roofline-inference_b200.tp")
    for hidden, rows in [(768, 4096), (4096, 4096), (1024, 0)]:
        with pytest.raises(ValueError, match="unsupported prefill exchange geometry"):
            T.PrefillExchange(hidden, rows, "cpu", local=True)


def test_row_parallel_oracle_matches_the_unsplit_projection():
    """The oracle of the tensor-parallel prefill exchange: splitting K over 1,
    2 or 4 ranks and adding the FP32 partials in rank order gives the unsplit
    projection's BF16 residual add and RMSNorm up to one BF16 step (the FP32
    sums differ only in order)."""
    from oracle import model_np
    from oracle.reference_np import bf16_to_f32, f32_to_bf16
    rng = np.random.default_rng(3)
    m, K, N = 7, 512, 256
    x = f32_to_bf16(rng.standard_normal((m, K)).astype(np.float32))
    W = f32_to_bf16((rng.standard_normal((N, K)) * K ** -0.5).astype(np.float32))
    h = f32_to_bf16(rng.standard_normal((m, N)).astype(np.float32))
    w = f32_to_bf16((1.0 + 0.1 * rng.standard_normal(N)).astype(np.float32))
    full_res, full_x = model_np.add_rms(h, model_np.matmul(x, W), w)
    for world in (1, 2, 4):
        k = K // world
        parts = [(x[:, r * k:(r + 1) * k], W[:, r * k:(r + 1) * k]) for r in range(world)]
        res, xn = model_np.row_parallel_add_rms(parts, h, w)
        for got, want in ((res, full_res), (xn, full_x)):
            g, f = bf16_to_f32(got).astype(np.float64), bf16_to_f32(want).astype(np.float64)
            assert np.all(np.abs(g - f) <= 2.0 ** -6 * np.abs(f) + 2.0 ** -7 * np.abs(f).max(-1, keepdims=True))
        if world == 1:
            assert np.array_equal(res, full_res) and np.array_equal(xn, full_x)
        res_only, none = model_np.row_parallel_add_rms(parts, h)
        assert none is None and np.array_equal(res_only, res)
