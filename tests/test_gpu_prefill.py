"""GPU parity of the tcgen05/TMEM causal prefill attention kernel against the
oracle and the golden fixtures.

Shapes: the reference test's (qL, kL) pairs (agent-test/v2/test_engine.py:81-99,
q scaled by 1.5, cap rounded to 256), the prefill sweep L in {16, 64, 256,
1024, 4096, 32768} and ragged sizes that are not multiples of the 128-row tile.
Tolerance: contract max-abs <= 2e-2 and mean-abs <= 2e-3 against the FP32
oracle; in addition the error may exceed the error of rounding the exact
result to BF16 only by the BF16 rounding of P (P.V runs on BF16 P)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import from_u16, load_golden, parity_errors, u16

pytestmark = pytest.mark.gpu
MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def _assert_parity(out, exact, rows=None):
    o = out if rows is None else out[rows[0]:rows[1]]
    e = exact if rows is None else exact[rows[0]:rows[1]]
    err = parity_errors(o, e)
    print(f"prefill parity: {err}")
    assert err["max"] <= MAX_ABS and err["mean"] <= MEAN_ABS, err
    assert err["max"] <= 2.0 * err["floor_max"] + 1e-6, err


def _case(wl, qL, kL, seed, qscale=1.0):
    cap = wl.round_cap(kL)
    buf = torch.zeros((2, 8, cap, 128), dtype=torch.bfloat16, device="cuda")
    buf[:, :, :kL] = wl.randn_bf16((2, 8, kL, 128), seed=seed, device="cuda")
    qLp = (qL + 31) // 32 * 32
    Q = torch.zeros((16, qLp, 128), dtype=torch.bfloat16, device="cuda")
    Q[:, :qL] = wl.randn_bf16((16, qL, 128), seed=seed + 1, device="cuda", scale=qscale)
    return Q, buf


@pytest.mark.parametrize("name", ["prefill_37x37", "prefill_128x300"])
def test_prefill_golden(rib, name):
    z = load_golden(name)
    qL, kL = int(z["qL"]), int(z["kL"])
    Q, K, V = (from_u16(z[k], "cuda") for k in ("Q", "K", "V"))
    out = rib.attention(Q, K[None], V[None], qL, kL, 128 ** -0.5)
    torch.cuda.synchronize()
    assert tuple(out.shape) == (qL, 16 * 128)
    _assert_parity(out, z["out"])


@pytest.mark.parametrize("qL,kL", [(37, 37), (128, 300), (1000, 1000), (512, 2600), (1, 1),
                                   (1, 700), (129, 129), (200, 4000)])
def test_prefill_reference_shapes(rib, wl, oracle, qL, kL):
    """agent-test/v2/test_engine.py:81-99 shapes plus single-row and ragged ones."""
    Q, buf = _case(wl, qL, kL, seed=qL * 7 + kL, qscale=1.5)
    out = rib.attention(Q, buf[0:1], buf[1:2], qL, kL, wl.SCALE)
    torch.cuda.synchronize()
    ref = oracle.prefill_attention(u16(Q), u16(buf[0]), u16(buf[1]), qL, kL, wl.SCALE)
    _assert_parity(out, ref)


@pytest.mark.parametrize("L", [16, 64, 256, 1024, 4096])
def test_prefill_sweep(rib, wl, oracle, L):
    """Config: causal prefill, Q/K/V BF16 N(0,1), positions 0..L-1."""
    Q, buf = _case(wl, L, L, seed=L)
    out = rib.attention(Q, buf[0:1], buf[1:2], L, L, wl.SCALE)
    torch.cuda.synchronize()
    ref = oracle.prefill_attention(u16(Q), u16(buf[0]), u16(buf[1]), L, L, wl.SCALE)
    _assert_parity(out, ref)


def test_prefill_32k_sampled_rows(rib, wl, oracle):
    """L = 32768: every row is computed on the GPU; the oracle checks the
    first, a middle and the last 128-row blocks (all 16 heads)."""
    L = 32768
    Q, buf = _case(wl, L, L, seed=3)
    out = rib.attention(Q, buf[0:1], buf[1:2], L, L, wl.SCALE)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    Qh, Kh, Vh = u16(Q), u16(buf[0]), u16(buf[1])
    for r0 in (0, 16384 - 64, L - 128):
        ref = oracle.prefill_attention(Qh, Kh, Vh, L, L, wl.SCALE, rows=(r0, r0 + 128))
        _assert_parity(out, ref, rows=(r0, r0 + 128))


def test_prefill_fused_pipeline(rib, wl, oracle):
    """qkv -> fused norm + RoPE + append into a Cache -> causal attention,
    the order Engine.prefill runs them (agent-test/v2/engine.py:111-124)."""
    L = 300
    qkv, qw, kw = wl.prefill_qkv(L, seed=5, device="cuda")
    cache = rib.Cache(1, 8, 128, L + 8, device="cuda")
    Lp = (L + 31) // 32 * 32
    Q = cache.append_qk_norm_rope(0, qkv, qw, kw, 16, 1e6, Lp)
    buf = cache.kv[0]
    out = rib.attention(Q, buf[0:1], buf[1:2], L, L, wl.SCALE)
    torch.cuda.synchronize()
    ref = oracle.prefill_attention(u16(Q), u16(buf[0]), u16(buf[1]), L, L, wl.SCALE)
    _assert_parity(out, ref)


def test_prefill_chunked_matches_single(rib, wl, oracle):
    """Chunked prefill with a cache offset (engine.py:176-182): the second
    chunk's queries attend to off + n keys with the bottom-right mask."""
    L1, L2 = 256, 200
    Q, buf = _case(wl, L1 + L2, L1 + L2, seed=9)
    full = rib.attention(Q, buf[0:1], buf[1:2], L1 + L2, L1 + L2, wl.SCALE)
    Q2 = torch.zeros((16, 224, 128), dtype=torch.bfloat16, device="cuda")
    Q2[:, :L2] = Q[:, L1:L1 + L2]
    part = rib.attention(Q2, buf[0:1], buf[1:2], L2, L1 + L2, wl.SCALE)
    torch.cuda.synchronize()
    d = (full[L1:].float() - part.float()).abs().max().item()
    assert d <= 2e-2, d


def test_prefill_device_status_clean(rib):
    from importlib import import_module
    assert import_module("roofline-inference_b200._lib").take_device_status() == 0
