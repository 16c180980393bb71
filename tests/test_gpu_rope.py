"""GPU parity of the fused QK-RMSNorm + RoPE (+ KV append) kernel against the
oracle and the golden fixtures.

Tolerances follow the reference test agent-test/v2/test_engine.py:62-78:
q/k within 3.2e-2 (one BF16 ulp at |x| <~ 4), V bit-exact, pad rows exactly
zero; the KV-cache write positions must be exact (rows outside
[offset, offset+L) untouched)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import bf16f, from_u16, load_golden, u16

pytestmark = pytest.mark.gpu
TOL = 3.2e-2


def _cmp_qk(got_u16, want_u16):
    d = np.abs(bf16f(got_u16) - bf16f(want_u16))
    assert d.max() <= TOL, d.max()
    # the angle is evaluated to full FP32 accuracy, so nearly every element
    # rounds to the same BF16 value as the FP64 oracle
    assert (got_u16 != want_u16).mean() < 0.02


@pytest.mark.parametrize("name", ["rope_L1_off0", "rope_L1_off5000", "rope_L37_off0",
                                  "rope_L64_off300"])
def test_rope_golden(rib, name):
    z = load_golden(name)
    dev = "cuda"
    qkv, qw, kw = (from_u16(z[k], dev) for k in ("qkv", "qw", "kw"))
    off, Lp = int(z["offset"]), int(z["Lp"])
    L = qkv.shape[0]
    if L == 1:
        q, kv = rib.qk_norm_rope(qkv[0], qw, kw, off, 16, 8, 1e6)
        assert tuple(q.shape) == (1, 16, 1, 128) and tuple(kv.shape) == (2, 8, 1, 128)
        q = q[0]
    else:
        q, kv = rib.qk_norm_rope_prefill(qkv, qw, kw, off, 16, 8, 1e6, Lp)
        assert tuple(q.shape) == (16, Lp, 128) and tuple(kv.shape) == (2, 8, L, 128)
        assert not q[:, L:].any()
    torch.cuda.synchronize()
    _cmp_qk(u16(q), z["Q"])
    _cmp_qk(u16(kv[0]), z["KV"][0])
    assert np.array_equal(u16(kv[1]), z["KV"][1])


def test_rope_position_tensor_argument(rib, wl):
    """pos may be a 1-element int32 tensor, as the engine passes it (engine.py:148)."""
    st = wl.decode_step(0, seed=2, device="cuda")
    a, _ = rib.qk_norm_rope(st.qkv, st.qw, st.kw, 777, 16, 8, 1e6)
    b, _ = rib.qk_norm_rope(st.qkv, st.qw, st.kw, torch.tensor([777], dtype=torch.int32,
                                                                 device="cuda"), 16, 8, 1e6)
    assert torch.equal(a, b)


@pytest.mark.parametrize("L,offset", [(1, 32768), (1, 0), (37, 100), (256, 4000), (4096, 0),
                                      (32768, 0)])
def test_append_matches_oracle_and_writes_exact_rows(rib, wl, oracle, L, offset):
    qkv, qw, kw = wl.prefill_qkv(L, seed=L + offset)
    cap = wl.round_cap(offset + L + 3)
    # sentinel-filled cache: every row outside [offset, offset+L) must survive
    cache = wl.randn_bf16((2, 8, cap, 128), seed=11, device="cuda")
    before = cache.clone()
    qkv_d, qw_d, kw_d = qkv.cuda(), qw.cuda(), kw.cuda()
    Lp = (L + 31) // 32 * 32
    Q = rib.qk_norm_rope_append(qkv_d, qw_d, kw_d, offset, 16, 8, 1e6, cache, Lp)
    torch.cuda.synchronize()
    Qo, KVo = oracle.qk_norm_rope(u16(qkv), u16(qw), u16(kw), offset, 16, 8, 1e6, Lp)
    _cmp_qk(u16(Q), Qo)
    got = u16(cache)
    _cmp_qk(got[0, :, offset:offset + L], KVo[0])
    assert np.array_equal(got[1, :, offset:offset + L], KVo[1])
    keep = np.ones(cap, bool)
    keep[offset:offset + L] = False
    assert np.array_equal(got[:, :, keep], u16(before)[:, :, keep])
    assert not Q[:, L:].any()


def test_append_capacity_exceeded(rib, wl):
    qkv, qw, kw = wl.prefill_qkv(40, seed=1, device="cuda")
    cache = torch.zeros((2, 8, 256, 128), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="KV capacity exceeded"):
        rib.qk_norm_rope_append(qkv, qw, kw, 230, 16, 8, 1e6, cache)
    c = rib.Cache(2, 8, 128, 256, device="cuda")
    c.offset = 250
    with pytest.raises(ValueError, match="KV capacity exceeded"):
        c.append_qk_norm_rope(0, qkv, qw, kw, 16, 1e6)
