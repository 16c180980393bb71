"""GPU parity of the fused QK-RMSNorm + RoPE (+ KV append) kernel against the
oracle, and against the reference's own Metal kernel through the golden
fixtures (its outputs, computed on the CPU by oracle/msl/runner.py).

Tolerances follow the reference test agent-test/v2/test_engine.py:62-78:
q/k within 3.2e-2 (one BF16 ulp at |x| <~ 4), V bit-exact, pad rows exactly
zero; the KV-cache write positions must be exact (rows outside
[offset, offset+L) untouched).  The kernel forms the RoPE angle in FP32 as the
reference does (kernels.py:134-138), so beyond the tolerance nearly every
element must be the same BF16 value as the oracle's and the reference
kernel's (differences come only from the order of the sum of squares)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import bf16f, from_u16, load_golden, u16

pytestmark = pytest.mark.gpu
TOL = 3.2e-2
MAX_DIFFER = 1e-3  # fraction of q/k elements allowed to differ by one ulp

ROPE_CASES = ["rope_L1_off0", "rope_L1_off5000", "rope_L1_off32768", "rope_L37_off0",
              "rope_L64_off300", "rope_L64_off32700"]


def _cmp_qk(got_u16, want_u16):
    d = np.abs(bf16f(got_u16) - bf16f(want_u16))
    assert d.max() <= TOL, d.max()
    assert (got_u16 != want_u16).mean() <= MAX_DIFFER, (got_u16 != want_u16).mean()


def _run_fixture(rib, z):
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
    return u16(q), u16(kv)


@pytest.mark.parametrize("name", ROPE_CASES)
def test_rope_golden(rib, name):
    z = load_golden(name)
    q, kv = _run_fixture(rib, z)
    # the oracle (FP32 angle, FP64 cos/sin)
    _cmp_qk(q, z["Q"])
    _cmp_qk(kv[0], z["KV"][0])
    assert np.array_equal(kv[1], z["KV"][1])
    # the reference's own kernel (agent-test/v2/kernels.py:116-146, 169-204)
    _cmp_qk(q, z["Q_ref"].reshape(q.shape))
    _cmp_qk(kv[0], z["KV_ref"][0].reshape(kv[0].shape))
    assert np.array_equal(kv[1], z["KV_ref"][1].reshape(kv[1].shape))


@pytest.mark.parametrize("pos", [0, 5000, 32768])
def test_rope_angle_counts(rib, wl, oracle, pos):
    """How many q/k elements the FP32 angle changes against an FP64 angle, at
    positions 0, 5000 and 32768: the kernel must agree with the FP32-angle
    oracle and differ from the FP64-angle one by what the oracles differ."""
    L = 64
    qkv, qw, kw = wl.prefill_qkv(L, seed=pos + 1)
    q, kv = rib.qk_norm_rope_prefill(qkv.cuda(), qw.cuda(), kw.cuda(), pos, 16, 8, 1e6, L)
    torch.cuda.synchronize()
    got = np.concatenate([u16(q).ravel(), u16(kv[0]).ravel()])
    a = oracle.qk_norm_rope(u16(qkv), u16(qw), u16(kw), pos, 16, 8, 1e6, L)
    b = oracle.qk_norm_rope(u16(qkv), u16(qw), u16(kw), pos, 16, 8, 1e6, L, angle_f64=True)
    f32 = np.concatenate([a[0].ravel(), a[1][0].ravel()])
    f64 = np.concatenate([b[0].ravel(), b[1][0].ravel()])
    n_f32, n_f64, n_or = int((got != f32).sum()), int((got != f64).sum()), int((f32 != f64).sum())
    print(f"rope angle counts pos={pos}: {got.size} q/k elements, kernel vs FP32-angle oracle "
          f"{n_f32}, vs FP64-angle oracle {n_f64}, FP32 vs FP64 oracles {n_or}")
    assert n_f32 <= MAX_DIFFER * got.size
    assert abs(n_f64 - n_or) <= n_f32 + 1


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
