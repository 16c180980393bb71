"""CPU: the oracle against the committed golden fixtures and against the
independent FP64 numpy restatement, plus closed-form properties."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import bf16f, load_golden


@pytest.mark.parametrize("name", ["rope_L1_off0", "rope_L1_off5000", "rope_L37_off0",
                                  "rope_L64_off300"])
def test_rope_oracle_matches_golden(oracle, name):
    z = load_golden(name)
    Q, KV = oracle.qk_norm_rope(z["qkv"], z["qw"], z["kw"], int(z["offset"]), 16, 8, 1e6,
                                int(z["Lp"]))
    assert np.array_equal(Q, z["Q"])
    assert np.array_equal(KV, z["KV"])
    L = KV.shape[2]
    assert not Q[:, L:].any()  # pad rows exactly zero (agent-test/v2/test_engine.py:73)


def test_decode_oracle_matches_golden(oracle):
    z = load_golden("decode_ctx512")
    pos, cap = int(z["pos"]), int(z["cap"])
    q, kv = oracle.qk_norm_rope(z["qkv"][None], z["qw"], z["kw"], pos, 16, 8, 1e6, 1)
    assert np.array_equal(q[:, 0], z["q"])
    assert np.array_equal(kv[0, :, 0], z["k_new"]) and np.array_equal(kv[1, :, 0], z["v_new"])
    cache = np.zeros((2, 8, cap, 128), np.uint16)
    cache[:, :, :pos] = z["cache_rows"]
    cache[:, :, pos] = kv[:, :, 0]
    of, ob = oracle.decode_attention(q[:, 0], cache, pos + 1, 128 ** -0.5)
    assert np.abs(of - z["out"]).max() < 1e-5
    # one BF16 rounding of the same value: differs at most where the FP32
    # result sits on a rounding boundary
    assert (ob != z["out_bf16"]).mean() < 1e-3


@pytest.mark.parametrize("name", ["prefill_37x37", "prefill_128x300"])
def test_prefill_oracle_matches_golden(oracle, name):
    z = load_golden(name)
    out = oracle.prefill_attention(z["Q"], z["K"], z["V"], int(z["qL"]), int(z["kL"]),
                                   128 ** -0.5)
    assert np.abs(out - z["out"]).max() < 1e-5


@pytest.mark.parametrize("L,offset", [(5, 32760), (3, 0), (2, 123456)])
def test_rope_oracle_vs_numpy(oracle, ref_np, wl, L, offset):
    from conftest import u16
    qkv, qw, kw = wl.prefill_qkv(L, seed=L + offset)
    a = oracle.qk_norm_rope(u16(qkv), u16(qw), u16(kw), offset, 16, 8, 1e6, L)
    b = ref_np.qk_norm_rope(u16(qkv), u16(qw), u16(kw), offset, 16, 8, 1e6, L)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


@pytest.mark.parametrize("n", [1, 2, 33, 700])
def test_decode_oracle_vs_numpy(oracle, ref_np, wl, n):
    from conftest import u16
    st = wl.decode_step(n, seed=n)
    cache = u16(st.cache)
    q = u16(wl.randn_bf16((16, 128), seed=n + 99))
    of, _ = oracle.decode_attention(q, cache, n, wl.SCALE)
    ex = ref_np.decode_attention(q, cache[0, :, :n], cache[1, :, :n], wl.SCALE)
    assert np.abs(of - ex).max() < 1e-5


def test_decode_single_key_returns_v(oracle, wl):
    """softmax over one key is 1, so the output is that key's V row exactly."""
    from conftest import u16
    st = wl.decode_step(1, seed=5)
    cache = u16(st.cache)
    q = u16(wl.randn_bf16((16, 128), seed=6))
    of, ob = oracle.decode_attention(q, cache, 1, wl.SCALE)
    v = cache[1, :, 0]  # [8, 128]
    assert np.array_equal(ob, np.repeat(v, 2, axis=0))


def test_prefill_first_row_sees_one_key(oracle, wl):
    """With qL == kL, query 0 sees only key 0 (bottom-right alignment)."""
    from conftest import u16
    K = u16(wl.randn_bf16((8, 64, 128), seed=1))
    V = u16(wl.randn_bf16((8, 64, 128), seed=2))
    Q = u16(wl.randn_bf16((16, 64, 128), seed=3))
    out = oracle.prefill_attention(Q, K, V, 64, 64, wl.SCALE)
    expect = np.concatenate([bf16f(V[h // 2, 0]) for h in range(16)])
    assert np.allclose(out[0], expect, atol=0, rtol=0)


def test_prefill_offset_rows_match_decode(oracle, wl):
    """Bottom-right alignment: the last query row of a prefill with qL < kL
    equals a decode over all kL keys."""
    from conftest import u16
    kL, qL = 300, 17
    st = wl.decode_step(kL, seed=8)
    cache = u16(st.cache)
    Q = u16(wl.randn_bf16((16, 32, 128), seed=9))
    out = oracle.prefill_attention(Q, cache[0], cache[1], qL, kL, wl.SCALE)
    of, _ = oracle.decode_attention(Q[:, qL - 1], cache, kL, wl.SCALE)
    assert np.abs(out[qL - 1] - of.reshape(-1)).max() < 1e-6
