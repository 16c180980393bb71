"""CPU: host-side logic -- the Cache interface of the reference
(agent-test/v2/engine.py:33-55), wrapper argument checks (they raise before
anything reaches the library) and the workload bookkeeping."""
from __future__ import annotations

import pytest
import torch


def test_cache_capacity_rounding_and_views(rib):
    c = rib.Cache(3, 8, 128, 300, device="cpu")
    assert c.capacity == 512 and c.offset == 0
    assert len(c.kv) == 3 and tuple(c.kv[0].shape) == (2, 8, 512, 128)
    kv = torch.randn(2, 8, 5, 128).to(torch.bfloat16)
    buf = c.update(1, kv)
    assert buf.data_ptr() == c.kv[1].data_ptr()
    K, V = c.views(1, 5)
    assert tuple(K.shape) == (1, 8, 5, 128)
    assert torch.equal(K[0], kv[0]) and torch.equal(V[0], kv[1])
    assert not c.kv[0].any() and not c.kv[2].any()
    # layers share one allocation, each layer contiguous
    assert c.kv[1].is_contiguous()
    assert c.kv[1].data_ptr() - c.kv[0].data_ptr() == 2 * 8 * 512 * 128 * 2


def test_cache_capacity_exceeded(rib):
    """engine.py:45-46 and test_engine.py:161-163."""
    c = rib.Cache(1, 8, 128, 4, device="cpu")
    assert c.capacity == 256
    with pytest.raises(ValueError, match="KV capacity exceeded"):
        c.update(0, torch.zeros((2, 8, 300, 128), dtype=torch.bfloat16))
    c.offset = 250
    with pytest.raises(ValueError, match="KV capacity exceeded"):
        c.update(0, torch.zeros((2, 8, 7, 128), dtype=torch.bfloat16))
    c.update(0, torch.zeros((2, 8, 6, 128), dtype=torch.bfloat16))


def test_wrappers_reject_cpu_and_wrong_dtype(rib):
    qkv = torch.zeros(4096, dtype=torch.bfloat16)
    w = torch.ones(128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        rib.qk_norm_rope(qkv, w, w, 0, 16, 8, 1e6)
    with pytest.raises(ValueError, match="bfloat16"):
        rib.qk_norm_rope(qkv.float(), w, w, 0, 16, 8, 1e6)
    with pytest.raises(ValueError):
        rib.decode_attention(torch.zeros(1, 16, 1, 128, dtype=torch.bfloat16),
                             torch.zeros(2, 8, 256, 128, dtype=torch.bfloat16), 10, 0.088)
    with pytest.raises(ValueError):
        rib.attention(torch.zeros(16, 32, 128, dtype=torch.bfloat16),
                      torch.zeros(1, 8, 256, 128, dtype=torch.bfloat16),
                      torch.zeros(1, 8, 256, 128, dtype=torch.bfloat16), 32, 32, 0.088)


def test_workload_counts(wl):
    L = 32768
    assert wl.prefill_flops(L) == 4096 * L * (L + 1)
    assert wl.decode_kv_bytes(32769) == 4096 * 32769
    # qL < kL: each query sees off + i + 1 keys
    assert wl.prefill_flops(2, 5) == 4 * 16 * 128 * (4 + 5)
    assert wl.round_cap(32769) == 33024


def test_seeded_inputs_are_deterministic(wl):
    a = wl.decode_step(64, seed=3)
    b = wl.decode_step(64, seed=3)
    assert torch.equal(a.qkv, b.qkv) and torch.equal(a.cache, b.cache)
    assert a.n == 65 and not a.cache[:, :, 64:].any()
    lens = wl.ragged_lengths(64, 512, 32768, seed=0)
    assert len(lens) == 64 and min(lens) >= 512 and max(lens) <= 32768
    assert lens == wl.ragged_lengths(64, 512, 32768, seed=0)
