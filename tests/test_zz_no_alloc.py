"""GPU: decode attention through the entry point that allocates nothing.

rib_decode_attention_noalloc serves callers that cannot call cudaMalloc or
lend device scratch -- a host whose device memory belongs to another
allocator or to a fixed budget, or a language binding with no device
allocator of its own.  It keeps its split-KV scratch in a fixed 2 MiB array
inside the library.  This test calls it through the C ABI and checks it
against the workspace-taking entry point, twice in a row (the array keeps
the previous call's contents), and checks that a size beyond the array is
refused.  The file is named so that pytest collects it last."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import bf16f

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def test_noalloc_decode_matches_workspace_entry_point(rib, wl):
    L = rib.load_library()
    n = 8193
    st = wl.decode_step(n - 1, seed=21, device="cuda")
    cap = st.cache.shape[2]
    stream = torch.cuda.current_stream().cuda_stream
    outs = []
    for call in range(2):
        q = wl.randn_bf16((16, 128), seed=40 + call, device="cuda")
        want = rib.decode_attention(q, st.cache, n, wl.SCALE).reshape(16, 128)
        got = torch.full((16, 128), float("nan"), dtype=torch.bfloat16, device="cuda")
        status = L.rib_decode_attention_noalloc(q.data_ptr(), st.cache.data_ptr(), cap, n, 16, 8,
                                                wl.SCALE, got.data_ptr(), stream)
        assert status == 0, L.rib_last_error_string()
        torch.cuda.synchronize()
        d = np.abs(bf16f(got).astype(np.float64) - bf16f(want).astype(np.float64))
        assert d.max() <= MAX_ABS and d.mean() <= MEAN_ABS, (call, d.max(), d.mean())
        outs.append(got.clone())
    assert not torch.equal(outs[0], outs[1])  # two different queries, two answers


def test_noalloc_decode_rejects_sizes_beyond_static_scratch(rib):
    L = rib.load_library()
    fake = 0x10000  # aligned dummy address; the size check runs before any launch
    n = 2000000  # needs about 4 MiB of scratch at 8 KV heads
    status = L.rib_decode_attention_noalloc(fake, fake, n, n, 16, 8, 0.088, fake,
                                            torch.cuda.current_stream().cuda_stream)
    assert status == 1
    assert b"static scratch" in L.rib_last_error_string()
