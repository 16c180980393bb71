"""Generates the committed golden fixtures in tests/golden/*.npz.

The reference's own tests (agent-test/v2/test_engine.py) draw their inputs
from mx.random and compare against MLX at run time, so no golden vector of
theirs survives without MLX.  These fixtures therefore hold seeded inputs and
the outputs of the independent FP64 numpy restatement (oracle/reference_np.py)
on the shapes those tests use, and the script refuses to write them unless
the C oracle (oracle/oracle.c) agrees.

Cases (shapes follow agent-test/v2/test_engine.py:62-99 and the single-layer
decode at context 512):
  rope_L{L}_off{off}   L, offset in {(1,0), (1,5000), (37,0), (64,300)}
  decode_ctx512        qkv of the new token at position 512, cache rows
                       0..511, norm+rope+append, decode over 513 keys
  prefill_{qL}x{kL}    (37,37) and (128,300); q scaled by 1.5 as in the
                       reference test
Run from the repository root:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import importlib
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from oracle import oracle as coracle  # noqa: E402
from oracle import reference_np as ref  # noqa: E402

wl = importlib.import_module("roofline-inference_b200.workloads")


def u16(t):
    return t.contiguous().view(dtype=__import__("torch").int16).numpy().view(np.uint16)


def rope_case(L, off, seed):
    qkv, qw, kw = wl.prefill_qkv(L, seed)
    Lp = (L + 31) // 32 * 32 if L > 1 else 1
    Q, KV = ref.qk_norm_rope(u16(qkv), u16(qw), u16(kw), off, 16, 8, 1e6, Lp)
    Qc, KVc = coracle.qk_norm_rope(u16(qkv), u16(qw), u16(kw), off, 16, 8, 1e6, Lp)
    dq = np.abs(ref.bf16_to_f32(Q) - ref.bf16_to_f32(Qc)).max()
    assert dq <= 1.6e-2, dq
    assert np.array_equal(KV[1], KVc[1])
    np.savez_compressed(HERE / f"rope_L{L}_off{off}.npz", qkv=u16(qkv), qw=u16(qw), kw=u16(kw),
                        offset=off, Lp=Lp, Q=Q, KV=KV)


def decode_case():
    st = wl.decode_step(512, seed=1)
    cache = u16(st.cache)  # [2, 8, cap, 128], rows 0..511 filled
    q, kv = ref.qk_norm_rope(u16(st.qkv)[None], u16(st.qw), u16(st.kw), st.pos, 16, 8, 1e6, 1)
    full = cache.copy()
    full[:, :, st.pos] = kv[:, :, 0]
    n = st.n
    out = ref.decode_attention(q[:, 0], full[0, :, :n], full[1, :, :n], wl.SCALE)
    of, ob = coracle.decode_attention(q[:, 0], full, n, wl.SCALE)
    assert np.abs(of - out).max() < 1e-5, np.abs(of - out).max()
    np.savez_compressed(HERE / "decode_ctx512.npz", qkv=u16(st.qkv), qw=u16(st.qw), kw=u16(st.kw),
                        cache_rows=cache[:, :, :st.pos], pos=st.pos, cap=cache.shape[2],
                        q=q[:, 0], k_new=kv[0, :, 0], v_new=kv[1, :, 0],
                        out=out.astype(np.float32), out_bf16=ref.f32_to_bf16(out.astype(np.float32)))


def prefill_case(qL, kL, seed):
    import torch
    K = wl.randn_bf16((8, kL, 128), seed * 3 + 1)
    V = wl.randn_bf16((8, kL, 128), seed * 3 + 2)
    q = wl.randn_bf16((16, qL, 128), seed * 3 + 3, scale=1.5)
    qLp = (qL + 31) // 32 * 32
    Q = torch.zeros((16, qLp, 128), dtype=torch.bfloat16)
    Q[:, :qL] = q
    out = ref.prefill_attention(u16(Q), u16(K), u16(V), qL, kL, wl.SCALE)
    oc = coracle.prefill_attention(u16(Q), u16(K), u16(V), qL, kL, wl.SCALE)
    assert np.abs(oc - out).max() < 1e-5, np.abs(oc - out).max()
    np.savez_compressed(HERE / f"prefill_{qL}x{kL}.npz", Q=u16(Q), K=u16(K), V=u16(V), qL=qL,
                        kL=kL, out=out.astype(np.float32))


def main():
    for i, (L, off) in enumerate([(1, 0), (1, 5000), (37, 0), (64, 300)]):
        rope_case(L, off, seed=10 + i)
    decode_case()
    prefill_case(37, 37, seed=13)
    prefill_case(128, 300, seed=14)
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
