"""Generates the committed golden fixtures in tests/golden/*.npz.

The reference's own tests (agent-test/v2/test_engine.py) draw their inputs
from mx.random and compare against MLX at run time, so no golden vector of
theirs survives without MLX.  The fixtures hold instead, on the shapes those
tests use:
  - outputs of the reference's own Metal kernels (qk_norm_rope,
    qk_norm_rope_prefill, attention, gemv, add_rms, skinny_matmul), run on the
    CPU by oracle/msl/runner.py: the reference's Python host code called
    unchanged with a stand-in mlx module, each kernel source compiled as C++
    against oracle/msl/shim.h (fields *_ref);
  - outputs of the oracle (oracle/reference_np.py, cross-checked against the
    C oracle oracle/oracle.c before anything is written).
Large inputs are not stored: they are regenerated from the recorded seeds by
the seeded generators of roofline-inference_b200/workloads.py and checked
against a stored SHA-256 of their bytes (field `inputs_sha256`).

Cases:
  rope_L{L}_off{off}    (1,0) (1,5000) (1,32768) (37,0) (64,300) (64,32700)
                        [test_engine.py:62-78 shapes, plus positions near 32k]
  decode_ctx512         new token at position 512: norm + RoPE + append,
                        decode over 513 keys
  prefill_{qL}x{kL}     (37,37) (128,300) with inputs; (1000,1000) (512,2600)
                        from seeds with a sample of rows; q scaled by 1.5
                        [test_engine.py:81-99]
  model_gemv_*, model_add_rms, model_skinny
                        the reference's GEMV epilogues (none / residual /
                        RMSNorm + SwiGLU / FP32 out), add_rms and the skinny
                        GEMM on seeded inputs [test_engine.py:22-49, 102-109]
Needs the reference checkout (REFERENCE_ROOT) and g++.  Run from the
repository root:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import importlib
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from oracle import oracle as coracle  # noqa: E402
from oracle import reference_np as ref  # noqa: E402
from oracle.msl import runner  # noqa: E402

wl = importlib.import_module("roofline-inference_b200.workloads")
SCALE = 128 ** -0.5


def u16(t):
    return t.contiguous().view(dtype=__import__("torch").int16).numpy().view(np.uint16)


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


# ------------------------------------------------------------------ inputs (also used by the tests)
def prefill_inputs(qL, kL, seed):
    """Q [16, qLp, 128] (q scaled by 1.5, pad rows zero), K, V [8, kL, 128] u16."""
    K = u16(wl.randn_bf16((8, kL, 128), seed * 3 + 1))
    V = u16(wl.randn_bf16((8, kL, 128), seed * 3 + 2))
    qLp = (qL + 31) // 32 * 32
    Q = np.zeros((16, qLp, 128), np.uint16)
    Q[:, :qL] = u16(wl.randn_bf16((16, qL, 128), seed * 3 + 3, scale=1.5))
    return Q, K, V


def model_inputs(N, K, seed):
    """W [N, K] (N(0, 0.02)), x [K], nw [K] (1 + 0.1 N(0, 1)), res [N] u16."""
    W = u16(wl.randn_bf16((N, K), seed * 5 + 1, scale=0.02))
    x = u16(wl.randn_bf16((K,), seed * 5 + 2))
    nw = u16((1.0 + 0.1 * wl.randn_bf16((K,), seed * 5 + 3).float()).bfloat16())
    res = u16(wl.randn_bf16((N,), seed * 5 + 4))
    return W, x, nw, res


def _cap_buf(K, V, kL):
    cap = wl.round_cap(kL)
    buf = np.zeros((2, 8, cap, 128), np.uint16)
    buf[0, :, :kL], buf[1, :, :kL] = K, V
    return buf


# ------------------------------------------------------------------ cases
def rope_case(L, off, seed):
    qkv, qw, kw = wl.prefill_qkv(L, seed)
    Lp = (L + 31) // 32 * 32 if L > 1 else 1
    Q, KV = ref.qk_norm_rope(u16(qkv), u16(qw), u16(kw), off, 16, 8, 1e6, Lp)
    Qc, KVc = coracle.qk_norm_rope(u16(qkv), u16(qw), u16(kw), off, 16, 8, 1e6, Lp)
    assert np.array_equal(Q, Qc) and np.array_equal(KV, KVc)
    if L == 1:
        q_ref, kv_ref = runner.qk_norm_rope(u16(qkv)[0], u16(qw), u16(kw), off)
        Q_ref, KV_ref = q_ref.reshape(16, 1, 128), kv_ref.reshape(2, 8, 1, 128)
    else:
        Q_ref, KV_ref = runner.qk_norm_rope_prefill(u16(qkv), u16(qw), u16(kw), off, Lp=Lp)
    np.savez_compressed(HERE / f"rope_L{L}_off{off}.npz", qkv=u16(qkv), qw=u16(qw), kw=u16(kw),
                        offset=off, Lp=Lp, Q=Q, KV=KV, Q_ref=Q_ref, KV_ref=KV_ref)
    return (Q != Q_ref).sum() + (KV != KV_ref).sum()


def decode_case():
    st = wl.decode_step(512, seed=1)
    cache = u16(st.cache)  # [2, 8, cap, 128], rows 0..511 filled
    q, kv = ref.qk_norm_rope(u16(st.qkv)[None], u16(st.qw), u16(st.kw), st.pos, 16, 8, 1e6, 1)
    q_ref, kv_ref = runner.qk_norm_rope(u16(st.qkv), u16(st.qw), u16(st.kw), st.pos)
    full = cache.copy()
    full[:, :, st.pos] = kv[:, :, 0]
    n = st.n
    out = ref.decode_attention(q[:, 0], full[0, :, :n], full[1, :, :n], SCALE)
    of, ob = coracle.decode_attention(q[:, 0], full, n, SCALE)
    assert np.abs(of - out).max() < 1e-5, np.abs(of - out).max()
    np.savez_compressed(HERE / "decode_ctx512.npz", qkv=u16(st.qkv), qw=u16(st.qw), kw=u16(st.kw),
                        cache_rows=cache[:, :, :st.pos], pos=st.pos, cap=cache.shape[2],
                        q=q[:, 0], k_new=kv[0, :, 0], v_new=kv[1, :, 0],
                        q_ref=q_ref.reshape(16, 128), kv_ref=kv_ref.reshape(2, 8, 128),
                        out=out.astype(np.float32), out_bf16=ref.f32_to_bf16(out.astype(np.float32)))


def prefill_case(qL, kL, seed, rows=None):
    Q, K, V = prefill_inputs(qL, kL, seed)
    buf = _cap_buf(K, V, kL)
    out_ref = runner.attention(Q, buf[0:1], buf[1:2], qL, kL, SCALE)
    out = coracle.prefill_attention(Q, K, V, qL, kL, SCALE)
    if qL * kL <= 128 * 300:
        o64 = ref.prefill_attention(Q, K, V, qL, kL, SCALE)
        assert np.abs(o64 - out).max() < 1e-5, np.abs(o64 - out).max()
    # the reference kernel keeps P and V in FP32: its error is the BF16 floor
    e_ref = np.abs(ref.bf16_to_f32(out_ref) - out).max()
    floor = np.abs(ref.round_bf16(out) - out).max()
    assert e_ref <= floor + 1e-6, (e_ref, floor)
    name = f"prefill_{qL}x{kL}"
    if rows is None:
        np.savez_compressed(HERE / f"{name}.npz", Q=Q, K=K, V=V, qL=qL, kL=kL, seed=seed,
                            out=out.astype(np.float32), out_ref=out_ref)
    else:
        idx = np.concatenate([np.arange(a, b) for a, b in rows])
        np.savez_compressed(HERE / f"{name}.npz", qL=qL, kL=kL, seed=seed, rows=idx,
                            inputs_sha256=sha(Q, K, V), out=out[idx].astype(np.float32),
                            out_ref=out_ref[idx])
    return e_ref, floor


def model_cases():
    """Reference GEMV epilogues, add_rms and skinny GEMM on seeded inputs."""
    cases = {
        # name: (N, K, seed, kwargs)
        "model_gemv_qkv": (4096, 1024, 21, dict(nw=True)),
        "model_gemv_res": (1024, 2048, 22, dict(res=True)),
        "model_gemv_swiglu": (6144, 1024, 23, dict(nw=True, swiglu=True)),
        "model_gemv_down": (1024, 3072, 24, dict(res=True)),
        "model_gemv_logits": (2048, 1024, 25, dict(nw=True, out_float=True)),
    }
    for name, (N, K, seed, kw) in cases.items():
        W, x, nw, res = model_inputs(N, K, seed)
        y = runner.gemv(W, x, nw_u16=nw if kw.get("nw") else None, res_u16=res if kw.get("res") else None,
                        swiglu=kw.get("swiglu", False), out_float=kw.get("out_float", False))
        np.savez_compressed(HERE / f"{name}.npz", N=N, K=K, seed=seed, inputs_sha256=sha(W, x, nw, res),
                            nw=int(bool(kw.get("nw"))), res=int(bool(kw.get("res"))),
                            swiglu=int(kw.get("swiglu", False)), out_float=int(kw.get("out_float", False)),
                            y_ref=y)
    a = u16(wl.randn_bf16((37, 1024), 31))
    b = u16(wl.randn_bf16((37, 1024), 32))
    w = u16(wl.randn_bf16((1024,), 33))
    r, n = runner.add_rms(a, b, w)
    np.savez_compressed(HERE / "model_add_rms.npz", a=a, b=b, w=w, r_ref=r, n_ref=n)
    x = u16(wl.randn_bf16((20, 1024), 34))
    W = u16(wl.randn_bf16((1024, 1024), 35, scale=0.03))
    np.savez_compressed(HERE / "model_skinny.npz", M=20, N=1024, K=1024, seed_x=34, seed_w=35,
                        inputs_sha256=sha(x, W), y_ref=runner.skinny_matmul(x, W))


def main():
    if not runner.available():
        raise SystemExit("reference checkout not found: set REFERENCE_ROOT")
    for i, (L, off) in enumerate([(1, 0), (1, 5000), (1, 32768), (37, 0), (64, 300), (64, 32700)]):
        d = rope_case(L, off, seed=10 + i)
        print(f"rope L={L} off={off}: {d} elements differ from the reference kernel")
    decode_case()
    print("prefill 37x37", prefill_case(37, 37, seed=13))
    print("prefill 128x300", prefill_case(128, 300, seed=14))
    print("prefill 1000x1000", prefill_case(1000, 1000, seed=15, rows=[(0, 64), (480, 544), (936, 1000)]))
    print("prefill 512x2600", prefill_case(512, 2600, seed=16, rows=[(0, 64), (448, 512)]))
    model_cases()
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
