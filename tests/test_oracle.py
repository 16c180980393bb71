"""CPU: the oracle pinned against the reference's own Metal kernels (their
outputs on the CPU, stored in tests/golden/ by make_golden.py), against the
independent FP64 numpy restatement, and against closed-form properties."""
from __future__ import annotations

import importlib

import numpy as np
import pytest

from conftest import bf16f, load_golden

ROPE_CASES = ["rope_L1_off0", "rope_L1_off5000", "rope_L1_off32768", "rope_L37_off0",
              "rope_L64_off300", "rope_L64_off32700"]


def _golden_mod():
    return importlib.import_module("golden.make_golden")


@pytest.mark.parametrize("name", ROPE_CASES)
def test_rope_oracle_matches_reference_kernel(oracle, name):
    """agent-test/v2/kernels.py:116-146 / 169-204 run on the CPU: the oracle's
    FP32-angle rope reproduces the reference kernel's BF16 outputs except
    where the two FP32 sums of squares (simd_sum order vs FP64) put one
    element on the other side of a rounding boundary."""
    z = load_golden(name)
    Q, KV = oracle.qk_norm_rope(z["qkv"], z["qw"], z["kw"], int(z["offset"]), 16, 8, 1e6,
                                int(z["Lp"]))
    assert np.array_equal(Q, z["Q"]) and np.array_equal(KV, z["KV"])
    L = KV.shape[2]
    assert not Q[:, L:].any()  # pad rows exactly zero (agent-test/v2/test_engine.py:73)
    assert not z["Q_ref"][:, L:].any()
    assert np.array_equal(KV[1], z["KV_ref"][1])  # V copied bit for bit
    differ = int((Q[:, :L] != z["Q_ref"][:, :L]).sum() + (KV[0] != z["KV_ref"][0]).sum())
    assert differ <= max(1, 1e-4 * (Q[:, :L].size + KV[0].size)), differ
    d = np.abs(bf16f(Q) - bf16f(z["Q_ref"])).max()
    assert d <= 3.2e-2, d  # one BF16 ulp at |x| <~ 4 (test_engine.py:75-77)


@pytest.mark.parametrize("name", ["rope_L1_off5000", "rope_L1_off32768", "rope_L64_off32700"])
def test_rope_fp64_angle_moves_outputs(oracle, name):
    """The FP64 (idealised) angle is not the reference's: at large positions
    it changes a few percent of the BF16 outputs by one ulp."""
    z = load_golden(name)
    Qf, KVf = oracle.qk_norm_rope(z["qkv"], z["qw"], z["kw"], int(z["offset"]), 16, 8, 1e6,
                                  int(z["Lp"]), angle_f64=True)
    frac = float((Qf != z["Q_ref"]).mean())
    assert 0 < frac < 0.1, frac
    assert np.abs(bf16f(Qf) - bf16f(z["Q_ref"])).max() <= 3.2e-2


def test_decode_oracle_matches_golden(oracle):
    z = load_golden("decode_ctx512")
    pos, cap = int(z["pos"]), int(z["cap"])
    q, kv = oracle.qk_norm_rope(z["qkv"][None], z["qw"], z["kw"], pos, 16, 8, 1e6, 1)
    assert np.array_equal(q[:, 0], z["q"]) and np.array_equal(q[:, 0], z["q_ref"])
    assert np.array_equal(kv[0, :, 0], z["k_new"]) and np.array_equal(kv[1, :, 0], z["v_new"])
    assert np.array_equal(kv[:, :, 0], z["kv_ref"])
    cache = np.zeros((2, 8, cap, 128), np.uint16)
    cache[:, :, :pos] = z["cache_rows"]
    cache[:, :, pos] = kv[:, :, 0]
    of, ob = oracle.decode_attention(q[:, 0], cache, pos + 1, 128 ** -0.5)
    assert np.abs(of - z["out"]).max() < 1e-5
    # one BF16 rounding of the same value: differs at most where the FP32
    # result sits on a rounding boundary
    assert (ob != z["out_bf16"]).mean() < 1e-3


def _prefill_fixture(name):
    z = load_golden(name)
    qL, kL = int(z["qL"]), int(z["kL"])
    if "Q" in z:
        return z, z["Q"], z["K"], z["V"], None
    Q, K, V = _golden_mod().prefill_inputs(qL, kL, int(z["seed"]))
    assert _golden_mod().sha(Q, K, V) == str(z["inputs_sha256"]), "seeded generator changed"
    return z, Q, K, V, z["rows"]


@pytest.mark.parametrize("name", ["prefill_37x37", "prefill_128x300", "prefill_1000x1000",
                                  "prefill_512x2600"])
def test_prefill_oracle_matches_reference_kernel(oracle, name):
    """agent-test/v2/attention.py:18-185 run on the CPU (FP32 P and V): its
    output is the FP32 oracle rounded once to BF16, to within FP32 noise."""
    z, Q, K, V, rows = _prefill_fixture(name)
    qL, kL = int(z["qL"]), int(z["kL"])
    out = oracle.prefill_attention(Q, K, V, qL, kL, 128 ** -0.5)
    if rows is not None:
        out = out[rows]
    assert np.abs(out - z["out"]).max() < 1e-5
    ref_k = bf16f(z["out_ref"])
    floor = np.abs(bf16f(oracle_round(out)) - out).max()
    assert np.abs(ref_k - out).max() <= floor + 1e-6
    assert (oracle_round(out) != z["out_ref"]).mean() < 1e-3


def oracle_round(x):
    from oracle.reference_np import f32_to_bf16
    return f32_to_bf16(np.asarray(x, np.float32))


@pytest.mark.parametrize("name", ["prefill_37x37", "prefill_128x300"])
def test_prefill_error_yardsticks(ref_np, name):
    """The yardsticks the GPU prefill test applies (test_engine.py:97-99):
    an MLX-BF16 SDPA restatement and a plain BF16-P SDPA, both against the
    FP32 result.  The reference kernel itself sits at the BF16 floor."""
    z = load_golden(name)
    qL, kL = int(z["qL"]), int(z["kL"])
    ex = z["out"].astype(np.float64)
    e_mlx = np.abs(bf16f(ref_np.prefill_attention_mlx_bf16(z["Q"], z["K"], z["V"], qL, kL, 128 ** -0.5)) - ex).max()
    e_p16 = np.abs(bf16f(ref_np.prefill_attention_bf16p(z["Q"], z["K"], z["V"], qL, kL, 128 ** -0.5)) - ex).max()
    e_ref = np.abs(bf16f(z["out_ref"]) - ex).max()
    floor = np.abs(bf16f(oracle_round(ex)) - ex).max()
    assert e_ref <= floor + 1e-6
    assert floor - 1e-6 <= e_p16 <= 2 * floor
    assert e_mlx > e_ref  # the BF16 scaling of Q costs MLX accuracy


@pytest.mark.parametrize("name", ["model_gemv_qkv", "model_gemv_res", "model_gemv_swiglu",
                                  "model_gemv_down", "model_gemv_logits"])
def test_model_gemv_matches_reference_kernel(name):
    """oracle/model_np.gemv against the reference's GEMV kernel
    (agent-test/v2/kernels.py:18-113): its epilogue rounding points are the
    reference's; FP64 against lane-strided FP32 sums leaves a few one-ulp
    differences."""
    from oracle import model_np
    z = load_golden(name)
    N, K = int(z["N"]), int(z["K"])
    W, x, nw, res = _golden_mod().model_inputs(N, K, int(z["seed"]))
    assert _golden_mod().sha(W, x, nw, res) == str(z["inputs_sha256"])
    y = model_np.gemv(W, x, nw=nw if int(z["nw"]) else None, res=res if int(z["res"]) else None,
                      swiglu_epi=bool(int(z["swiglu"])), out_float=bool(int(z["out_float"])))
    if int(z["out_float"]):
        yr = z["y_ref"].astype(np.float64)
        assert np.abs(y - yr).max() <= 1e-5 * max(1.0, np.abs(yr).max())
        return
    yf, yr = bf16f(y), bf16f(z["y_ref"])
    ulp = np.abs(yr) * 2.0 ** -7 + 1e-30
    assert (np.abs(yf - yr) <= ulp).all()
    assert (y != z["y_ref"]).mean() < 0.02


def test_model_add_rms_matches_reference_kernel():
    """add_rms (kernels.py:227-268): the residual is bit-exact
    (test_engine.py:43-49); the normed row differs only by sum order."""
    from oracle import model_np
    z = load_golden("model_add_rms")
    r, n = model_np.add_rms(z["a"], z["b"], z["w"])
    assert np.array_equal(r, z["r_ref"])
    assert (n != z["n_ref"]).mean() < 1e-3
    assert np.abs(bf16f(n) - bf16f(z["n_ref"])).max() <= np.abs(bf16f(z["n_ref"])).max() * 2.0 ** -7


def test_model_skinny_matmul_matches_reference_kernel(wl):
    """The reference's small-M GEMM (kernels.py:273-334) against
    oracle/model_np.matmul: BF16 outputs of the same FP32-accumulated
    product, one ulp apart at most."""
    from conftest import u16
    from oracle import model_np
    z = load_golden("model_skinny")
    x = u16(wl.randn_bf16((int(z["M"]), int(z["K"])), int(z["seed_x"])))
    W = u16(wl.randn_bf16((int(z["N"]), int(z["K"])), int(z["seed_w"]), scale=0.03))
    assert _golden_mod().sha(x, W) == str(z["inputs_sha256"])
    y = model_np.matmul(x, W)
    yf, yr = bf16f(y), bf16f(z["y_ref"])
    assert (np.abs(yf - yr) <= np.abs(yr) * 2.0 ** -7 + 1e-30).all()
    assert (y != z["y_ref"]).mean() < 0.02


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
