"""GPU: the model kernels (csrc/model_kernels.cuh) and the Qwen3 engine
against the numpy model oracle (oracle/model_np.py).

Tolerances: the CUDA path sums in FP32, the oracle in FP64, so a BF16 result
may sit one BF16 step away where the exact value is near a rounding boundary;
the checks allow one step (2^-8 relative) on a small fraction of elements and
exact equality elsewhere.  Engine logits: max-abs <= 2e-2 and mean-abs <= 2e-3,
both relative to the largest logit; greedy tokens equal wherever the oracle's
top-2 margin exceeds the measured logit error."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import ROOT  # noqa: F401

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.fixture(scope="module")
def mnp():
    from oracle import model_np
    return model_np


def u16(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def bf(x: np.ndarray) -> np.ndarray:
    from oracle.reference_np import bf16_to_f32
    return bf16_to_f32(x)


def rand_bf16(shape, seed, scale=1.0, device=DEV):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(torch.bfloat16).to(device)


def assert_bf16_close(got: np.ndarray, want: np.ndarray, frac_exact=0.98, rel=2.0 ** -7, abs_tol=0.0):
    """Every element within `rel` of the oracle (one BF16 step is 2^-8) plus
    `abs_tol` (FP32-vs-FP64 summation error); most elements identical."""
    a, b = bf(got).astype(np.float64), bf(want).astype(np.float64)
    tol = rel * np.abs(b) + abs_tol + 1e-30
    assert np.all(np.abs(a - b) <= tol), float(np.max(np.abs(a - b) / tol))
    assert np.mean(a == b) >= frac_exact, float(np.mean(a == b))


def gemv_abs_tol(mnp, W, x, nw):
    """Per-row bound for a dot product summed in FP32 instead of FP64, plus one
    BF16 step of the pre-epilogue value (residual and SwiGLU round it first)."""
    xin = mnp.rms_norm(u16(x), u16(nw)) if nw is not None else u16(x)
    Wf, xf = np.abs(bf(u16(W)).astype(np.float64)), np.abs(bf(xin).astype(np.float64))
    acc = bf(u16(W)).astype(np.float64) @ bf(xin).astype(np.float64)
    return 1e-5 * (Wf @ xf) + 2.0 ** -7 * np.abs(acc)


# ------------------------------------------------------------------ GEMV
@pytest.mark.parametrize("N,K,epi", [(6144, 1024, "swiglu"), (1024, 3072, "res"), (4096, 1024, "norm"),
                                     (1000, 512, "none"), (40, 256, "norm"), (72, 136, "none")])
def test_gemv_wide_same_results(rib, N, K, epi):
    """The RIB_GEMV_WIDE launch form (16 warps per CTA) gives the same bits as
    the default form; shapes it does not cover (K without a compile-time
    chunk count) fall back to the default form."""
    W = rand_bf16((N, K), 11, 0.05)
    x = rand_bf16((K,), 12)
    nw = rand_bf16((K,), 13, 0.1) + 1 if epi in ("norm", "swiglu") else None
    res = rand_bf16((N,), 14) if epi == "res" else None
    a = rib.gemv(W, x, nw=nw, res=res, swiglu=epi == "swiglu")
    b = rib.gemv(W, x, nw=nw, res=res, swiglu=epi == "swiglu", wide=True)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("N,K", [(4096, 1024), (1024, 2048), (1024, 3072), (1000, 512), (40, 256),
                                 (1024, 384), (64, 1536), (72, 136)])
@pytest.mark.parametrize("epi", ["none", "norm", "res", "swiglu"])
def test_gemv(rib, mnp, N, K, epi):
    W = rand_bf16((N, K), 1, 0.05)
    x = rand_bf16((K,), 2)
    nw = rand_bf16((K,), 3, 0.1) + 1 if epi in ("norm", "swiglu") else None
    res = rand_bf16((N,), 4) if epi == "res" else None
    y = rib.gemv(W, x, nw=nw, res=res, swiglu=epi == "swiglu")
    want = mnp.gemv(u16(W), u16(x), nw=None if nw is None else u16(nw), res=None if res is None else u16(res),
                    swiglu_epi=epi == "swiglu")
    assert y.shape == ((N // 2,) if epi == "swiglu" else (N,))
    tol = gemv_abs_tol(mnp, W, x, nw)
    if epi == "swiglu":  # y = bf16(silu(g) * u): the gate and up errors both scale y
        g, u = bf(mnp.gemv(u16(W), u16(x), nw=u16(nw))).astype(np.float64).reshape(2, -1)
        tol = 2 * (tol[:N // 2] * np.abs(u) + tol[N // 2:] * np.abs(g))
        assert_bf16_close(u16(y), want, rel=2.0 ** -6, abs_tol=tol)
    else:
        assert_bf16_close(u16(y), want, abs_tol=tol)


def test_gemv_lm_head_logits(rib, mnp):
    """The tall LM-head shape (rows-per-warp 4 path), FP32 out, fused final norm."""
    V, K = 151936, 1024
    W = rand_bf16((V, K), 5, 0.02)
    x, nw = rand_bf16((K,), 6), rand_bf16((K,), 7, 0.1) + 1
    y = rib.gemv(W, x, nw=nw, out_float=True)
    want = mnp.gemv(u16(W), u16(x), nw=u16(nw), out_float=True)
    yh = y.cpu().numpy()
    scale = np.abs(bf(u16(W))).astype(np.float64) @ np.abs(bf(mnp.rms_norm(u16(x), u16(nw))))
    assert np.all(np.abs(yh - want) <= 1e-5 * scale + 1e-6)
    assert int(rib.argmax(y).item()) == int(np.argmax(want)) or \
        abs(np.sort(want)[-1] - np.sort(want)[-2]) < 1e-4


def test_gemv_output_buffer_and_errors(rib):
    W, x = rand_bf16((64, 256), 8), rand_bf16((256,), 9)
    out = torch.empty(64, dtype=torch.bfloat16, device=DEV)
    assert rib.gemv(W, x, out=out).data_ptr() == out.data_ptr()
    with pytest.raises(ValueError):
        rib.gemv(W, rand_bf16((128,), 1))
    with pytest.raises(ValueError):
        rib.gemv(W, x, res=rand_bf16((64,), 1), out_float=True)


# ------------------------------------------------------------------ row kernels
@pytest.mark.parametrize("rows,W", [(1, 1024), (37, 1024), (5, 256), (3, 3072)])
def test_add_rms_and_rms_norm(rib, mnp, rows, W):
    a, b, w = rand_bf16((rows, W), 10), rand_bf16((rows, W), 11), rand_bf16((W,), 12, 0.1) + 1
    r, n = rib.add_rms(a, b, w)
    wr, wn = mnp.add_rms(u16(a), u16(b), u16(w))
    np.testing.assert_array_equal(u16(r), wr)           # one rounded add: exact
    assert_bf16_close(u16(n), wn)
    assert_bf16_close(u16(rib.rms_norm(a, w)), mnp.rms_norm(u16(a), u16(w)))


@pytest.mark.parametrize("rows,F", [(1, 3072), (33, 3072), (4, 16)])
def test_swiglu(rib, mnp, rows, F):
    gu = rand_bf16((rows, 2 * F), 13, 2.0)
    assert_bf16_close(u16(rib.swiglu(gu)), mnp.swiglu(u16(gu)), frac_exact=0.98, rel=2.0 ** -6)


def test_embedding_and_bad_token(rib):
    table = rand_bf16((1000, 1024), 14)
    toks = torch.tensor([0, 999, 5, 5], dtype=torch.int32, device=DEV)
    y = rib.embedding(table, toks)
    assert torch.equal(y, table[toks.long()])
    rib._lib.take_device_status()
    bad = rib.embedding(table, torch.tensor([3, 1000], dtype=torch.int32, device=DEV))
    assert rib._lib.take_device_status() == 1          # RIB_EINVAL recorded on the device
    assert torch.equal(bad[0], table[3]) and not bad[1].any()


def test_argmax_first_on_ties(rib):
    x = torch.randn(151936, device=DEV)
    assert int(rib.argmax(x).item()) == int(torch.argmax(x).item())
    x[:] = -1.0
    x[700] = 5.0
    x[70000] = 5.0
    x[150000] = 5.0
    assert int(rib.argmax(x).item()) == 700
    small = torch.tensor([-3.0, -1.0, -2.0], device=DEV)
    assert int(rib.argmax(small).item()) == 1


def test_append_at_device_offset(rib):
    nq, nkv = 16, 8
    qkv = rand_bf16((3, (nq + 2 * nkv) * 128), 15)
    qw, kw = rand_bf16((128,), 16, 0.1) + 1, rand_bf16((128,), 17, 0.1) + 1
    c1 = torch.zeros((2, nkv, 256, 128), dtype=torch.bfloat16, device=DEV)
    c2 = c1.clone()
    q1 = rib.qk_norm_rope_append(qkv, qw, kw, 77, nq, nkv, 1e6, c1, 32)
    off = torch.tensor([77], dtype=torch.int32, device=DEV)
    q2 = rib.qk_norm_rope_append_at(qkv, qw, kw, off, nq, nkv, 1e6, c2, 32)
    assert torch.equal(q1, q2) and torch.equal(c1, c2)
    # offset + L past the capacity: caught on the device, nothing written
    rib._lib.take_device_status()
    c3 = torch.zeros_like(c1)
    rib.qk_norm_rope_append_at(qkv, qw, kw, torch.tensor([254], dtype=torch.int32, device=DEV), nq, nkv,
                               1e6, c3, 32)
    assert rib._lib.take_device_status() == 2          # RIB_ECAPACITY
    assert not c3.any()


# ------------------------------------------------------------------ engine
def _engine_check(rib, mnp, cfg, n_prompt, n_decode, seed):
    wt = rib.random_weights(cfg, seed=seed)               # CPU, seeded
    oracle = mnp.Qwen3Oracle(mnp.weights_to_numpy(wt), cfg, n_prompt + n_decode + 8)
    eng = rib.Engine(wt.to(DEV))
    cache = eng.new_cache(n_prompt + n_decode + 8)
    toks = np.random.default_rng(seed).integers(0, cfg.vocab_size, n_prompt).astype(np.int32)
    got = [eng.prefill(torch.tensor(toks, device=DEV), cache, last=True).reshape(-1).cpu().numpy()]
    want = [oracle.prefill(toks)]
    tok = int(np.argmax(want[0]))
    for _ in range(n_decode):
        got.append(eng.decode(torch.tensor([tok], dtype=torch.int32, device=DEV), cache,
                              return_logits=True).cpu().numpy())
        want.append(oracle.decode(tok))
        tok = int(np.argmax(want[-1]))
    assert cache.offset == oracle.offset == n_prompt + n_decode
    for g, w in zip(got, want):
        scale = np.abs(w).max()
        err = np.abs(g - w)
        assert err.max() <= 2e-2 * scale and err.mean() <= 2e-3 * scale, (err.max() / scale, err.mean() / scale)
        top2 = np.sort(w)[-2:]
        if top2[1] - top2[0] > 2 * err.max():
            assert int(np.argmax(g)) == int(np.argmax(w))
    return eng


def test_engine_tiny_matches_oracle(rib, mnp):
    cfg = rib.Qwen3Config(num_layers=2, hidden_size=256, num_heads=2, num_kv_heads=1,
                          intermediate_size=512, vocab_size=1000)
    _engine_check(rib, mnp, cfg, n_prompt=40, n_decode=5, seed=21)


def test_engine_qwen3_shapes_two_layers(rib, mnp):
    """Qwen3-0.6B widths (hidden 1024, 16/8 heads, FFN 3072, vocab 151936), 2 layers."""
    cfg = rib.Qwen3Config(num_layers=2)
    _engine_check(rib, mnp, cfg, n_prompt=300, n_decode=3, seed=22)


def test_decode_graph_matches_eager(rib):
    cfg = rib.Qwen3Config(num_layers=3, hidden_size=256, num_heads=2, num_kv_heads=1,
                          intermediate_size=512, vocab_size=1000)
    eng = rib.Engine(rib.random_weights(cfg, seed=23).to(DEV))
    prompt = list(np.random.default_rng(23).integers(0, cfg.vocab_size, 50))
    eager = list(eng.generate(prompt, max_tokens=12, use_graph=False))
    graph = list(eng.generate(prompt, max_tokens=12, use_graph=True))
    assert len(eager) == 12 and eager == graph
    # chunked prefill gives the same tokens
    assert list(eng.generate(prompt, max_tokens=12, chunk=16)) == eager


def test_decode_graph_state_and_launch_count(rib):
    cfg = rib.Qwen3Config(num_layers=2, hidden_size=256, num_heads=2, num_kv_heads=1,
                          intermediate_size=512, vocab_size=1000)
    eng = rib.Engine(rib.random_weights(cfg, seed=24).to(DEV))
    cache = eng.new_cache(64)
    eng.prefill(torch.arange(10, dtype=torch.int32, device=DEV), cache, last=False)
    ref_cache = eng.new_cache(64)
    ref_cache.storage.copy_(cache.storage)
    ref_cache.offset = cache.offset
    g = eng.decode_graph(cache)
    assert g.launches_per_step == 1 + 5 * cfg.num_layers + 2
    g.set_state(7, cache.offset)
    toks_g, tok = [], torch.tensor([7], dtype=torch.int32, device=DEV)
    toks_e = []
    for _ in range(4):
        g.replay()
        toks_g.append(int(g.tok.item()))
        tok = eng.decode(tok, ref_cache)
        toks_e.append(int(tok.item()))
    assert toks_g == toks_e
    assert int(g.pos.item()) == cache.offset == ref_cache.offset == 14
    assert torch.equal(cache.storage[:, :, :, :14], ref_cache.storage[:, :, :, :14])


# ------------------------------------------------------------------ persistent decode step
def _persistent_vs_graph(rib, cfg, seed, n_prompt=37, steps=6):
    eng = rib.Engine(rib.random_weights(cfg, seed=seed).to(DEV))
    cap = n_prompt + steps + 16
    ca, cb = eng.new_cache(cap), eng.new_cache(cap)
    toks = torch.tensor(np.random.default_rng(seed).integers(0, cfg.vocab_size, n_prompt).astype(np.int32),
                        device=DEV)
    first = rib.argmax(eng.prefill(toks, ca, last=True).reshape(-1))
    cb.storage.copy_(ca.storage)
    cb.offset = ca.offset
    g, pd = eng.decode_graph(ca), eng.persistent_decode(cb)
    g.set_state(first, ca.offset)
    pd.set_state(first, cb.offset)
    tg, tp, errs = [], [], []
    for _ in range(steps):
        g.replay()
        pd.replay(logits=True)
        tg.append(int(g.tok.item()))
        tp.append(int(pd.tok.item()))
        scale = g.logits.abs().max().item()
        errs.append((pd.logits - g.logits).abs().max().item() / scale)
    assert rib._lib.take_device_status() == 0
    assert tp == tg, (tp, tg)
    assert max(errs) <= 1e-2, errs
    assert int(pd.pos.item()) == cb.offset == ca.offset == n_prompt + steps
    assert torch.equal(ca.storage[:, :, :, :cb.offset], cb.storage[:, :, :, :cb.offset])
    return eng


def test_persistent_step_tiny_config(rib):
    """The generic instantiation (runtime K loops, no prefetch)."""
    cfg = rib.Qwen3Config(num_layers=3, hidden_size=256, num_heads=2, num_kv_heads=1,
                          intermediate_size=512, vocab_size=1000)
    _persistent_vs_graph(rib, cfg, seed=31)


def test_persistent_step_qwen3_widths(rib):
    """The Qwen3-0.6B instantiation (prefetched weight rows), 2 layers."""
    eng = _persistent_vs_graph(rib, rib.Qwen3Config(num_layers=2), seed=32)
    prompt = list(np.random.default_rng(33).integers(0, 151936, 70))
    a = list(eng.generate(prompt, max_tokens=10, mode="persistent"))
    b = list(eng.generate(prompt, max_tokens=10, mode="graph"))
    assert a == b and len(a) == 10


# ------------------------------------------------------------------ batched ragged decode
def test_batched_ragged_decode_matches_single(rib):
    """Sequences of different lengths in their own caches decode together:
    each row's logits match the single-sequence decode of the same token
    (teacher-forced for 3 steps), and generate_batch gives each prompt the
    tokens of its own generate() wherever the logit margin is clear."""
    from importlib import import_module
    batch = import_module("roofline-inference_b200.batch")
    cfg = rib.Qwen3Config(num_layers=2, hidden_size=256, num_heads=4, num_kv_heads=2,
                          intermediate_size=512, vocab_size=1000)
    eng = rib.Engine(rib.random_weights(cfg, seed=41).to(DEV))
    rng = np.random.default_rng(41)
    prompts = [list(rng.integers(0, cfg.vocab_size, n)) for n in (5, 70, 33, 129)]
    cb, cs = [], []
    for p in prompts:
        for lst in (cb, cs):
            c = eng.new_cache(len(p) + 8)
            eng.prefill(torch.tensor(p, dtype=torch.int32, device=DEV), c, last=False)
            lst.append(c)
    dec = batch.BatchDecoder(eng, cb)
    toks = torch.tensor([3, 7, 11, 13], dtype=torch.int32, device=DEV)
    for step in range(3):
        lb = dec.logits(toks)
        for i, c in enumerate(cs):
            ls = eng.decode(toks[i:i + 1], c, return_logits=True)
            rel = float((lb[i] - ls).abs().max() / ls.abs().max())
            assert rel <= 1e-2, (step, i, rel)
        toks = toks + 1
    assert [c.offset for c in cb] == [c.offset for c in cs] == [len(p) + 3 for p in prompts]
    assert rib._lib.take_device_status() == 0
    out = batch.generate_batch(eng, prompts, max_tokens=6)
    assert [len(o) for o in out] == [6] * 4
    for p, o in zip(prompts, out):
        assert o[0] == next(iter(eng.generate(p, max_tokens=1, use_graph=False)))


def test_batched_decode_graph_matches_eager(rib):
    """The CUDA-graph replay of the batched step gives the eager step's logits
    and tokens, advances every cache, and leaves the device status clean."""
    from importlib import import_module
    batch = import_module("roofline-inference_b200.batch")
    cfg = rib.Qwen3Config(num_layers=3, hidden_size=256, num_heads=4, num_kv_heads=2,
                          intermediate_size=512, vocab_size=1000)
    eng = rib.Engine(rib.random_weights(cfg, seed=43).to(DEV))
    rng = np.random.default_rng(43)
    prompts = [list(rng.integers(0, cfg.vocab_size, n)) for n in (9, 300, 41)]
    ce, cg = [], []
    for p in prompts:
        for lst in (ce, cg):
            c = eng.new_cache(len(p) + 6)
            eng.prefill(torch.tensor(p, dtype=torch.int32, device=DEV), c, last=False)
            lst.append(c)
    de = batch.BatchDecoder(eng, ce)
    dg = batch.BatchDecoder(eng, cg).capture()
    assert [c.offset for c in cg] == [len(p) for p in prompts]     # capture does not advance
    toks = torch.tensor([5, 6, 7], dtype=torch.int32, device=DEV)
    for step in range(4):
        le = de.logits(toks)
        tg = dg.step(toks)
        rel = float((le - dg.graph_logits).abs().max() / le.abs().max())
        assert rel <= 1e-3, (step, rel)
        agree = tg.cpu() == torch.argmax(le, dim=1).to(torch.int32).cpu()
        top2 = torch.topk(le, 2, dim=1).values
        assert bool(torch.all(agree | ((top2[:, 0] - top2[:, 1]) < 1e-2).cpu())), step
        toks = (toks * 3 + 1) % cfg.vocab_size
    assert [c.offset for c in cg] == [c.offset for c in ce] == [len(p) + 4 for p in prompts]
    assert rib._lib.take_device_status() == 0


def test_argmax_rows(rib):
    x = torch.randn(5, 151936, device=DEV)
    x[3, 10] = 100.0
    x[3, 20] = 100.0
    L = rib.load_library()
    out = torch.empty(5, dtype=torch.int32, device=DEV)
    assert L.rib_argmax_rows_f32(x.data_ptr(), 5, x.shape[1], out.data_ptr(),
                                 torch.cuda.current_stream().cuda_stream) == 0
    want = torch.argmax(x, dim=1).to(torch.int32)
    assert torch.equal(out, want) and int(out[3]) == 10


@pytest.mark.parametrize("rows,n", [(3, 1001), (7, 5), (2, 1), (4, 4099)])
def test_argmax_rows_ragged_alignment(rib, rows, n):
    """Rows whose starts fall off the 16-byte grid (n not a multiple of 4):
    the scalar head, vector body and scalar tail cover every element, and a
    tie inside the head keeps the first index."""
    g = torch.Generator(device=DEV).manual_seed(n)
    x = torch.randn(rows, n, device=DEV, generator=g)
    if n > 3:
        x[rows - 1, 1] = 50.0
        x[rows - 1, n - 1] = 50.0           # tie with a tail element: the first index wins
        x[0, n - 1] = 60.0                  # maximum in the tail
    L = rib.load_library()
    out = torch.empty(rows, dtype=torch.int32, device=DEV)
    assert L.rib_argmax_rows_f32(x.data_ptr(), rows, n, out.data_ptr(),
                                 torch.cuda.current_stream().cuda_stream) == 0
    assert torch.equal(out, torch.argmax(x, dim=1).to(torch.int32))


# ------------------------------------------------------------------ continuous batching
def test_scheduler_greedy_consistent(rib):
    """Requests served by the continuous-batching scheduler (fewer slots than
    requests, a pool that holds only some of them at once, chunked prefill,
    the step replayed from a CUDA graph while members join and leave) each get
    a greedy continuation: every token is the argmax, up to a near-tie margin,
    of the single-sequence engine's logits at its position given the same
    prefix, and the count and stopping rule are those of generate()."""
    from importlib import import_module
    sched = import_module("roofline-inference_b200.scheduler")
    cfg = rib.Qwen3Config(num_layers=2, hidden_size=256, num_heads=4, num_kv_heads=2,
                          intermediate_size=512, vocab_size=1000)
    eng = rib.Engine(rib.random_weights(cfg, seed=47).to(DEV))
    rng = np.random.default_rng(47)
    lens, mts = (5, 300, 40, 129, 700, 17), (6, 4, 9, 1, 5, 12)
    prompts = [[int(t) for t in rng.integers(0, cfg.vocab_size, n)] for n in lens]
    s = sched.Scheduler(eng, pool_rows=4 * 256 + 1024, slots=2, max_len=1024, chunk=256)
    ids = [s.submit(p, m) for p, m in zip(prompts, mts)]
    out = s.run()
    assert s.decode_steps > 0 and s.dec.graph is not None
    assert s.pool.free_pages == s.pool.pages
    for rid, p, m in zip(ids, prompts, mts):
        o = out[rid]
        assert len(o) == m, (rid, o)
        full = p + o[:-1]
        c = eng.new_cache(len(full) + 1)
        lg = eng.prefill(torch.tensor(full, dtype=torch.int32, device=DEV), c, last=True, all_logits=True)[0]
        for j, t in enumerate(o):
            row = lg[len(p) - 1 + j]
            margin = float(row.max() - row[t])
            assert margin <= 1e-2 * float(row.abs().max()), (rid, j, margin)
    assert rib._lib.take_device_status() == 0


# ------------------------------------------------------------------ tensor-parallel exchange, one rank
def test_tp_exchange_single_rank(rib):
    """The tensor-parallel kernels in a one-rank group: the partial-sum
    epilogue followed by an in_sum GEMV equals the residual GEMV chain
    bit for bit (one rank: the sum is the partial), over several exchanges
    (both buffer regions), and the exchanged argmax adds the slice offset."""
    import torch.distributed as dist
    from importlib import import_module
    tp = import_module("roofline-inference_b200.tp")
    dist.init_process_group("nccl", store=dist.HashStore(), rank=0, world_size=1, device_id=DEV)
    try:
        x = tp.TPExchange(512, DEV)
        L = rib.load_library()
        ws = torch.empty(int(L.rib_argmax_workspace_bytes()), dtype=torch.uint8, device=DEV)
        for it in range(3):
            Wo, o = rand_bf16((512, 256), 20 + it, 0.05), rand_bf16((256,), 30 + it)
            Wgu, nw = rand_bf16((768, 512), 40 + it, 0.05), rand_bf16((512,), 50 + it, 0.1) + 1
            h = rand_bf16((512,), 60 + it)
            x.gemv(Wo, o, epi=tp.EPI_PEER_PARTIAL)
            h1 = torch.empty_like(h)
            a = torch.empty(384, dtype=torch.bfloat16, device=DEV)
            x.gemv(Wgu, h, nw=nw, epi=2, out=a, in_sum=True, x_out=h1)
            want_h1 = rib.gemv(Wo, o, res=h)
            assert torch.equal(h1, want_h1), it
            assert torch.equal(a, rib.gemv(Wgu, want_h1, nw=nw, swiglu=True)), it
            lg = torch.randn(1000, device=DEV)
            lg[137 + it] = 50.0
            tok = torch.empty(1, dtype=torch.int32, device=DEV)
            x.argmax(lg, 5000, tok, ws)
            assert int(tok) == 5137 + it
        torch.cuda.synchronize()
        assert int(x.epoch) == 6 and int(x.done) == 0
        assert rib._lib.take_device_status() == 0
        x.close()
    finally:
        dist.destroy_process_group()


def test_qk_norm_rope_append_batched_matches_per_cache(rib):
    """The batched append (one launch for B caches of different capacities,
    each at its own position) writes the same K/V rows and returns the same q
    as B single-cache appends, bit for bit."""
    nq, nkv, B = 16, 8, 5
    g = torch.Generator(device=DEV).manual_seed(3)
    qkv = (torch.randn((B, (nq + 2 * nkv) * 128), generator=g, device=DEV)).to(torch.bfloat16)
    qw = (1 + 0.1 * torch.randn(128, generator=g, device=DEV)).to(torch.bfloat16)
    kw = (1 + 0.1 * torch.randn(128, generator=g, device=DEV)).to(torch.bfloat16)
    caps = [256, 512, 256, 768, 1024]
    positions = [0, 300, 255, 700, 513]
    ca = [torch.zeros((2, nkv, c, 128), dtype=torch.bfloat16, device=DEV) for c in caps]
    cb = [torch.zeros_like(c) for c in ca]
    q = rib.qk_norm_rope_append_batched(
        qkv, qw, kw, torch.tensor(positions, dtype=torch.int32, device=DEV),
        torch.tensor([c.data_ptr() for c in ca], dtype=torch.int64, device=DEV),
        torch.tensor(caps, dtype=torch.int32, device=DEV), nq, nkv, 1e6)
    for i in range(B):
        qi = rib.qk_norm_rope_append(qkv[i], qw, kw, positions[i], nq, nkv, 1e6, cb[i])
        assert torch.equal(q[i], qi.reshape(nq, 128)), i
        assert torch.equal(ca[i], cb[i]), i
    assert rib._lib.take_device_status() == 0
