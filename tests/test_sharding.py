"""CPU: the multi-GPU host logic with two gloo ranks.

Each rank runs its shard of the work with the oracle (the checker, on CPU)
and the shards are combined with a real torch.distributed all-gather; the
result must equal the unsharded oracle.  Covers KV-head sharding of one
sequence (norm/RoPE/append + decode) and sequence sharding of a ragged batch."""
from __future__ import annotations

import importlib
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT, u16


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _init(rank, world, port):
    sys.path.insert(0, str(ROOT))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))


def _kv_head_worker(rank, world, port, result_q):
    try:
        _init(rank, world, port)
        from oracle import oracle
        sh = importlib.import_module("roofline-inference_b200.sharding")
        wl = importlib.import_module("roofline-inference_b200.workloads")
        ctx = 300
        st = wl.decode_step(ctx, seed=5)               # full 8-head layer, same on every rank
        h0, h1 = sh.head_range(rank, world)
        nkv = h1 - h0
        qkv = sh.shard_qkv(st.qkv, rank, world)
        cache = st.cache[:, h0:h1].contiguous()
        q, kv = oracle.qk_norm_rope(u16(qkv)[None], u16(st.qw), u16(st.kw), st.pos, 2 * nkv, nkv,
                                    1e6, 1)
        c = u16(cache).copy()
        c[:, :, st.pos] = kv[:, :, 0]
        _, ob = oracle.decode_attention(q[:, 0], c, st.n, wl.SCALE)
        local = torch.from_numpy(ob.view(np.int32).copy())    # [2*nkv, 64]: BF16 pairs (gloo has no int16)
        flat = torch.empty((world * local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype)
        dist.all_gather_into_tensor(flat, local)
        full = sh.assemble_heads(flat.view((world,) + tuple(local.shape)))
        result_q.put((rank, full.numpy().view(np.uint16).copy()))
        dist.destroy_process_group()
    except Exception as e:  # surface the failure to the parent
        result_q.put((rank, repr(e)))


def _ragged_worker(rank, world, port, result_q):
    try:
        _init(rank, world, port)
        from oracle import oracle
        sh = importlib.import_module("roofline-inference_b200.sharding")
        wl = importlib.import_module("roofline-inference_b200.workloads")
        lens = wl.ragged_lengths(7, 1, 400, seed=3)
        cap = wl.round_cap(max(lens))
        caches = [u16(wl.randn_bf16((2, 8, cap, 128), seed=50 + b)) for b in range(len(lens))]
        q = u16(wl.randn_bf16((len(lens), 16, 128), seed=60))
        assign = sh.balance_sequences(lens, world)
        slots = sh.slots_per_rank(assign)
        mine = assign[rank]
        local = torch.zeros((slots, 16, 64), dtype=torch.int32)  # BF16 pairs (gloo has no int16)
        if mine:
            _, ob = oracle.decode_attention_batched(q[mine], [caches[i] for i in mine],
                                                    [lens[i] for i in mine], wl.SCALE)
            local[:len(mine)] = torch.from_numpy(ob.view(np.int32).copy())
        flat = torch.empty((world * slots, 16, 64), dtype=torch.int32)
        dist.all_gather_into_tensor(flat, local)
        full = sh.scatter_back(flat.view(world, slots, 16, 64), assign, len(lens))
        result_q.put((rank, full.numpy().view(np.uint16).copy()))
        dist.destroy_process_group()
    except Exception as e:
        result_q.put((rank, repr(e)))


def _run(worker, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for r, v in results.items():
        assert not isinstance(v, str), f"rank {r}: {v}"
    return results


def test_kv_head_sharding_matches_unsharded(oracle, wl):
    results = _run(_kv_head_worker)
    st = wl.decode_step(300, seed=5)
    q, kv = oracle.qk_norm_rope(u16(st.qkv)[None], u16(st.qw), u16(st.kw), st.pos, 16, 8, 1e6, 1)
    c = u16(st.cache).copy()
    c[:, :, st.pos] = kv[:, :, 0]
    _, ob = oracle.decode_attention(q[:, 0], c, st.n, wl.SCALE)
    for r, full in results.items():
        assert np.array_equal(full, ob), r


def test_sequence_sharding_matches_unsharded(oracle, wl):
    results = _run(_ragged_worker)
    lens = wl.ragged_lengths(7, 1, 400, seed=3)
    cap = wl.round_cap(max(lens))
    caches = [u16(wl.randn_bf16((2, 8, cap, 128), seed=50 + b)) for b in range(len(lens))]
    q = u16(wl.randn_bf16((len(lens), 16, 128), seed=60))
    _, ob = oracle.decode_attention_batched(q, caches, lens, wl.SCALE)
    for r, full in results.items():
        assert np.array_equal(full, ob), r


def test_head_ranges_and_qkv_slices():
    sh = importlib.import_module("roofline-inference_b200.sharding")
    assert [sh.head_range(r, 4) for r in range(4)] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    with pytest.raises(ValueError):
        sh.head_range(0, 3)
    qkv = torch.arange(4096, dtype=torch.float32)
    parts = [sh.shard_qkv(qkv, r, 2) for r in range(2)]
    assert all(p.numel() == 2048 for p in parts)
    # rank 1: q heads 8..15, k heads 4..7 (rows 20..23), v heads 4..7 (rows 28..31)
    x = parts[1].reshape(16, 128)[:, 0]
    assert x.tolist() == [h * 128.0 for h in list(range(8, 16)) + list(range(20, 24)) +
                          list(range(28, 32))]


def test_balance_sequences_is_lpt_and_complete():
    sh = importlib.import_module("roofline-inference_b200.sharding")
    lens = [100, 90, 80, 10, 10, 10]
    a = sh.balance_sequences(lens, 2)
    assert sorted(a[0] + a[1]) == list(range(6))
    loads = [sum(lens[i] for i in x) for x in a]
    # LPT is within 4/3 of the optimum, which is at least max(total / world, max len)
    assert max(loads) <= 4 / 3 * max(sum(lens) / 2, max(lens))
    assert loads == [130, 170]
    assert sh.slots_per_rank(a) == max(len(x) for x in a)


def _tp_worker(rank, world, port, result_q):
    """One tensor-parallel layer on CPU: this rank's slices of the O, gate/up
    and down projections (tp.shard_layer), FP32 partial sums all-reduced over
    gloo, the SwiGLU on this rank's intermediate slice, and the LM-head slice
    all-gathered."""
    try:
        _init(rank, world, port)
        rib = importlib.import_module("roofline-inference_b200")
        tp = importlib.import_module("roofline-inference_b200.tp")
        sh = importlib.import_module("roofline-inference_b200.sharding")
        cfg = rib.Qwen3Config(num_layers=1, hidden_size=256, num_heads=8, num_kv_heads=4,
                              intermediate_size=512, vocab_size=1000)
        w = rib.random_weights(cfg, seed=21)
        layer = {k: v.float() for k, v in w.layers[0].items()}
        h0, h1 = sh.head_range(rank, world, cfg.num_kv_heads)
        f0, f1 = tp.split_range(cfg.intermediate_size, rank, world)
        v0, v1 = tp.split_range(cfg.vocab_size, rank, world)
        s = tp.shard_layer(layer, h0, h1, f0, f1, cfg.num_heads, cfg.num_kv_heads)
        g = torch.Generator().manual_seed(3)
        o_all = torch.randn(4, cfg.q_dim, generator=g)           # attention outputs of 4 tokens
        x = torch.randn(4, cfg.hidden_size, generator=g)          # normalised MLP input
        part = o_all[:, 2 * h0 * 128:2 * h1 * 128] @ s["o"].t()   # row-parallel O
        dist.all_reduce(part)
        gu = x @ s["gu"].t()                                      # column-parallel gate / up
        F = f1 - f0
        act = torch.nn.functional.silu(gu[:, :F]) * gu[:, F:]
        down = act @ s["down"].t()                                # row-parallel down
        dist.all_reduce(down)
        logits = x @ w.embed[v0:v1].float().t()                   # vocabulary-parallel LM head
        parts = [torch.empty_like(logits) for _ in range(world)]
        dist.all_gather(parts, logits)
        result_q.put((rank, (part.numpy(), down.numpy(), torch.cat(parts, dim=1).numpy())))
        dist.destroy_process_group()
    except Exception as e:
        result_q.put((rank, repr(e)))


def test_tensor_parallel_layer_matches_unsharded():
    """Two gloo ranks: the tensor-parallel split of a Qwen3 layer reproduces
    the unsplit products (O, SwiGLU MLP, LM head) on every rank."""
    results = _run(_tp_worker)
    rib = importlib.import_module("roofline-inference_b200")
    cfg = rib.Qwen3Config(num_layers=1, hidden_size=256, num_heads=8, num_kv_heads=4,
                          intermediate_size=512, vocab_size=1000)
    w = rib.random_weights(cfg, seed=21)
    layer = {k: v.float() for k, v in w.layers[0].items()}
    g = torch.Generator().manual_seed(3)
    o_all = torch.randn(4, cfg.q_dim, generator=g)
    x = torch.randn(4, cfg.hidden_size, generator=g)
    F = cfg.intermediate_size
    gu = x @ layer["gu"].t()
    want = (o_all @ layer["o"].t(),
            (torch.nn.functional.silu(gu[:, :F]) * gu[:, F:]) @ layer["down"].t(),
            x @ w.embed.float().t())
    for r, got in results.items():
        for a, b in zip(got, want):
            np.testing.assert_allclose(a, b.numpy(), rtol=1e-4, atol=1e-4)
