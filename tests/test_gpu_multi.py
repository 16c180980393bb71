"""GPU, 2 ranks (one process per GPU, NCCL for set-up only): decode attention
fused with the NVLink all-gather, against the oracle on all 8 heads.

Each rank owns 4 of the 8 KV heads of a 4-layer, 4096-context sweep, runs
three calls (epochs 1-3, both output regions) with different queries, and
checks that its gathered buffer holds every rank's heads within the decode
tolerance.  Skips unless two GPUs are visible."""
from __future__ import annotations

import datetime
import importlib
import os
import socket
import sys

import numpy as np
import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu
LAYERS, CTX = 4, 4096


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q_out):
    try:
        sys.path.insert(0, str(ROOT))
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        torch.distributed.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                             timeout=datetime.timedelta(seconds=60))
        from oracle import oracle
        rib = importlib.import_module("roofline-inference_b200")
        wl = importlib.import_module("roofline-inference_b200.workloads")
        sh = importlib.import_module("roofline-inference_b200.sharding")
        ng = importlib.import_module("roofline-inference_b200.nvlink_gather")
        h0, h1 = sh.head_range(rank, world)
        nkv = h1 - h0
        n = CTX + 1
        cap = wl.round_cap(n)
        full = wl.randn_bf16((LAYERS, 2, 8, cap, 128), seed=77)       # same on every rank
        caches = full[:, :, h0:h1].contiguous().to(dev)
        stride = caches[0].numel() * 2
        ptrs = torch.tensor([caches.data_ptr() + i * stride for i in range(LAYERS)],
                            dtype=torch.int64, device=dev)
        lens = torch.full((LAYERS,), n, dtype=torch.int32, device=dev)
        L = rib.load_library()
        ws = torch.zeros(L.rib_decode_workspace_bytes(LAYERS, n, nkv), dtype=torch.uint8, device=dev)
        G = ng.NVLinkGather(LAYERS, 2 * nkv, dev)
        u16 = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
        worst = 0.0
        for call in range(3):
            q_full = wl.randn_bf16((LAYERS, 16, 128), seed=100 + call)
            out = G.decode(q_full[:, 2 * h0:2 * h1].contiguous().to(dev), ptrs, lens, n, cap,
                           wl.SCALE, ws)
            torch.cuda.synchronize(dev)
            got = out.float().cpu().numpy()
            of, _ = oracle.decode_attention_batched(u16(q_full), [u16(full[i]) for i in range(LAYERS)],
                                                    [n] * LAYERS, wl.SCALE)
            d = np.abs(got - of)
            assert d.max() <= 2e-2 and d.mean() <= 2e-3, (call, d.max(), d.mean())
            worst = max(worst, float(d.max()))
        status = importlib.import_module("roofline-inference_b200._lib").take_device_status()
        G.close()
        torch.distributed.destroy_process_group()
        q_out.put((rank, (worst, status)))
    except Exception as e:  # report to the parent
        q_out.put((rank, repr(e)))


def test_decode_nvlink_gather_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r, v in res.items():
        assert not isinstance(v, str), f"rank {r}: {v}"
        assert v[1] == 0, f"rank {r}: device status {v[1]}"


# ------------------------------------------------------------------ sharded Qwen3 forward
def _engine_worker(rank, world, port, q_out):
    try:
        sys.path.insert(0, str(ROOT))
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        torch.distributed.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                             timeout=datetime.timedelta(seconds=60))
        rib = importlib.import_module("roofline-inference_b200")
        cfg = rib.Qwen3Config(num_layers=2, hidden_size=256, num_heads=4, num_kv_heads=2,
                              intermediate_size=512, vocab_size=1000)
        w = rib.random_weights(cfg, seed=61).to(dev)           # identical on every rank
        prompt = [int(t) for t in np.random.default_rng(62).integers(0, cfg.vocab_size, 45)]
        eng = rib.Engine(w, shard=True)
        assert eng.n_kv == 1 and eng.nq_local == 2
        graph = list(eng.generate(prompt, max_tokens=10))                 # CUDA-graph steps
        eager = list(eng.generate(prompt, max_tokens=10, use_graph=False))
        # prefill logits of the sharded forward against the single-GPU forward
        toks = torch.tensor(prompt, dtype=torch.int32, device=dev)
        ls = eng.prefill(toks, eng.new_cache(64), last=True).reshape(-1)
        ref = rib.Engine(w)                                     # no collective calls
        lr = ref.prefill(toks, ref.new_cache(64), last=True).reshape(-1)
        rel = float((ls - lr).abs().max() / lr.abs().max())
        single = list(ref.generate(prompt, max_tokens=10))
        status = importlib.import_module("roofline-inference_b200._lib").take_device_status()
        eng.close()
        torch.distributed.destroy_process_group()
        q_out.put((rank, (graph, eager, single, rel, status)))
    except Exception as e:  # report to the parent
        q_out.put((rank, repr(e)))


def test_sharded_engine_two_gpus():
    """KV-head sharded Qwen3 forward on 2 GPUs: both ranks generate the same
    tokens as the single-GPU engine (graph and eager decode), and the sharded
    prefill's logits match the single-GPU ones."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_engine_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r, v in res.items():
        assert not isinstance(v, str), f"rank {r}: {v}"
        graph, eager, single, rel, status = v
        assert status == 0, f"rank {r}: device status {status}"
        assert rel <= 1e-2, f"rank {r}: prefill logits differ by {rel}"
        assert graph == eager == single, (r, graph, eager, single)
    assert res[0][0] == res[1][0]


# ------------------------------------------------------------------ tensor-parallel Qwen3 forward
def _tp_worker(rank, world, port, q_out):
    try:
        sys.path.insert(0, str(ROOT))
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        torch.distributed.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                             timeout=datetime.timedelta(seconds=60))
        rib = importlib.import_module("roofline-inference_b200")
        cfg = rib.Qwen3Config(num_layers=2, hidden_size=256, num_heads=4, num_kv_heads=2,
                              intermediate_size=512, vocab_size=1000)
        w = rib.random_weights(cfg, seed=63).to(dev)           # identical on every rank
        prompt = [int(t) for t in np.random.default_rng(64).integers(0, cfg.vocab_size, 45)]
        eng = rib.Engine(w, tp=True)
        assert eng.tp and eng.n_kv == 1 and eng.layers[0]["down"].shape[1] == 256
        ref = rib.Engine(w)                                     # single GPU, no collective calls
        toks = torch.tensor(prompt, dtype=torch.int32, device=dev)
        # prefill logits, then three eager decode steps' logits, against the single-GPU engine
        ct, cr = eng.new_cache(64), ref.new_cache(64)
        rels = [float((eng.prefill(toks, ct, last=True).reshape(-1) - (lr := ref.prefill(toks, cr, last=True)
                                                                        .reshape(-1))).abs().max()
                      / lr.abs().max())]
        t = torch.tensor([7], dtype=torch.int32, device=dev)
        for _ in range(3):
            lt = eng.decode(t, ct, return_logits=True)
            lr = ref.decode(t, cr, return_logits=True)
            rels.append(float((lt - lr).abs().max() / lr.abs().max()))
            t = (t * 5 + 3) % cfg.vocab_size
        graph = list(eng.generate(prompt, max_tokens=10))                 # CUDA-graph steps
        eager = list(eng.generate(prompt, max_tokens=10, use_graph=False))
        # every generated token is the single-GPU greedy choice for its prefix, up to a near tie
        full = torch.tensor(prompt + graph[:-1], dtype=torch.int32, device=dev)
        la = ref.prefill(full, ref.new_cache(64), last=True, all_logits=True)[0]
        margins = [float((la[len(prompt) - 1 + j].max() - la[len(prompt) - 1 + j][tk])
                         / la[len(prompt) - 1 + j].abs().max()) for j, tk in enumerate(graph)]
        status = importlib.import_module("roofline-inference_b200._lib").take_device_status()
        eng.close()
        torch.distributed.destroy_process_group()
        q_out.put((rank, (graph, eager, rels, max(margins), status)))
    except Exception as e:  # report to the parent
        q_out.put((rank, repr(e)))


def test_tp_engine_two_gpus():
    """Tensor-parallel Qwen3 forward on 2 GPUs (projections split, partial
    sums and argmax keys exchanged over NVLink inside the kernels): prefill and
    decode logits match the single-GPU engine, graph and eager decode give the
    same tokens on both ranks, and each token is the single-GPU greedy choice
    for its prefix up to a near-tie margin."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_tp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r, v in res.items():
        assert not isinstance(v, str), f"rank {r}: {v}"
        graph, eager, rels, margin, status = v
        assert status == 0, f"rank {r}: device status {status}"
        assert max(rels) <= 1e-2, f"rank {r}: logits differ by {rels}"
        assert graph == eager, (r, graph, eager)
        assert margin <= 1e-2, (r, margin)
    assert res[0][0] == res[1][0]


# ------------------------------------------------------------------ tensor-parallel prefill exchange
def _tpp_worker(rank, world, port, q_out):
    try:
        sys.path.insert(0, str(ROOT))
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        torch.distributed.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                             timeout=datetime.timedelta(seconds=60))
        sys.path.insert(0, str(ROOT / "tests"))
        from test_gpu_tp_prefill import close_bf16, expected
        wl = importlib.import_module("roofline-inference_b200.workloads")
        T = importlib.import_module("roofline-inference_b200.tp")
        u16 = lambda t: t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
        H, K = 1024, 1024                      # K: this rank's columns of a 2048-wide input
        ex = T.PrefillExchange(H, 4096, dev)
        results = []
        # ragged and full row counts, with and without the norm, on the same buffers (epochs 1-4)
        for call, (M, norm) in enumerate([(4096, True), (37, True), (1, False), (1000, True)]):
            As = [wl.randn_bf16((M, K), seed=1000 * call + r) for r in range(world)]
            Ws = [wl.randn_bf16((H, K), seed=1000 * call + 100 + r, scale=(K * world) ** -0.5) for r in range(world)]
            h = wl.randn_bf16((M, H), seed=1000 * call + 500)
            nw = (wl.randn_bf16((H,), seed=1000 * call + 600, scale=0.1) + 1.0).to(torch.bfloat16) if norm else None
            hd = h.to(dev)
            _, x = ex.project_add_rms(As[rank].to(dev), Ws[rank].to(dev), hd, None if nw is None else nw.to(dev))
            torch.cuda.synchronize(dev)
            res, xr = expected([(u16(a), u16(w)) for a, w in zip(As, Ws)], u16(h), None if nw is None else u16(nw))
            close_bf16(hd, res, f"call {call} residual")
            if norm:
                close_bf16(x, xr, f"call {call} normalised")
            results.append((u16(hd), None if x is None else u16(x)))
        status = importlib.import_module("roofline-inference_b200._lib").take_device_status()
        ex.close()
        torch.distributed.destroy_process_group()
        q_out.put((rank, (results, status)))
    except Exception as e:  # report to the parent
        q_out.put((rank, repr(e)))


def test_tp_prefill_exchange_two_gpus():
    """The tensor-parallel prefill exchange on 2 GPUs: each rank's owner-slot
    GEMM partials and the reduce kernel's NVLink row stores give, on both
    ranks, the oracle's residual add + RMSNorm of the rank-order sum, and the
    two ranks' results are bit-identical."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_tpp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r, v in res.items():
        assert not isinstance(v, str), f"rank {r}: {v}"
        assert v[1] == 0, f"rank {r}: device status {v[1]}"
    for (h0, x0), (h1, x1) in zip(res[0][0], res[1][0]):
        assert np.array_equal(h0, h1)
        assert (x0 is None and x1 is None) or np.array_equal(x0, x1)
