#!/usr/bin/env python
"""Benchmark of the B200 Qwen3 attention hot path.

Headline (one JSON line on rank 0): GQA decode-attention HBM throughput at 32k
context -- the decode sweep workload: 28 layers with independent seeded BF16
N(0,1) caches, 16 q heads / 8 KV heads / head_dim 128, one new token attending
to 32769 keys per layer.  A step decodes all 28 layers in one layer-batched
launch of the split-KV kernel (the layers are independent, so one launch does
the same work as 28 and does not pay 28 launch latencies).  With N GPUs the
8 KV heads are sharded (8/N per rank, no cross-rank softmax) and the decode
kernel itself stores each head output into every rank's buffer over NVLink
(nvlink_gather.py), so the step is one launch; decode + an NCCL all-gather
is timed beside it as the baseline.  Metric: algorithmic KV bytes (4096 B
per key per layer) / step time, whole job.

Also reported: the same sweep as 28 per-layer launches (engine-style), the
causal prefill attention TFLOP/s at L = 32768 (tcgen05 kernel), the end-to-end
figure through the public Python API with host buffers, the roofline of the
dominant kernel, the clocks seen during the timed region and the CPU oracle
timed on the host cores.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""
from __future__ import annotations

import argparse
import datetime
import importlib
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "GQA decode-attn HBM GB/s (% of peak) at 32k ctx; causal prefill attn TFLOPS"
CTX = 32768
N_LAYERS = 28
NKV_TOTAL = 8
PREFILL_L = 32768


def profile_traffic(name: str) -> dict | None:
    """The DRAM traffic record of one ncu capture (profiles/<name>.json:
    dram__bytes_read.sum + dram__bytes_write.sum of the captured launch and
    the algorithmic bytes or FLOPs it carried), or None."""
    p = ROOT / "profiles" / f"{name}.json"
    return json.loads(p.read_text()) if p.exists() else None


def decode_traffic_ratio(kernel: str) -> float | None:
    """DRAM bytes (read + write) per algorithmic KV byte of `kernel` from one
    ncu capture of the one-GPU launch; traffic grows with the keys processed,
    so it scales to a rank's share at N > 1.  None when the record is of
    another kernel."""
    rec = profile_traffic("decode_kernel_traffic")
    if rec is None or rec.get("kernel") != kernel:
        return None
    return float(rec["traffic_per_algorithmic_byte"])


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured (MEASURED_PEAKS.json)"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during a region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        if self.path and os.path.exists(self.path):
            for line in open(self.path):
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
            os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return float("nan")

        sm = [num(r[1]) for r in rows]
        smax = max(num(r[2]) for r in rows)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        loaded = [s for s in sm if s > 0.5 * smax] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": smax, "reasons": reasons,
                "samples": len(rows)}


# ---------------------------------------------------------------- helpers
def load_rib():
    return importlib.import_module("roofline-inference_b200")


def head_range(rank: int, world: int) -> tuple[int, int]:
    if NKV_TOTAL % world:
        raise SystemExit(f"--gpus must divide {NKV_TOTAL} KV heads")
    return importlib.import_module("roofline-inference_b200.sharding").head_range(rank, world,
                                                                                 NKV_TOTAL)


def make_decode_workload(rank: int, world: int, device, ctx: int = CTX, layers: int = N_LAYERS):
    """Caches for this rank's KV heads of every layer, seeded per (layer, head)
    so that the union over ranks is the 1-GPU workload."""
    wl = importlib.import_module("roofline-inference_b200.workloads")
    h0, h1 = head_range(rank, world)
    nkv = h1 - h0
    n = ctx + 1
    cap = wl.round_cap(n)
    caches = torch.empty((layers, 2, nkv, cap, 128), dtype=torch.bfloat16, device=device)
    for layer in range(layers):
        for j, h in enumerate(range(h0, h1)):
            for kv in range(2):
                caches[layer, kv, j, :n] = wl.randn_bf16((n, 128), seed=(layer * 64 + h) * 2 + kv,
                                                         device=device)
            caches[layer, :, j, n:] = 0
    q = torch.empty((layers, 2 * nkv, 128), dtype=torch.bfloat16, device=device)
    for layer in range(layers):
        for j, h in enumerate(range(h0, h1)):
            q[layer, 2 * j:2 * j + 2] = wl.randn_bf16((2, 128), seed=900000 + layer * 64 + h,
                                                      device=device)
    return {"caches": caches, "q": q, "n": n, "cap": cap, "nkv": nkv, "h0": h0}


class DecodePlan:
    """Preallocated arguments of the layer-batched decode launch (C ABI)."""

    def __init__(self, rib, w, device):
        self.L = rib.load_library()
        self.w = w
        layers = w["caches"].shape[0]
        stride = w["caches"][0].numel() * 2
        self.ptrs = torch.tensor([w["caches"].data_ptr() + i * stride for i in range(layers)],
                                 dtype=torch.int64, device=device)
        self.lens = torch.full((layers,), w["n"], dtype=torch.int32, device=device)
        self.out = torch.empty_like(w["q"])
        self.layers = layers
        nbytes = self.L.rib_decode_workspace_bytes(layers, w["n"], w["nkv"])
        self.ws = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        self.per_layer_ws = torch.zeros(self.L.rib_decode_workspace_bytes(1, w["n"], w["nkv"]),
                                        dtype=torch.uint8, device=device)
        self.device = device
        self.scale = 128 ** -0.5

    def launch(self):
        st = self.L.rib_decode_attention_batched(
            self.w["q"].data_ptr(), self.ptrs.data_ptr(), self.lens.data_ptr(), self.layers,
            self.w["n"], self.w["cap"], 2 * self.w["nkv"], self.w["nkv"], self.scale,
            self.out.data_ptr(), self.ws.data_ptr(), self.ws.numel(),
            torch.cuda.current_stream(self.device).cuda_stream)
        if st != 0:
            raise RuntimeError(f"decode launch failed: status {st}")

    def launch_layer(self, i: int):
        w = self.w
        st = self.L.rib_decode_attention(
            w["q"][i].data_ptr(), w["caches"][i].data_ptr(), w["cap"], w["n"], 2 * w["nkv"],
            w["nkv"], self.scale, self.out[i].data_ptr(), self.per_layer_ws.data_ptr(),
            self.per_layer_ws.numel(), torch.cuda.current_stream(self.device).cuda_stream)
        if st != 0:
            raise RuntimeError(f"decode launch failed: status {st}")


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------- parity checks
# Run after the timed regions, on the outputs the timed path produced: a plain
# PyTorch FP32 restatement on the device (not the CUDA kernels, not the CPU
# oracle) recomputes a sample of each result from the same seeds, and the
# error is the max over ranks.  Tolerance: the contract's max-abs <= 2e-2 and
# mean-abs <= 2e-3 on attention outputs; for the model, logits within 2e-2 of
# the largest logit and greedy tokens equal unless the reference's top two
# logits are within that margin (a near tie).
PARITY_MAX_ABS, PARITY_MEAN_ABS, PARITY_LOGIT_REL = 2e-2, 2e-3, 2e-2


def _bf(x: torch.Tensor) -> torch.Tensor:
    """Round an FP32 tensor to BF16 and back (the kernels' rounding points)."""
    return x.to(torch.bfloat16).float()


def ref_attention(q, K, V, scale, causal_offset=None):
    """softmax(scale q K^T) V in FP32: q [H, m, 128], K/V [nkv, n, 128] -> [H, m, 128]
    (GQA head h -> h // (H / nkv)); causal_offset: query i sees keys <= offset + i."""
    g = q.shape[0] // K.shape[0]
    Kf = K.float().repeat_interleave(g, 0)
    Vf = V.float().repeat_interleave(g, 0)
    s = torch.matmul(q.float(), Kf.transpose(1, 2)) * scale
    if causal_offset is not None:
        m, n = q.shape[1], K.shape[1]
        mask = torch.arange(n, device=q.device)[None, :] > (causal_offset + torch.arange(m, device=q.device))[:, None]
        s = s.masked_fill(mask, float("-inf"))
    return torch.matmul(torch.softmax(s, dim=-1), Vf)


def attention_errors(got: torch.Tensor, want: torch.Tensor) -> dict:
    d = (got.float() - want.float()).abs()
    return {"max_abs": float(d.max()), "mean_abs": float(d.mean())}


def reduce_errors(errs: list[dict], world: int, device) -> dict:
    """Max over the listed checks and over ranks; pass against the contract."""
    mx = max((e["max_abs"] for e in errs), default=0.0)
    mean = max((e["mean_abs"] for e in errs), default=0.0)
    mx, mean = max_over_ranks(mx, world, device), max_over_ranks(mean, world, device)
    return {"max_abs": mx, "mean_abs": mean, "checks": len(errs) * world,
            "pass": bool(mx <= PARITY_MAX_ABS and mean <= PARITY_MEAN_ABS)}


def ref_rms(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """n = bf16(w * bf16(x * inv)), inv = 1/sqrt(mean(x^2) + 1e-6) (agent-test/v2/kernels.py:48-55)."""
    inv = torch.rsqrt(x.double().pow(2).mean(-1, keepdim=True) + 1e-6).float()
    return _bf(w.float() * _bf(x * inv))


def ref_rope(x: torch.Tensor, pos: torch.Tensor, base: float) -> torch.Tensor:
    """Non-traditional RoPE of [n, heads, 128] at positions pos [n]; the angle
    float(pos) * exp2(-(d/64) log2(base)) in FP32 (kernels.py:134-143)."""
    d = torch.arange(64, dtype=torch.float32, device=x.device) / 64.0
    lb = torch.tensor(math.log2(base), dtype=torch.float32, device=x.device)
    inv = torch.exp2((-d * lb).double()).float()
    th = (pos.float()[:, None] * inv[None]).double()[:, None, :]
    c, s = torch.cos(th), torch.sin(th)
    x1, x2 = x[..., :64].double(), x[..., 64:].double()
    return _bf(torch.cat([x1 * c - x2 * s, x1 * s + x2 * c], dim=-1).float())


def ref_model_logits(wt, tokens: list[int]) -> torch.Tensor:
    """FP32 logits of the last of `tokens` from a full causal pass of the
    Qwen3 forward (agent-test/v2/engine.py:102-142) in plain PyTorch on the
    device, BF16 rounding where the reference's kernels round."""
    cfg = wt.config
    nq, nkv = cfg.num_heads, cfg.num_kv_heads
    dev = wt.embed.device
    idx = torch.tensor(tokens, dtype=torch.long, device=dev)
    n = len(tokens)
    pos = torch.arange(n, device=dev)
    h = wt.embed[idx].float()
    x = ref_rms(h, wt.layers[0]["in_norm"])
    for i, l in enumerate(wt.layers):
        qkv = _bf(x @ l["qkv"].float().t()).reshape(n, nq + 2 * nkv, 128)
        q = ref_rope(ref_rms(qkv[:, :nq], l["q_norm"]), pos, cfg.rope_theta)
        k = ref_rope(ref_rms(qkv[:, nq:nq + nkv], l["k_norm"]), pos, cfg.rope_theta)
        v = qkv[:, nq + nkv:]
        o = ref_attention(q.transpose(0, 1), k.transpose(0, 1), v.transpose(0, 1), 128 ** -0.5,
                          causal_offset=0)
        o = _bf(o.transpose(0, 1).reshape(n, nq * 128))
        h = _bf(h + _bf(o @ l["o"].float().t()))
        x = ref_rms(h, l["post_norm"])
        gu = _bf(x @ l["gu"].float().t())
        F = gu.shape[-1] // 2
        g, u = gu[:, :F], gu[:, F:]
        a = _bf(_bf(g * _bf(torch.sigmoid(g))) * u)
        h = _bf(h + _bf(a @ l["down"].float().t()))
        if i + 1 < len(wt.layers):
            x = ref_rms(h, wt.layers[i + 1]["in_norm"])
    return ref_rms(h[-1:], wt.final_norm)[0] @ wt.embed.float().t()


def decode_sweep_parity(out_full: torch.Tensor, world: int, device, ctx: int = CTX,
                        layers=(0, N_LAYERS - 1)) -> dict:
    """The decode sweep's outputs [28, 16, 128] (every head of every layer,
    gathered over NVLink at N > 1) against the FP32 restatement for `layers`,
    regenerated from the workload's seeds."""
    wl = importlib.import_module("roofline-inference_b200.workloads")
    n = ctx + 1
    errs = []
    for layer in layers:
        K = torch.empty((NKV_TOTAL, n, 128), dtype=torch.bfloat16, device=device)
        V = torch.empty_like(K)
        for h in range(NKV_TOTAL):
            K[h] = wl.randn_bf16((n, 128), seed=(layer * 64 + h) * 2, device=device)
            V[h] = wl.randn_bf16((n, 128), seed=(layer * 64 + h) * 2 + 1, device=device)
        q = torch.cat([wl.randn_bf16((2, 128), seed=900000 + layer * 64 + h, device=device)
                       for h in range(NKV_TOTAL)])
        want = ref_attention(q[:, None], K, V, 128 ** -0.5)[:, 0]
        errs.append(attention_errors(out_full[layer], want))
        del K, V
    r = reduce_errors(errs, world, device)
    r["sample"] = f"layers {list(layers)}, all 16 heads, {n} keys"
    return r


def model_parity(rib, world: int, device, steps: int = 6) -> dict:
    """The Qwen3 forward (2 layers at Qwen3-0.6B widths, vocab 151936, seeded
    random weights) as the bench runs it -- one GPU, or at N > 1 KV-head
    sharded and tensor parallel -- against ref_model_logits: the prefill's
    logits of a 37-token prompt, then `steps` decode steps teacher-forced with
    the reference's greedy tokens (eager path), and the greedy tokens of
    Engine.generate (the CUDA-graph step) against the reference's greedy
    continuation."""
    cfg = rib.Qwen3Config(num_layers=2)
    wt = rib.random_weights(cfg, seed=11, device=device)
    g = torch.Generator().manual_seed(5)
    prompt = [int(t) for t in torch.randint(0, cfg.vocab_size, (37,), generator=g)]
    # the reference's greedy continuation, with each step's top-two margin
    ref_toks, margins, ref_logits = list(prompt), [], []
    for _ in range(steps + 1):
        lg = ref_model_logits(wt, ref_toks)
        top = torch.topk(lg, 2).values
        margins.append(float((top[0] - top[1]) / lg.abs().max()))
        ref_logits.append(lg)
        ref_toks.append(int(torch.argmax(lg)))
    modes = [("single_gpu", {})] if world == 1 else [("kv_head_shard", {"shard": True}),
                                                     ("tensor_parallel", {"tp": True})]
    out = {}
    for name, kw in modes:
        eng = rib.Engine(wt, **kw)
        cache = eng.new_cache(64)
        lg = eng.prefill(torch.tensor(prompt, dtype=torch.int32, device=device), cache, last=True).reshape(-1)
        worst, tok_ok = 0.0, True
        for t in range(steps + 1):
            ref = ref_logits[t]
            worst = max(worst, float((lg - ref).abs().max() / ref.abs().max()))
            if int(torch.argmax(lg)) != ref_toks[len(prompt) + t] and margins[t] > PARITY_LOGIT_REL:
                tok_ok = False
            if t < steps:
                lg = eng.decode(torch.tensor([ref_toks[len(prompt) + t]], dtype=torch.int32, device=device),
                                cache, return_logits=True).reshape(-1)
        gen = list(eng.generate(prompt, max_tokens=steps + 1))
        gen_ok = True
        for t, tok in enumerate(gen):
            if tok != ref_toks[len(prompt) + t]:
                gen_ok = margins[t] <= PARITY_LOGIT_REL  # a near tie: later tokens may diverge
                break
        eng.close()
        worst = max_over_ranks(worst, world, device)
        ok = max_over_ranks(0.0 if (tok_ok and gen_ok) else 1.0, world, device) == 0.0
        out[name] = {"logits_max_rel": worst, "tokens_ok": ok,
                     "pass": bool(ok and worst <= PARITY_LOGIT_REL)}
    out["sample"] = (f"2 layers, Qwen3-0.6B widths, 37-token prompt + {steps} teacher-forced decode steps; "
                     f"greedy tokens of Engine.generate (CUDA-graph step)")
    out["pass"] = all(v["pass"] for k, v in out.items() if isinstance(v, dict))
    del wt
    torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------- CPU leg
def cpu_sample_workload(layers_sample: int = 4, ctx: int = CTX):
    """Host copies of `layers_sample` layers of the decode sweep (the same
    seeds as the GPU workload), as uint16 BF16 bit patterns."""
    import numpy as np
    wl = importlib.import_module("roofline-inference_b200.workloads")
    n = ctx + 1
    cap = wl.round_cap(n)
    caches, qs = [], []
    for layer in range(layers_sample):
        c = np.zeros((2, NKV_TOTAL, cap, 128), np.uint16)
        for h in range(NKV_TOTAL):
            for kv in range(2):
                t = wl.randn_bf16((n, 128), seed=(layer * 64 + h) * 2 + kv)
                c[kv, h, :n] = t.view(torch.int16).numpy().view(np.uint16)
        caches.append(c)
        qs.append(np.concatenate([wl.randn_bf16((2, 128), seed=900000 + layer * 64 + h)
                                  .view(torch.int16).numpy().view(np.uint16)
                                  for h in range(NKV_TOTAL)]))
    return np.stack(qs), caches, n


def cpu_pass(sample) -> float:
    """One pass of the C oracle (all host threads) over the sample; seconds."""
    from oracle import oracle as coracle
    q, caches, n = sample
    t0 = time.perf_counter()
    coracle.decode_attention_batched(q, caches, [n] * len(caches), 128 ** -0.5)
    return time.perf_counter() - t0


def cpu_decode_sample(layers_sample: int = 4, ctx: int = CTX, budget_s: float = 12.0) -> dict:
    """Times the C oracle (OpenMP, all host threads) on `layers_sample` layers
    of the decode sweep at `ctx`, repeated for about `budget_s` seconds; value
    in GB/s of KV read (4096 B per key per layer)."""
    from oracle import oracle as coracle
    threads = coracle.set_threads(os.cpu_count())
    sample = cpu_sample_workload(layers_sample, ctx)
    cpu_pass(sample)  # warm
    reps, t_total = 0, 0.0
    while t_total < budget_s and reps < 10000:
        t_total += cpu_pass(sample)
        reps += 1
    bytes_per = layers_sample * 4096 * sample[2]
    return {"value": bytes_per * reps / t_total / 1e9, "unit": "GB/s", "cores": threads,
            "kind": "port",
            "sample": f"{layers_sample} of {N_LAYERS} layers at ctx {ctx} (all 8 KV heads), "
                      f"{reps} passes in {t_total:.1f} s, C oracle (OpenMP FP32)",
            "seconds": t_total}


def run_reference(args):
    """--impl reference: the reference's CPU path for this workload.  MLX (the
    reference's attention backend) is not installable here, so the CPU oracle
    port of its semantics is timed on the host cores; each step is one pass
    over a 4-layer sample of the 28-layer sweep."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle as coracle
    threads = coracle.set_threads(os.cpu_count())
    layers_sample = 4
    sample = cpu_sample_workload(layers_sample)
    for _ in range(max(args.warmup, 0)):
        cpu_pass(sample)
    secs = [cpu_pass(sample) for _ in range(args.steps)]
    bytes_per = layers_sample * 4096 * sample[2]
    total = sum(secs)
    v = bytes_per * len(secs) / total / 1e9
    desc = (f"{layers_sample} of {N_LAYERS} layers at ctx {CTX} (all 8 KV heads) per step, "
            f"C oracle (OpenMP FP32)")
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "GB/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": total / len(secs) * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"decode sweep: {N_LAYERS} layers x ctx {CTX} (+1 new token), "
                                   f"16q/8kv heads, head_dim 128", "sample": desc},
            "cpu_baseline": {"value": v, "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": desc},
            "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "MLX (the reference's attention backend) is not installable offline; "
                    "the oracle port of its semantics runs on the host cores"}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU leg
def run_ours(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        torch.distributed.init_process_group(
            "nccl", device_id=device, timeout=datetime.timedelta(seconds=120))
    rib = load_rib()
    pk = peaks()

    w = make_decode_workload(rank, world, device)
    plan = DecodePlan(rib, w, device)
    # all-gather output, concatenated along dim 0: [world * layers, nq_local, 128]
    gathered = torch.empty((world * plan.out.shape[0],) + tuple(plan.out.shape[1:]),
                           dtype=torch.bfloat16, device=device)
    stream = torch.cuda.current_stream(device)

    gather = None
    if world > 1:  # decode fused with the NVLink all-gather of head outputs
        gather = importlib.import_module("roofline-inference_b200.nvlink_gather").NVLinkGather(
            N_LAYERS, 2 * w["nkv"], device)

    def step():
        if gather is not None:
            gather.decode(w["q"], plan.ptrs, plan.lens, w["n"], w["cap"], plan.scale, plan.ws)
        else:
            plan.launch()

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        # The sampler's start-up leaves the GPU idle for 0.3 s; the warm-up
        # steps run after it, right before the timed ones, so that the timed
        # steps start at the clocks of a busy GPU.
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        barrier(world)
        start.record(stream)
        for _ in range(args.steps):
            step()
        end.record(stream)
        torch.cuda.synchronize()
        barrier(world)
    ms_local = start.elapsed_time(end) / args.steps
    ms = max_over_ranks(ms_local, world, device)
    # parity of the timed step's own outputs (every rank's heads at N > 1)
    parity = {"decode_sweep": decode_sweep_parity(gather.output() if gather is not None else plan.out,
                                                  world, device)}
    # Each step is exactly one launch of the decode kernel, so the average
    # launch duration is this rank's timed region over K.  (Events recorded
    # between the launches would split the programmatic-dependent-launch
    # chain and time the gaps they cause, not the kernel.)
    launch_ms = ms_local
    bytes_step_total = N_LAYERS * 4096 * w["n"]          # all ranks
    bytes_launch_local = N_LAYERS * 2 * w["nkv"] * 128 * 2 * w["n"]
    value = bytes_step_total / (ms * 1e-3) / 1e9
    achieved = bytes_launch_local / (launch_ms * 1e-3) / 1e9
    clk = clocks.summary()
    choice = int(rib.load_library().rib_decode_kernel_choice(N_LAYERS, w["n"], w["nkv"]))
    kernel = "rib::decode::decode_streamk_kernel" if choice == 1 else "rib::decode::decode_kernel"
    ratio = decode_traffic_ratio(kernel)

    # ---- N > 1 baseline: the same step as decode + a separate NCCL all-gather
    nccl = None
    if world > 1:
        def nccl_step():
            plan.launch()
            torch.distributed.all_gather_into_tensor(gathered, plan.out)
        for _ in range(args.warmup):
            nccl_step()
        torch.cuda.synchronize()
        barrier(world)
        a0, b0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        for _ in range(args.steps):
            nccl_step()
        b0.record(stream)
        torch.cuda.synchronize()
        nccl_ms = max_over_ranks(a0.elapsed_time(b0) / args.steps, world, device)
        nccl = {"value": bytes_step_total / (nccl_ms * 1e-3) / 1e9, "unit": "GB/s",
                "ms_per_step": nccl_ms,
                "path": "decode kernel + torch.distributed.all_gather_into_tensor (NCCL)"}
        # the same decode with no exchange at all: what the gather adds is the
        # difference (every rank still times its own launches, max over ranks)
        for _ in range(args.warmup):
            plan.launch()
        torch.cuda.synchronize()
        barrier(world)
        a1, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a1.record(stream)
        for _ in range(args.steps):
            plan.launch()
        b1.record(stream)
        torch.cuda.synchronize()
        local_ms = max_over_ranks(a1.elapsed_time(b1) / args.steps, world, device)
        nccl["decode_only_ms_per_step"] = local_ms
        nccl["fused_exchange_us"] = (ms - local_ms) * 1e3
        nccl["nccl_exchange_us"] = (nccl_ms - local_ms) * 1e3

    # ---- engine-style: 28 per-layer launches of the same sweep
    for i in range(N_LAYERS):
        plan.launch_layer(i)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(args.steps):
        for i in range(N_LAYERS):
            plan.launch_layer(i)
    b.record(stream)
    torch.cuda.synchronize()
    per_layer_ms = a.elapsed_time(b) / args.steps
    per_layer_gbs = bytes_launch_local / (per_layer_ms * 1e-3) / 1e9

    # ---- end to end through the public API with host buffers
    e2e = run_e2e(rib, w, rank, world, device, args, gather, plan)

    # ---- the sweep's other contexts (4096, 8192) and the ctx-512 layer latency
    sweep = run_sweep_contexts(rib, rank, world, device, args, pk)
    ctx512 = run_ctx512_latency(rib, device, args)

    # ---- batched ragged decode (64 sequences), sequence-sharded
    ragged = run_ragged(rib, rank, world, device, args, pk)
    parity["ragged_batch"] = ragged.pop("parity")

    # ---- prefill (tcgen05 kernel), one GPU's view
    prefill = run_prefill(rib, device, args, pk) if not args.no_prefill else None
    if prefill is not None and "unavailable" not in prefill:
        prefill["by_length"] = run_prefill_sweep(rib, device, args, pk)

    # ---- the full Qwen3-0.6B forward (one replica per GPU)
    full_model = run_full_model(rib, rank, world, device, args) if not args.no_model else None
    if full_model is not None and world > 1:   # the same sequence with the projections split too
        full_model["tensor_parallel"] = run_full_model(rib, rank, world, device, args, tp=True)
    if not args.no_model:
        parity["model"] = model_parity(rib, world, device)
    parity["pass"] = all(v.get("pass", False) for v in parity.values())

    device_status = importlib.import_module("roofline-inference_b200._lib").take_device_status()
    if gather is not None:
        gather.close()
    if rank != 0:
        if world > 1:
            torch.distributed.destroy_process_group()
        return
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"decode sweep: {N_LAYERS} layers x ctx {CTX} (+1 new token), "
                               f"16q/8kv heads, head_dim 128, independent seeded BF16 N(0,1) "
                               f"caches",
                   "launch": "layer-batched (one decode launch per step for all 28 layers)",
                   "parallelism": f"kv-head shard x{world}" + (
                       ", all-gather fused into the decode kernel (NVLink peer stores)"
                       if world > 1 else ""),
                   "l2": f"inputs {bytes_step_total / 1e9:.2f} GB per step > 126 MB L2, no flush",
                   "kv_bytes_per_step": bytes_step_total},
        "pct_of_hbm_peak": value / pk["hbm_gbs"] / world * 100.0,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / pk["hbm_gbs"],
                     "traffic": None if ratio is None else bytes_launch_local * ratio,
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of the "
                                       "one-GPU launch of the same kernel "
                                       "(profiles/decode_kernel_traffic.json), scaled by keys",
                     "kernel": kernel,
                     "peak_source": pk["source"] + " hbm_gbs (copy, burst)",
                     "bytes_per_launch": bytes_launch_local, "launch_ms": launch_ms},
        "nccl_allgather_baseline": nccl,
        "per_layer_launches": {"value": per_layer_gbs, "unit": "GB/s", "ms_per_step": per_layer_ms,
                               "frac": per_layer_gbs / pk["hbm_gbs"]},
        "sweep_contexts": sweep,
        "decode_ctx512": ctx512,
        "prefill": prefill,
        "full_model": full_model,
        "ragged_batch": ragged,
        "e2e": e2e,
        "gpu_launches": args.steps,
        "device_status": device_status,
        "clocks": clk,
        "parity": parity,
    }
    rl = importlib.import_module("roofline-inference_b200.roofline_line")
    dline = rl.decode_attention_line(w["n"])
    line["reference_line"] = {
        "model": "Level-A bound max(FLOPs/P, bytes/B, exps/rate), configs/b200.yaml "
                 "(measured peaks), attention only, cold start",
        "decode_sweep": {"time_s": dline["time_s"] / world, "bottleneck": dline["bottleneck"],
                         "measured_s": ms * 1e-3,
                         "fraction": dline["time_s"] / world / (ms * 1e-3)},
    }
    if prefill and "ms" in prefill:
        pline = rl.prefill_attention_line(PREFILL_L)
        line["reference_line"]["prefill_32k"] = {
            "time_s": pline["time_s"], "bottleneck": pline["bottleneck"],
            "measured_s": prefill["ms"] * 1e-3,
            "fraction": pline["time_s"] / (prefill["ms"] * 1e-3)}
    if world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_decode_sample()
    print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def run_ragged(rib, rank, world, device, args, pk):
    """Batched ragged decode: 64 sequences, contexts U[512, 32768] (seeded),
    one contiguous cache each, one new token each.  Sequences are balanced
    over the ranks by total context (LPT); at N > 1 every rank's outputs
    reach every rank through the decode kernel's NVLink stores (all 16 heads
    per rank, one slot per sequence).  Metric: KV bytes / step time."""
    wl = importlib.import_module("roofline-inference_b200.workloads")
    sh = importlib.import_module("roofline-inference_b200.sharding")
    lens = wl.ragged_lengths(64, 512, 32768, seed=0)
    assign = sh.balance_sequences(lens, world)
    slots = sh.slots_per_rank(assign)
    mine = assign[rank]
    cap = wl.round_cap(max(lens))
    pool = torch.zeros((slots, 2, NKV_TOTAL, cap, 128), dtype=torch.bfloat16, device=device)
    q = torch.zeros((slots, 16, 128), dtype=torch.bfloat16, device=device)
    my_lens = []
    for j, i in enumerate(mine):
        pool[j, :, :, :lens[i]] = wl.randn_bf16((2, NKV_TOTAL, lens[i], 128), seed=1000 + i,
                                                device=device)
        q[j] = wl.randn_bf16((16, 128), seed=2000 + i, device=device)
        my_lens.append(lens[i])
    my_lens += [1] * (slots - len(mine))  # padding slots: one key, output ignored
    L = rib.load_library()
    stride = pool[0].numel() * 2
    ptrs = torch.tensor([pool.data_ptr() + j * stride for j in range(slots)], dtype=torch.int64,
                        device=device)
    lens_d = torch.tensor(my_lens, dtype=torch.int32, device=device)
    max_n = max(my_lens)
    ws = torch.zeros(L.rib_decode_workspace_bytes(slots, max_n, NKV_TOTAL), dtype=torch.uint8,
                     device=device)
    out = torch.empty((slots, 16, 128), dtype=torch.bfloat16, device=device)
    stream = torch.cuda.current_stream(device)
    gather = None
    if world > 1:
        gather = importlib.import_module("roofline-inference_b200.nvlink_gather").NVLinkGather(
            slots, 16, device)

    def step():
        if gather is not None:
            gather.decode(q, ptrs, lens_d, max_n, cap, 128 ** -0.5, ws)
        else:
            st = L.rib_decode_attention_batched(q.data_ptr(), ptrs.data_ptr(), lens_d.data_ptr(),
                                                slots, max_n, cap, 16, NKV_TOTAL, 128 ** -0.5,
                                                out.data_ptr(), ws.data_ptr(), ws.numel(),
                                                stream.cuda_stream)
            if st != 0:
                raise RuntimeError(f"ragged decode failed: status {st}")

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(args.steps):
        step()
    b.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(a.elapsed_time(b) / args.steps, world, device)
    # parity of the timed step's outputs: 4 sequences, wherever they ran
    gout = gather.output() if gather is not None else None
    errs = []
    for i in range(4):
        r = next(rr for rr in range(world) if i in assign[rr])
        j = assign[r].index(i)
        got = gout[j, 16 * r:16 * r + 16] if gout is not None else out[j]
        kv = wl.randn_bf16((2, NKV_TOTAL, lens[i], 128), seed=1000 + i, device=device)
        want = ref_attention(wl.randn_bf16((16, 128), seed=2000 + i, device=device)[:, None], kv[0], kv[1],
                             128 ** -0.5)[:, 0]
        errs.append(attention_errors(got, want))
        del kv
    parity = reduce_errors(errs, world, device)
    parity["sample"] = "sequences 0-3 (all 16 heads), read from the rank and slot that ran them"
    if gather is not None:
        gather.close()
    total = sum(4096 * n for n in lens)
    v = total / (ms * 1e-3) / 1e9
    return {"value": v, "unit": "GB/s", "ms_per_step": ms, "sequences": len(lens),
            "kv_bytes_per_step": total, "frac_of_hbm_peak_x_gpus": v / (pk["hbm_gbs"] * world),
            "sharding": f"sequences, LPT by context, {slots} slots per rank",
            "contexts": "U[512, 32768], seed 0", "parity": parity}


def run_e2e(rib, w, rank, world, device, args, gather, plan):
    """Same sweep through the public API: per step, copy the 28 layers' qkv
    rows of the new token from pinned host memory, run the fused
    norm + RoPE + append of all 28 layers (one launch, new token at position
    32768) and one layer-batched decode, and read the outputs back to pinned
    host memory."""
    wl = importlib.import_module("roofline-inference_b200.workloads")
    nkv, pos = w["nkv"], w["n"] - 1
    nq = 2 * nkv
    width = (nq + 2 * nkv) * 128
    qkv_host = torch.empty((N_LAYERS, width), dtype=torch.bfloat16).pin_memory()
    for layer in range(N_LAYERS):
        qkv_host[layer] = wl.randn_bf16((width,), seed=500000 + layer * 8 + rank)
    out_host = torch.empty((N_LAYERS, NKV_TOTAL * 2, 128), dtype=torch.bfloat16).pin_memory()
    qw = wl.norm_weights(1, device)
    kw = wl.norm_weights(2, device)
    qkv_dev = torch.empty((N_LAYERS, width), dtype=torch.bfloat16, device=device)
    lens = torch.full((N_LAYERS,), w["n"], dtype=torch.int32, device=device)
    pos_dev = torch.full((N_LAYERS,), pos, dtype=torch.int32, device=device)
    caps = torch.full((N_LAYERS,), w["cap"], dtype=torch.int32, device=device)
    caches = w["caches"]
    stream = torch.cuda.current_stream(device)
    launches = 2 if gather is not None else 1

    def step():
        qkv_dev.copy_(qkv_host, non_blocking=True)
        if gather is not None:
            # every layer's norm + RoPE + append in one launch (the layers as a batch of caches)
            q = rib.qk_norm_rope_append_batched(qkv_dev, qw, kw, pos_dev, plan.ptrs, caps, nq, nkv, 1e6)
            full = gather.decode(q, plan.ptrs, lens, w["n"], w["cap"], 128 ** -0.5, plan.ws)
        else:
            # the norm + RoPE + append of all 28 layers inside the decode launch
            full = rib.decode_attention_qkv(qkv_dev, qw, kw, 1e6, caches, lens, 128 ** -0.5, max_n=w["n"])
        out_host.copy_(full, non_blocking=True)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(args.steps):
        step()
    b.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(a.elapsed_time(b) / args.steps, world, device)
    total = N_LAYERS * 4096 * w["n"]
    return {"value": total / (ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": ms,
            "h2d_bytes_per_step": qkv_host.numel() * 2,
            "d2h_bytes_per_step": out_host.numel() * 2,
            "gpu_launches_per_step": launches,
            "path": ("qk_norm_rope_append_batched (28 layers, one launch) + NVLinkGather.decode (fused all-gather)"
                     if world > 1 else
                     "decode_attention_qkv (public API: the 28 layers' norm + RoPE + append fused into the decode launch)")}


def run_prefill(rib, device, args, pk):
    """Causal prefill attention at L = 32768 on one GPU (Q/K/V BF16 N(0,1),
    positions 0..L-1): FLOPs 4096 * L * (L + 1) per call."""
    wl = importlib.import_module("roofline-inference_b200.workloads")
    L = PREFILL_L
    cap = wl.round_cap(L)
    try:
        Q = wl.randn_bf16((16, L, 128), seed=71, device=device)
        K = torch.zeros((1, 8, cap, 128), dtype=torch.bfloat16, device=device)
        V = torch.zeros((1, 8, cap, 128), dtype=torch.bfloat16, device=device)
        K[0, :, :L] = wl.randn_bf16((8, L, 128), seed=72, device=device)
        V[0, :, :L] = wl.randn_bf16((8, L, 128), seed=73, device=device)
        rib.attention(Q, K, V, L, L, wl.SCALE)
    except ValueError as e:  # kernel not available in this build
        return {"unavailable": str(e)}
    torch.cuda.synchronize()
    reps = max(args.steps, 3)
    for _ in range(args.warmup):
        rib.attention(Q, K, V, L, L, wl.SCALE)
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(reps)]
    stream = torch.cuda.current_stream(device)
    for a, b in evs:
        a.record(stream)
        rib.attention(Q, K, V, L, L, wl.SCALE)
        b.record(stream)
    sm_mhz = sm_clock_mhz(device)  # sampled while the last launches still run
    torch.cuda.synchronize()
    ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
    flops = wl.prefill_flops(L)
    tf = flops / (ms * 1e-3) / 1e12
    # DRAM traffic of this very launch (L = 32768) from one ncu capture; K and V
    # re-reads depend on L and L2 residency, so no other L is scaled from it.
    rec = profile_traffic("prefill_kernel_traffic")
    traffic = None
    if rec is not None and int(rec["L"]) == L:
        traffic = float(rec["dram_bytes_read_per_launch"]) + float(rec["dram_bytes_write_per_launch"])
    # The loop runs back to back for reps * ms, long enough for the 1000 W cap to
    # lower the SM clock, so the sustained cuBLAS figure is reported beside the burst one.
    return {"value": tf, "unit": "TFLOP/s", "L": L, "ms": ms, "flops": flops, "launches": reps,
            "sm_mhz_in_loop": sm_mhz,
            "roofline": {"bound": "tensor", "achieved": tf, "peak": pk["bf16_tflops"],
                         "unit": "TFLOP/s", "frac": tf / pk["bf16_tflops"],
                         "peak_source": pk["source"] + " bf16_tflops (burst)",
                         "peak_sustained": pk["bf16_tflops_sustained"],
                         "frac_of_sustained": tf / pk["bf16_tflops_sustained"],
                         "traffic": traffic,
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of this launch "
                                           "(profiles/prefill_kernel_traffic.json)" if traffic else None,
                         "algorithmic_bytes": (2 * 16 + 2 * 8) * L * 128 * 2,  # Q, O, K, FP16 V once each
                         "kernel": "rib::prefill::prefill_kernel"}}


def run_prefill_sweep(rib, device, args, pk) -> dict:
    """Causal prefill at every prompt length of the prefill configuration,
    L in {16, 64, 256, 1024, 4096, 32768}, with the fused work in the timed
    call: per call the pre-norm qkv rows [L, 4096] go through the fused
    per-head RMSNorm + RoPE (theta 1e6, positions 0..L-1) + KV-cache append
    (rib.qk_norm_rope_append) and then the causal attention over the written
    cache (rib.attention), the order Engine.prefill runs them.

    Device time: the pair is captured once in a CUDA graph and replayed; L2 is
    flushed (a 256 MB write) before every replay and CUDA events bracket the
    replay alone.  Host-to-host time: the same pair called eagerly through
    the public API, back to back (the host path a short prompt pays).
    TFLOP/s counts the attention's 4096 L (L + 1) FLOPs; the append moves
    16 KiB per token (qkv read, Q and K/V written)."""
    wl = importlib.import_module("roofline-inference_b200.workloads")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    out = {}
    for L in (16, 64, 256, 1024, 4096, 32768):
        qkv, qw, kw = wl.prefill_qkv(L, seed=L + 3, device=device)
        cap = wl.round_cap(L)
        cache = torch.zeros((2, 8, cap, 128), dtype=torch.bfloat16, device=device)
        Lp = (L + 31) // 32 * 32

        def pair():
            Q = rib.qk_norm_rope_append(qkv, qw, kw, 0, 16, 8, wl.ROPE_THETA, cache, Lp)
            return rib.attention(Q, cache[0:1], cache[1:2], L, L, wl.SCALE)

        for _ in range(max(args.warmup, 3)):
            pair()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(device)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            pair()
            torch.cuda.synchronize()
            with torch.cuda.graph(g, stream=side):
                pair()
        torch.cuda.synchronize()
        reps = 10 if L == 32768 else 30
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(reps)]
        for a, b in evs:
            flush.zero_()
            a.record(stream)
            g.replay()
            b.record(stream)
        torch.cuda.synchronize()
        dev_ms = statistics.median(a.elapsed_time(b) for a, b in evs)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            pair()
        b.record(stream)
        torch.cuda.synchronize()
        eager_ms = a.elapsed_time(b) / reps
        del g
        fl = wl.prefill_flops(L)
        tf = fl / (dev_ms * 1e-3) / 1e12
        out[str(L)] = {"us_device": dev_ms * 1e3, "us_eager": eager_ms * 1e3, "tflops": tf,
                       "frac_of_bf16_peak": tf / pk["bf16_tflops"], "flops": fl,
                       "append_bytes": 16384 * L}
        del qkv, cache
        torch.cuda.empty_cache()
    return {"lengths": out, "unit": "TFLOP/s (attention FLOPs over the fused append + attention time)",
            "timing": "device: CUDA-graph replay of the pair, L2 flushed before each, median of 10-30; "
                      "eager: public API back to back"}


def sm_clock_mhz(device):
    """Current SM clock of `device` through NVML, or None."""
    try:
        import pynvml
        pynvml.nvmlInit()
        idx = device.index if device.index is not None else torch.cuda.current_device()
        return int(pynvml.nvmlDeviceGetClockInfo(pynvml.nvmlDeviceGetHandleByIndex(idx),
                                                 pynvml.NVML_CLOCK_SM))
    except Exception:
        return None


def run_sweep_contexts(rib, rank, world, device, args, pk):
    """The decode sweep at contexts 4096 and 8192 (28 layers, one layer-batched
    launch per step, this rank's KV heads; no cross-GPU exchange): whole-job
    GB/s = all ranks' K/V bytes / the max over ranks of the step time."""
    out = {}
    for ctx in (4096, 8192):
        w = make_decode_workload(rank, world, device, ctx=ctx)
        plan = DecodePlan(rib, w, device)
        for _ in range(max(3, args.warmup)):
            plan.launch()
        stream = torch.cuda.current_stream(device)
        barrier(world)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(args.steps):
            plan.launch()
        b.record(stream)
        torch.cuda.synchronize()
        ms = max_over_ranks(a.elapsed_time(b) / args.steps, world, device)
        gbs = N_LAYERS * 4096 * w["n"] / (ms * 1e-3) / 1e9
        out[str(ctx)] = {"value": gbs, "unit": "GB/s", "ms_per_step": ms,
                         "frac_of_hbm_peak_x_gpus": gbs / (pk["hbm_gbs"] * world),
                         "kv_bytes_per_step": N_LAYERS * 4096 * w["n"]}
        del plan, w
        torch.cuda.empty_cache()
    return out


def run_ctx512_latency(rib, device, args):
    """Single-layer decode at context 512 (the reference's CPU-runnable
    configuration): the fused norm + RoPE + append of the new token at
    position 512, then attention over 513 keys.  Device time per layer from a
    CUDA graph of 28 such layers (distinct caches), and host-to-host time of
    one eager layer through the public API (with a synchronise)."""
    wl = importlib.import_module("roofline-inference_b200.workloads")
    L = rib.load_library()
    layers, pos = N_LAYERS, 512
    cache = rib.Cache(layers, 8, 128, pos + 1, device=device)
    cache.storage[:, :, :, :pos].copy_(wl.randn_bf16(tuple(cache.storage[:, :, :, :pos].shape), seed=5,
                                                     device=device))
    st = wl.decode_step(pos, seed=1, device=device)
    posd = torch.tensor([pos], dtype=torch.int32, device=device)
    nk = torch.tensor([pos + 1], dtype=torch.int32, device=device)
    ptrs = torch.tensor([cache.kv[i].data_ptr() for i in range(layers)], dtype=torch.int64, device=device)
    q = torch.empty((16, 1, 128), dtype=torch.bfloat16, device=device)
    out = torch.empty((1, 16, 128), dtype=torch.bfloat16, device=device)
    ws = torch.zeros(int(L.rib_decode_workspace_bytes(1, cache.capacity, 8)), dtype=torch.uint8,
                     device=device)

    def layer(i):
        rib.qk_norm_rope_append_at(st.qkv, st.qw, st.kw, posd, 16, 8, 1e6, cache.kv[i], out=q)
        rc = L.rib_decode_attention_batched(q.data_ptr(), ptrs.data_ptr() + 8 * i, nk.data_ptr(), 1,
                                            cache.capacity, cache.capacity, 16, 8, wl.SCALE,
                                            out.data_ptr(), ws.data_ptr(), ws.numel(),
                                            torch.cuda.current_stream(device).cuda_stream)
        if rc != 0:
            raise RuntimeError(f"decode launch failed: status {rc}")

    side = torch.cuda.Stream(device=device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        layer(0)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        for i in range(layers):
            layer(i)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    reps = max(3, min(args.steps, 50))
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        g.replay()
    b.record()
    b.synchronize()
    dev_us = a.elapsed_time(b) * 1000 / (reps * layers)
    # eager, host to host: one layer through the public API per call
    for _ in range(3):
        layer(0)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(reps):
        layer(0)
        torch.cuda.synchronize()
    host_us = (time.perf_counter() - t0) * 1e6 / reps
    del g
    bytes_layer = 4096 * 512 + 3 * 4096 + 16384
    return {"us_per_layer_device": dev_us, "us_per_layer_host_sync": host_us, "layers": layers,
            "bytes_per_layer": bytes_layer,
            "path": "qk_norm_rope_append_at + decode_attention_batched (batch 1) per layer; device time "
                    "from a CUDA graph of 28 layers, host time from eager calls with a synchronise"}


def run_full_model(rib, rank, world, device, args, tp: bool = False):
    """Qwen3-0.6B forward with random N(0, 0.02) weights (28 layers, hidden
    1024, 16/8 heads, FFN 3072, vocab 151936, tied embeddings, BF16): the
    engine's CUDA-graph decode step at context 32768 (K/V seeded N(0, 1)), and
    a 4096-token prompt + 128 generated tokens through Engine.generate (host
    token ids in, host token ids out; wall clock).  At N > 1 one sequence runs
    KV-head sharded over all ranks (Engine(shard=True): each rank owns 8/N KV
    heads, the decode kernel gathers every head's output over NVLink, the
    rest of the layer runs on every rank); times are the max over ranks.
    With tp the projections are split too (Engine(tp=True): O / down partial
    sums and the argmax keys exchanged over NVLink inside the GEMV kernels;
    in prefill inside the tcgen05 GEMM's epilogue and the add_rms kernel).
    Each figure is reported against the full-model Level-A line (cold start)."""
    rl = importlib.import_module("roofline-inference_b200.roofline_line")
    cfg = rib.QWEN3_0_6B
    # the same seed on every rank: identical weights, as a sharded engine needs
    eng = rib.Engine(rib.random_weights(cfg, seed=11, device=device), shard=world > 1, tp=tp and world > 1)
    out = {"model": "Qwen3-0.6B, random-init N(0, 0.02) weights, BF16",
           "parallelism": (f"tensor parallel x{world}" if tp else f"kv-head shard x{world}") if world > 1
           else "1 GPU",
           "kv_heads_per_rank": eng.n_kv}

    # decode step at context 32768
    ctx, steps, warm = 32768, max(1, min(args.steps, 200)), max(3, min(args.warmup, 20))
    cache = eng.new_cache(ctx + 2 * (steps + warm) + 8)
    g = torch.Generator(device=device)
    g.manual_seed(12 + rank)     # this rank's KV heads
    for i in range(cfg.num_layers):
        cache.storage[i, :, :, :ctx].normal_(generator=g)
    cache.offset = ctx
    dg = eng.decode_graph(cache)
    dg.set_state(1, ctx)
    for _ in range(warm):
        dg.replay()
    stream = torch.cuda.current_stream(device)
    barrier(world)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        dg.replay()
    b.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(a.elapsed_time(b) / steps, world, device)
    line = rl.model_decode_line(cfg, ctx + warm)
    if world == 1:  # the same step as one persistent cooperative launch per token
        cache.offset = ctx + warm + steps
        pers = eng.persistent_decode(cache)
        pers.set_state(1, cache.offset)
        for _ in range(warm):
            pers.replay()
        torch.cuda.synchronize()
        a.record(stream)
        for _ in range(steps):
            pers.replay()
        b.record(stream)
        torch.cuda.synchronize()
        pms = a.elapsed_time(b) / steps
        out["decode_step_persistent"] = {
            "ms_per_token": pms, "tokens_per_s": 1000.0 / pms, "launches_per_step": 1,
            "path": "rib_qwen3_decode_step: one cooperative launch per token, 169 grid barriers",
            "fraction_of_line": line["time_s"] * 1e3 / pms}
        del pers
    out["decode_step"] = {
        "context": f"{ctx + warm}..{ctx + warm + steps}", "steps": steps, "ms_per_token": ms,
        "tokens_per_s": 1000.0 / ms, "launches_per_step": dg.launches_per_step,
        "path": "one CUDA-graph replay per token (embedding, 28 x [norm+QKV GEMV, split-KV decode "
                "attention with the qk-norm+RoPE+KV append fused in, O GEMV+residual, norm+gate/up "
                "GEMV+SwiGLU, down GEMV+residual], final norm + LM-head GEMV, argmax)"
                + ("; tensor parallel: O/down partial sums and argmax keys exchanged over NVLink "
                   "inside the GEMV and argmax kernels" if tp else ""),
        "reference_line_ms": line["time_s"] * 1e3, "reference_bottleneck": line["bottleneck"],
        "reference_line_scope": "one GPU (the whole model's bytes over one GPU's bandwidth)",
        "fraction_of_line": line["time_s"] * 1e3 / ms}
    del dg, cache
    torch.cuda.empty_cache()

    # a 4096-token prompt + 128 generated tokens
    P, G = 4096, 128
    prompt = torch.randint(0, cfg.vocab_size, (P,), generator=torch.Generator().manual_seed(13))
    prompt = prompt.tolist()
    list(eng.generate(prompt, max_tokens=G))          # warm-up: captures the session's graph
    ttft, dec, tot = [], [], []
    for _ in range(3):
        barrier(world)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        it = eng.generate(prompt, max_tokens=G)
        next(it)
        t1 = time.perf_counter()
        rest = list(it)
        t2 = time.perf_counter()
        if len(rest) != G - 1:
            raise RuntimeError(f"generated {len(rest) + 1} tokens, expected {G}")
        ttft.append(max_over_ranks(t1 - t0, world, device))
        dec.append(max_over_ranks(t2 - t1, world, device))
        tot.append(max_over_ranks(t2 - t0, world, device))
    rline = rl.request_line(cfg, P, G)
    t_ttft, t_dec, t_tot = statistics.median(ttft), statistics.median(dec), statistics.median(tot)
    out["request"] = {
        "prompt": P, "generated": G, "repeats": 3, "timing": "host wall clock, median",
        "ttft_ms": t_ttft * 1e3, "decode_tokens_per_s": (G - 1) / t_dec,
        "total_ms": t_tot * 1e3,
        "reference_line": {"ttft_ms": rline["ttft_s"] * 1e3, "total_ms": rline["total_s"] * 1e3},
        "fraction_ttft": rline["ttft_s"] / t_ttft, "fraction_total": rline["total_s"] / t_tot}
    if world > 1:
        out["request"]["prefill_exchange"] = (
            "O / down row partials stored by the tcgen05 GEMM's epilogue into their owner rank's buffer over "
            "NVLink; one kernel reduces, stores the BF16 rows into every rank and applies add_rms (no NCCL)"
            if tp else "attention outputs all-gathered with NCCL (all_gather_into_tensor)")
    if world == 1 and not tp:
        out["batched_decode"] = run_model_batch(rib, eng, device, args)
        out["serving"] = run_serving(rib, eng, device)
    eng.close()  # collective when sharded
    return out


def run_model_batch(rib, eng, device, args):
    """Batched ragged decode of the whole model on one GPU: 64 independent
    sequences with contexts drawn U[512, 4096] (seeded), each in its own cache
    (K/V copied from a seeded N(0, 1) block), one token each per step through
    BatchDecoder (GEMM projections over the 64 rows, batched append, ragged
    split-KV attention, row argmax).  Tokens/s and the step against the
    batched Level-A line (weights read once per step, every sequence's K/V)."""
    rl = importlib.import_module("roofline-inference_b200.roofline_line")
    cfg = eng.cfg
    steps, warm = max(1, min(args.steps, 20)), 3
    ctxs, dec = batch_workload(eng, device, steps + warm + 2)
    tok = torch.arange(64, dtype=torch.int32, device=device)
    for _ in range(warm):
        tok = dec.step(tok)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(device)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        tok = dec.step(tok)
    b.record(stream)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    line = rl.model_batch_decode_line(cfg, [c + warm for c in ctxs])
    res = {"sequences": 64, "contexts": "U[512, 4096], seed 0", "steps": steps, "ms_per_step": ms,
           "tokens_per_s": 64 * 1000.0 / ms, "kv_bytes_per_step": sum(ctxs) * cfg.num_layers * 4096,
           "reference_line_ms": line["time_s"] * 1e3, "reference_bottleneck": line["bottleneck"],
           "fraction_of_line": line["time_s"] * 1e3 / ms,
           "launches_per_step": dec.launches_per_step,
           "path": "BatchDecoder.step replayed from one CUDA graph: cuBLAS GEMMs for the projections at 64 rows "
                   "(faster there than this package's few-row and tiled GEMMs), SwiGLU kernel, "
                   "rib_qk_norm_rope_append_batched, rib_decode_attention_ragged, add_rms kernels, "
                   "cuBLAS FP32-output LM-head GEMM, rib_argmax_rows_f32"}
    del dec
    torch.cuda.empty_cache()
    return res


def run_serving(rib, eng, device):
    """Continuous batching: 128 requests (prompts U[128, 2048] tokens, outputs
    U[32, 256] tokens, seeded), all submitted at once, served by the
    Scheduler with 64 decode slots, 4096-token prefill chunks and a KV arena
    for 64 requests of the largest size.  Host wall clock around run(), after
    two short warm-up requests (graph capture, first cuBLAS calls)."""
    g = torch.Generator().manual_seed(21)
    n = 128
    plens = torch.randint(128, 2049, (n,), generator=g).tolist()
    outs = torch.randint(32, 257, (n,), generator=g).tolist()
    prompts = [torch.randint(0, eng.cfg.vocab_size, (k,), generator=g).tolist() for k in plens]
    s = rib.Scheduler(eng, pool_rows=64 * 2560, slots=64, max_len=2560, chunk=4096)
    for k in range(2):  # warm-up (untimed): captures the step's graph, first cuBLAS calls
        s.submit(torch.randint(0, eng.cfg.vocab_size, (64 + k,), generator=g).tolist(), 4)
    s.run()
    warm_steps, warm_decode = s.steps, s.decode_steps
    s.finished.clear()
    for p, m in zip(prompts, outs):
        s.submit(p, m)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    res = s.run()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    gen = sum(len(v) for v in res.values())
    out = {"requests": n, "prompt_tokens": sum(plens), "generated_tokens": gen, "wall_s": wall,
           "output_tokens_per_s": gen / wall, "total_tokens_per_s": (gen + sum(plens)) / wall,
           "scheduler_steps": s.steps - warm_steps, "decode_steps": s.decode_steps - warm_decode,
           "mean_active_slots": (gen - n) / max(1, s.decode_steps - warm_decode),
           "config": "prompts U[128, 2048], outputs U[32, 256], seed 21; 64 slots, chunk 4096, "
                     "arena 64 x 2560 rows",
           "timing": "host wall clock around Scheduler.run, after a two-request warm-up that captures "
                     "the step's CUDA graph"}
    del s
    torch.cuda.empty_cache()
    return out


def batch_workload(eng, device, extra: int):
    """64 sequences with contexts U[512, 4096] (seed 0), each in its own cache
    with room for `extra` more tokens, K/V copied from a seeded N(0, 1) block;
    returns the contexts and a captured BatchDecoder over the caches."""
    wl = importlib.import_module("roofline-inference_b200.workloads")
    batch_mod = importlib.import_module("roofline-inference_b200.batch")
    cfg = eng.cfg
    ctxs = wl.ragged_lengths(64, 512, 4096, seed=0)
    src = wl.randn_bf16((2, cfg.num_kv_heads, max(ctxs), 128), seed=14, device=device)
    caches = []
    for c in ctxs:
        cache = eng.new_cache(c + extra)
        cache.storage[:, :, :, :c].copy_(src[None, :, :, :c].expand(cfg.num_layers, -1, -1, -1, -1))
        cache.offset = c
        caches.append(cache)
    return ctxs, batch_mod.BatchDecoder(eng, caches).capture()


def run_case(case: str):
    """Bounded workloads for ncu captures: decode-small is the layer-batched
    decode over 4 layers at ctx 32768 (537 MB of KV, above L2, 3 launches;
    the stream-K kernel); decode-28 is the bench's own launch (28 layers,
    3.76 GB of KV, the split kernel; 3 launches, for one-pass metrics only);
    prefill-small is causal prefill at L = 16384 (128 MB of Q/K/V, above L2;
    3 launches), prefill-32k the same at L = 32768 (the bench's launch);
    decode-4k is the 28-layer sweep at ctx 4096 (470 MB of KV, the stream-K
    decode kernel; 3 launches); model-decode is the
    Qwen3-0.6B decode step at context 4096 (1.19 GB of weights and 0.47 GB of
    K/V, above L2): the graph's eager
    warm-up step and 3 replays of 143 launches each (the append fused into
    the decode attention launch); model-batch is the
    64-sequence ragged batched decode step (contexts U[512, 4096], 17.9 GB
    of K/V): the capture's eager warm-up step and 3 graph replays;
    model-prefill is three 4096-token prefills of Qwen3-0.6B (last row's
    logits), the TTFT path of the request benchmark; gemm is one launch of
    each Qwen3 prefill projection at 4096 tokens (O, gate/up + SwiGLU, down,
    QKV + norm + RoPE + append); tp-exchange is the tensor-parallel prefill
    exchange of one rank (M = 32768 rows, K = 1024, hidden 1024: 128 MB of
    FP32 partials, above L2): three pairs of the owner-slot GEMM and the
    reduce + gather + add_rms kernel, each followed by the plain FP32 GEMM of
    the same shape."""
    rib = load_rib()
    wl = importlib.import_module("roofline-inference_b200.workloads")
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    if case in ("decode-small", "decode-4k", "decode-28"):
        w = make_decode_workload(0, 1, device, layers=4) if case == "decode-small" else \
            make_decode_workload(0, 1, device, ctx=4096) if case == "decode-4k" else \
            make_decode_workload(0, 1, device)
        plan = DecodePlan(rib, w, device)
        for _ in range(3):
            plan.launch()
    elif case == "model-decode":
        eng = rib.Engine(rib.random_weights(rib.QWEN3_0_6B, seed=11, device=device))
        ctx = 4096
        cache = eng.new_cache(ctx + 64)
        g = torch.Generator(device=device)
        g.manual_seed(12)
        for i in range(rib.QWEN3_0_6B.num_layers):
            cache.storage[i, :, :, :ctx].normal_(generator=g)
        cache.offset = ctx
        dg = eng.decode_graph(cache)
        dg.set_state(1, ctx)
        for _ in range(3):
            dg.replay()
    elif case == "model-prefill":
        eng = rib.Engine(rib.random_weights(rib.QWEN3_0_6B, seed=11, device=device))
        toks = torch.randint(0, rib.QWEN3_0_6B.vocab_size, (4096,), generator=torch.Generator().manual_seed(13))
        toks = toks.to(torch.int32).to(device)
        for _ in range(3):
            eng.prefill(toks, eng.new_cache(4096 + 256), last=True)
    elif case == "gemm":
        G = importlib.import_module("roofline-inference_b200.gemm")
        M = 4096
        x = wl.randn_bf16((M, 1024), seed=81, device=device)
        for N, K, epi in ((1024, 2048, "bf16"), (6144, 1024, "swiglu"), (1024, 3072, "bf16")):
            A = x if K == 1024 else wl.randn_bf16((M, K), seed=K, device=device)
            W = wl.randn_bf16((N, K), seed=N, device=device, scale=0.02)
            G.gemm(A, W, epi=epi)
        W = wl.randn_bf16((4096, 1024), seed=82, device=device, scale=0.02)
        qw, kw = wl.norm_weights(1, device), wl.norm_weights(2, device)
        cache = torch.zeros((2, 8, M, 128), dtype=torch.bfloat16, device=device)
        G.gemm_qkv_rope(x, W, qw, kw, G.rope_table(0, M, 1e6, device), 0, 16, 8, cache, M)
    elif case == "tp-exchange":
        G = importlib.import_module("roofline-inference_b200.gemm")
        T = importlib.import_module("roofline-inference_b200.tp")
        M, K, H = 32768, 1024, 1024
        ex = T.PrefillExchange(H, M, device, local=True)
        A = wl.randn_bf16((M, K), seed=91, device=device)
        W = wl.randn_bf16((H, K), seed=92, device=device, scale=K ** -0.5)
        h = wl.randn_bf16((M, H), seed=93, device=device)
        nw = (1.0 + 0.1 * wl.randn_bf16((H,), seed=94, device=device).float()).to(torch.bfloat16)
        out = torch.empty_like(h)
        for _ in range(3):
            ex.project_add_rms(A, W, h, nw, out)
            G.gemm(A, W, epi="f32", small=False)
        ex.close()
    elif case == "model-batch":
        eng = rib.Engine(rib.random_weights(rib.QWEN3_0_6B, seed=11, device=device))
        _, dec = batch_workload(eng, device, 8)
        tok = torch.arange(64, dtype=torch.int32, device=device)
        for _ in range(3):
            tok = dec.step(tok)
    else:
        L = 32768 if case == "prefill-32k" else 16384
        Q = wl.randn_bf16((16, L, 128), seed=71, device=device)
        K = wl.randn_bf16((1, 8, L, 128), seed=72, device=device)
        V = wl.randn_bf16((1, 8, L, 128), seed=73, device=device)
        for _ in range(3):
            rib.attention(Q, K, V, L, L, wl.SCALE)
    torch.cuda.synchronize()
    print(f"case {case} done")


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-model", action="store_true", help="skip the full Qwen3-0.6B forward")
    ap.add_argument("--case", choices=["decode-small", "decode-4k", "decode-28", "prefill-small", "prefill-32k",
                                       "model-decode",
                                       "model-prefill", "gemm", "tp-exchange",
                             "model-batch"], default=None,
                    help="run a bounded case for profiling (ncu) and exit")
    args = ap.parse_args()
    if args.case:
        run_case(args.case)
        return
    if args.warmup < 3 and args.impl == "ours":
        print("note: fewer than 3 warm-up steps", file=sys.stderr)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
