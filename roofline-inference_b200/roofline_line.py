"""Level-A reference lines for the attention scenarios on B200.

Restates the reference's calibrated resource bound
    T >= max(FLOPs / P_peak, DRAM bytes / B, exp count / exp rate)
(src/roofline/bound.py:96-145, README.md:76-84) for the attention-only
workloads this repository measures, using configs/b200.yaml, which follows
the reference's device-spec schema (src/roofline/device.py:102-130).  Each
measured number is reported as a fraction of the line: line time / measured
time (1.0 = at the bound).

Counts follow src/roofline/workload.py:
  decode   one new token per sequence attends n keys: FLOPs 2*H*d*(keys +
           values) per layer (workload.py:149), KV bytes 2*nkv*d*2 per key
           (workload.py:156), one exp per score; q in and o out are added.
  prefill  causal, pairs = qL*off + qL(qL+1)/2: FLOPs 4*H*d*pairs
           (workload.py:176-179), one exp per score; Q, K, V read and O
           written once (the resident-input credit is 0: a cold start,
           bound.py:96-105 with initial_resident_bytes=0).
"""
from __future__ import annotations

from pathlib import Path

import yaml

SPEC = Path(__file__).resolve().parent / "configs" / "b200.yaml"


def _eff(q: dict) -> float:
    """Quantity.effective (device.py:24-26): measured overrides value."""
    return float(q["measured"]) if q.get("measured") is not None else float(q["value"])


def load_spec(path: str | Path = SPEC) -> dict:
    data = yaml.safe_load(Path(path).read_text())
    gpu = data["engines"]["gpu"]
    return {
        "name": data["name"],
        "bf16": _eff(gpu["compute"]["bf16"]),
        "bf16_datasheet": float(gpu["compute"]["bf16"]["value"]),
        "bandwidth": min(_eff(gpu["bandwidth"]), _eff(data["memory"]["total_bandwidth"])),
        "bandwidth_datasheet": float(gpu["bandwidth"]["value"]),
        "exp": _eff(gpu["special"]["exp"]),
    }


def _line(flops: float, dram_bytes: float, exps: float, spec: dict) -> dict:
    res = {"compute": flops / spec["bf16"], "dram_bandwidth": dram_bytes / spec["bandwidth"],
           "exp": exps / spec["exp"]}
    t = max(res.values())
    return {"time_s": t, "bottleneck": max(res, key=res.get), "resource_time_s": res,
            "flops": flops, "dram_bytes": dram_bytes, "exps": exps,
            "device": spec["name"]}


def decode_attention_line(n_keys: int, layers: int = 28, batch: int = 1, nq: int = 16,
                          nkv: int = 8, head_dim: int = 128, spec: dict | None = None) -> dict:
    """Decode attention over `n_keys` keys (new token included) per layer."""
    spec = spec or load_spec()
    flops = 2 * layers * nq * head_dim * (n_keys + n_keys) * batch
    kv = layers * batch * 2 * nkv * head_dim * 2 * n_keys
    qo = layers * batch * 2 * nq * head_dim * 2
    exps = layers * batch * nq * n_keys
    return _line(flops, kv + qo, exps, spec)


def prefill_attention_line(qL: int, kL: int | None = None, nq: int = 16, nkv: int = 8,
                           head_dim: int = 128, spec: dict | None = None) -> dict:
    """Causal prefill attention of one layer."""
    spec = spec or load_spec()
    kL = qL if kL is None else kL
    pairs = qL * (kL - qL) + qL * (qL + 1) // 2
    flops = 4 * nq * head_dim * pairs
    dram = 2 * head_dim * (2 * nq * qL + 2 * nkv * kL)  # Q in, O out, K and V in
    return _line(flops, dram, nq * pairs, spec)


def fraction(line: dict, measured_s: float) -> float:
    """Line time / measured time: 1.0 means the measurement sits on the bound."""
    return line["time_s"] / measured_s


# ------------------------------------------------------------------ full model
# Qwen3 forward lines, restating src/roofline/workload.py:decode/prefill and
# bound.py:request_time for a dense GQA model with tied embeddings; cold start
# (initial_resident_bytes = 0 in bound.py:96-116).

def _params(cfg) -> dict:
    d, q, kv, f = cfg.hidden_size, cfg.q_dim, cfg.kv_dim, cfg.intermediate_size
    linear = d * q + 2 * d * kv + q * d + 3 * d * f                  # model.py layer_linear_params
    norms = 2 * d + 2 * cfg.head_dim                                   # model.py layer_norm_params (qk_norm)
    return {"linear": linear, "norms": norms,
            "weights_read": (cfg.num_layers * (linear + norms) + d + cfg.vocab_size * d) * 2}


def model_decode_line(cfg, context: int, batch: int = 1, spec: dict | None = None) -> dict:
    """One decode step with `context` cached tokens (workload.py:decode)."""
    spec = spec or load_spec()
    P, L = _params(cfg), cfg.num_layers
    keys = context + 1
    flops = (2 * L * P["linear"] * batch + 2 * L * cfg.num_heads * cfg.head_dim * 2 * keys * batch
             + 2 * cfg.vocab_size * cfg.hidden_size * batch)
    vec = L * cfg.kv_dim * 2                                           # kv_bytes_per_token // 2
    dram = P["weights_read"] + 2 * batch * 4 + batch * 2 * context * vec + batch * 2 * vec
    return _line(flops, dram, L * cfg.num_heads * keys * batch, spec)


def model_prefill_line(cfg, prompt_len: int, batch: int = 1, spec: dict | None = None) -> dict:
    """Prefill of a prompt with logits for its last position only
    (workload.py:prefill with prune_final=True)."""
    spec = spec or load_spec()
    P, L, p = _params(cfg), cfg.num_layers, prompt_len
    pairs = p * (p + 1) // 2
    d, q, f = cfg.hidden_size, cfg.q_dim, cfg.intermediate_size
    dead = 2 * d * q + 3 * d * f
    linear = 2 * L * P["linear"] * batch * p - 2 * dead * batch * (p - 1)
    final_scores = cfg.num_heads * batch * p
    attention = 4 * cfg.head_dim * (cfg.num_heads * pairs * batch * (L - 1) + final_scores)
    flops = linear + attention + 2 * cfg.vocab_size * d * batch
    dram = P["weights_read"] + (batch * p + batch) * 4 + batch * p * 2 * L * cfg.kv_dim * 2
    exps = cfg.num_heads * pairs * batch * (L - 1) + final_scores
    return _line(flops, dram, exps, spec)


def request_line(cfg, prompt_len: int, gen: int, spec: dict | None = None) -> dict:
    """T = TTFT(L) + sum_{i=1}^{gen-1} T_decode(L + i - 1) (bound.py:193-217)."""
    spec = spec or load_spec()
    ttft = model_prefill_line(cfg, prompt_len, spec=spec)["time_s"]
    steps = [model_decode_line(cfg, prompt_len + i - 1, spec=spec)["time_s"] for i in range(1, gen)]
    return {"ttft_s": ttft, "decode_s": sum(steps), "total_s": ttft + sum(steps),
            "decode_first_s": steps[0] if steps else 0.0, "decode_last_s": steps[-1] if steps else 0.0,
            "prompt_len": prompt_len, "gen": gen, "device": spec["name"]}


def model_batch_decode_line(cfg, contexts: list[int], spec: dict | None = None) -> dict:
    """One decode step of len(contexts) independent sequences: every weight is
    read once for the whole batch (workload.py:decode with batch > 1 reads
    _weights_read_bytes once), each sequence reads its own cached K/V."""
    spec = spec or load_spec()
    lines = [model_decode_line(cfg, c, spec=spec) for c in contexts]
    w = _params(cfg)["weights_read"]
    dram = w + sum(l["dram_bytes"] - w for l in lines)
    return _line(sum(l["flops"] for l in lines), dram, sum(l["exps"] for l in lines), spec)
