"""CPU: the B200 device spec follows the reference's schema, and the
attention reference lines use the reference's own work counts.

When a checkout of the reference is found (REFERENCE_ROOT; by default the
one the build container mounts), the spec is loaded with the reference's
src/roofline/device.py:load_device and the counts are compared with
src/roofline/workload.py:decode/prefill for Qwen3-0.6B; without it those
tests skip and the closed-form checks still run."""
from __future__ import annotations

import importlib
import sys
from pathlib import Path

import pytest

from oracle.msl.runner import reference_root

REF_SRC = reference_root() / "src"
REF_MODEL = reference_root() / "configs" / "models" / "qwen3_0.6b.yaml"


@pytest.fixture(scope="module")
def rl():
    return importlib.import_module("roofline-inference_b200.roofline_line")


@pytest.fixture(scope="module")
def reference_roofline():
    if not (REF_SRC / "roofline").exists():
        pytest.skip("reference roofline package not mounted")
    sys.path.insert(0, str(REF_SRC))
    return importlib.import_module("roofline")


def test_spec_loads_with_reference_loader(rl, reference_roofline):
    dev = reference_roofline.load_device(rl.SPEC)
    assert dev.engine("gpu").peak_flops("bf16").effective == pytest.approx(1.6526e15)
    assert dev.bandwidth("gpu") == pytest.approx(6.5427e12)
    assert dev.engine("gpu").special["exp"].effective == pytest.approx(4.653e12)
    assert [lv.name for lv in dev.hierarchy] == ["sm", "chip"]


def test_counts_match_reference_workloads(rl, reference_roofline):
    model = reference_roofline.load_model(REF_MODEL)
    ctx = 32768
    w = reference_roofline.decode(model, 1, ctx)
    line = rl.decode_attention_line(ctx + 1)  # keys = context + the new token
    assert line["flops"] == w.flops["attention"]
    # KV read of the cached context; the line also reads the new token's K/V
    assert line["dram_bytes"] - 28 * 4096 - 28 * 2 * 16 * 128 * 2 == w.bytes["kv_read"]
    p = reference_roofline.prefill(model, 1, 4096, prune_final=False)
    pl = rl.prefill_attention_line(4096)
    assert 28 * pl["flops"] == p.flops["attention"]
    # reference physical bound of its whole decode workload on this device runs
    b = reference_roofline.physical_bound(w, reference_roofline.load_device(rl.SPEC),
                                          initial_resident_bytes=0)
    assert b.bottleneck == "dram_bandwidth" and b.time_s > 0


def test_lines_closed_form(rl):
    spec = rl.load_spec()
    d = rl.decode_attention_line(32769)
    assert d["bottleneck"] == "dram_bandwidth"
    assert d["time_s"] == pytest.approx((28 * 4096 * 32769 + 28 * 8192) / spec["bandwidth"])
    p = rl.prefill_attention_line(32768)
    assert p["flops"] == 4096 * 32768 * 32769
    assert p["bottleneck"] == "compute"
    assert p["time_s"] == pytest.approx(4096 * 32768 * 32769 / spec["bf16"])
    assert rl.fraction(p, 2 * p["time_s"]) == pytest.approx(0.5)


def test_model_lines_match_reference(rl, reference_roofline):
    """Full-model lines equal the reference's own physical bound (cold start)
    for Qwen3-0.6B on configs/b200.yaml."""
    import importlib as _il
    cfg = _il.import_module("roofline-inference_b200").QWEN3_0_6B
    model = reference_roofline.load_model(REF_MODEL)
    dev = reference_roofline.load_device(rl.SPEC)
    for ctx in (512, 4096, 32768):
        w = reference_roofline.decode(model, 1, ctx)
        b = reference_roofline.physical_bound(w, dev, initial_resident_bytes=0)
        line = rl.model_decode_line(cfg, ctx)
        assert line["flops"] == w.total_flops
        assert line["dram_bytes"] == pytest.approx(b.traffic["total"])
        assert line["time_s"] == pytest.approx(b.time_s)
    for p in (16, 1024, 4096):
        w = reference_roofline.prefill(model, 1, p)
        b = reference_roofline.physical_bound(w, dev, initial_resident_bytes=0)
        line = rl.model_prefill_line(cfg, p)
        assert line["flops"] == w.total_flops
        assert line["dram_bytes"] == pytest.approx(b.traffic["total"])
        assert line["time_s"] == pytest.approx(b.time_s)


def test_request_line_closed_form(rl):
    import importlib as _il
    cfg = _il.import_module("roofline-inference_b200").QWEN3_0_6B
    r = rl.request_line(cfg, 4096, 128)
    assert r["ttft_s"] == pytest.approx(rl.model_prefill_line(cfg, 4096)["time_s"])
    assert r["decode_first_s"] == pytest.approx(rl.model_decode_line(cfg, 4096)["time_s"])
    assert r["total_s"] == pytest.approx(r["ttft_s"] + r["decode_s"])
    d = rl.model_decode_line(cfg, 32768)
    assert d["bottleneck"] == "dram_bandwidth"
    assert 4.9e9 < d["dram_bytes"] < 5.0e9          # 1.19 GB weights + 3.76 GB K/V


def test_batch_decode_line_matches_reference(rl, reference_roofline):
    """Equal contexts: the batched line is the reference's decode(model, B, ctx)."""
    import importlib as _il
    cfg = _il.import_module("roofline-inference_b200").QWEN3_0_6B
    model = reference_roofline.load_model(REF_MODEL)
    dev = reference_roofline.load_device(rl.SPEC)
    w = reference_roofline.decode(model, 8, 4096)
    b = reference_roofline.physical_bound(w, dev, initial_resident_bytes=0)
    line = rl.model_batch_decode_line(cfg, [4096] * 8)
    assert line["flops"] == w.total_flops
    assert line["dram_bytes"] == pytest.approx(b.traffic["total"])
    assert line["time_s"] == pytest.approx(b.time_s)
