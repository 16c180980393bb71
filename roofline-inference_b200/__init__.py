"""B200-native (sm_100a) Qwen3 attention hot path, and the Qwen3 forward around it.

Drop-in for the attention entry points of the reference's v2 engine
(aeilot/roofline-inference, agent-test/v2): fused QK-RMSNorm + RoPE (+ KV
append), split-KV GQA decode attention and tcgen05/TMEM causal prefill
attention, implemented as CUDA kernels behind a C ABI
(include/rib_attention.h) and called from these thin PyTorch wrappers.

The directory name contains a hyphen, so it is imported with importlib:
    sys.path.insert(0, <repository root>)
    rib = importlib.import_module("roofline-inference_b200")
"""
from . import _lib
from .attention import attention, decode_attention, decode_attention_batched, decode_attention_qkv
from .cache import Cache
from .kernels import (add_rms, argmax, embedding, gemv, qk_norm_rope, qk_norm_rope_append,
                      qk_norm_rope_append_at, qk_norm_rope_append_batched, qk_norm_rope_prefill, rms_norm,
                      swiglu)
from .model import QWEN3_0_6B, DecodeGraph, Engine, Qwen3Config, Qwen3Weights, random_weights
from .batch import BatchDecoder, SlotDecoder, generate_batch
from .pool import KVPool, PoolFull
from .scheduler import Request, Scheduler

__all__ = [
    "BatchDecoder",
    "Cache",
    "DecodeGraph",
    "Engine",
    "KVPool",
    "PoolFull",
    "QWEN3_0_6B",
    "Qwen3Config",
    "Qwen3Weights",
    "Request",
    "Scheduler",
    "SlotDecoder",
    "add_rms",
    "argmax",
    "embedding",
    "gemv",
    "generate_batch",
    "qk_norm_rope_append_at",
    "qk_norm_rope_append_batched",
    "random_weights",
    "rms_norm",
    "swiglu",
    "attention",
    "decode_attention",
    "decode_attention_batched",
    "decode_attention_qkv",
    "qk_norm_rope",
    "qk_norm_rope_append",
    "qk_norm_rope_prefill",
    "build",
    "load_library",
]


def build(force: bool = False, verbose: bool = False):
    """Compiles the CUDA extension for sm_100a (in-tree .so)."""
    return _lib.build(force=force, verbose=verbose)


def load_library():
    """Builds if needed and loads the C-ABI library; raises if it cannot."""
    return _lib.load()
