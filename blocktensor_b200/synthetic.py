"""Seeded synthetic workloads (random-init models, prompt ids) and model shapes.

The generator is counter based: element i of stream s under seed k is a
function of (k, s, i) only, computed with splitmix64 integer hashing, so the
device generator (bt_engine_generate), this module and the CPU oracle produce
identical values.  Normal-looking values are the sum of four 16-bit uniforms,
centred and scaled to the requested sigma.
"""
from __future__ import annotations

import numpy as np

from .native import ModelConfig

M64 = (1 << 64) - 1
STREAM_PROMPT = 0xF000


def splitmix64(z: np.ndarray) -> np.ndarray:
    z = (z + np.uint64(0x9E3779B97F4A7C15)).astype(np.uint64)
    z = ((z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)).astype(np.uint64)
    z = ((z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)).astype(np.uint64)
    return z ^ (z >> np.uint64(31))


def _sm64_int(z: int) -> int:
    z = (z + 0x9E3779B97F4A7C15) & M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
    return z ^ (z >> 31)


def stream_base(seed: int, stream: int) -> int:
    return _sm64_int(_sm64_int(seed) ^ ((stream * 0xD1B54A32D192ED03) & M64))


def tokens(seed: int, n: int, vocab: int, stream: int = STREAM_PROMPT) -> np.ndarray:
    """Uniform token ids in [0, vocab)."""
    base = np.uint64(stream_base(seed, stream))
    with np.errstate(over="ignore"):
        h = splitmix64(base + np.arange(n, dtype=np.uint64))
    return ((h >> np.uint64(32)) % np.uint64(vocab)).astype(np.uint32)


def normal(seed: int, stream: int, n: int, sigma: float, offset: int = 0) -> np.ndarray:
    k = np.float32(np.float64(sigma) / 37837.22712838299)
    base = np.uint64(stream_base(seed, stream))
    with np.errstate(over="ignore"):
        h = splitmix64(base + np.uint64(offset) + np.arange(n, dtype=np.uint64))
    m = np.uint64(0xFFFF)
    s = ((h & m).astype(np.int64) + ((h >> np.uint64(16)) & m).astype(np.int64)
         + ((h >> np.uint64(32)) & m).astype(np.int64) + (h >> np.uint64(48)).astype(np.int64))
    return (s - 131070).astype(np.float32) * k


# Model shapes (vocab, dim, hidden, layers, heads, kv_heads, head_dim)
SHAPES = {
    "tiny": (32000, 288, 768, 6, 6, 6, 48),             # Llama-style tiny decoder
    "llama2-7b": (32000, 4096, 11008, 32, 32, 32, 128),  # Llama-2-7B shape
    "tinyllama-1.1b": (32000, 2048, 5632, 22, 32, 4, 64),
    "llama3-70b": (128256, 8192, 28672, 80, 64, 8, 128),
}
ROPE_THETA = {"tiny": 10000.0, "llama2-7b": 10000.0, "tinyllama-1.1b": 10000.0, "llama3-70b": 500000.0}


def config(name: str, max_seq: int, eps: float = 1e-5) -> ModelConfig:
    v, d, f, l, h, kvh, hd = SHAPES[name]
    return ModelConfig(v, d, f, l, h, kvh, hd, max_seq, eps)


def weight_bytes(cfg: ModelConfig) -> int:
    """int8 + fp32-per-32 scale bytes of all projection matrices and the head."""
    D, F, V, L = cfg.dim, cfg.hidden_dim, cfg.vocab_size, cfg.num_layers
    KV = cfg.num_kv_heads * cfg.head_dim
    params = L * (2 * D * D + 2 * KV * D + 3 * F * D) + V * D
    return params + params // 32 * 4


def step_bytes(cfg: ModelConfig, context: int, kv_bytes: int) -> int:
    """Algorithmic HBM bytes of one batch-1 decode step at context c = pos + 1:
    weights + norms 4*D*(2L+1) + one embedding row 4*D + KV read 2*L*c*KVH*hd*b + KV write."""
    D, L = cfg.dim, cfg.num_layers
    KV = cfg.num_kv_heads * cfg.head_dim
    return weight_bytes(cfg) + 4 * D * (2 * L + 1) + 4 * D + 2 * L * KV * kv_bytes * (context + 1)
