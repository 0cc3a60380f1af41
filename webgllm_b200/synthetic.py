"""Seeded synthetic inputs of the BASELINE configs (no datasets, no files).

Config 0/1 weights: per 32-weight block, scale d = fp16(|N(0,1)| * 0.02 / 8)
and codes uniform on 0..15, written as llama.cpp Q4_0 blocks (18 bytes: the
fp16 scale, then byte j holding code j low and code j + 16 high). Activations
N(0,1). numpy default_rng throughout, so every run and every host draws the
same numbers.
"""
from __future__ import annotations

import numpy as np


def q4_0_blocks(N: int, K: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    nb = N * (K // 32)
    d = (np.abs(rng.standard_normal(nb)) * 0.02 / 8).astype(np.float16)
    q = rng.integers(0, 16, size=(nb, 32), dtype=np.uint8)
    out = np.zeros((nb, 18), dtype=np.uint8)
    out[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    out[:, 2:] = q[:, :16] | (q[:, 16:] << 4)
    return out.reshape(-1)


def activations(M: int, K: int, seed: int, dtype=np.float32) -> np.ndarray:
    rng = np.random.default_rng(seed + 1_000_003)
    return rng.standard_normal((M, K)).astype(dtype)
