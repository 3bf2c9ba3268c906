"""Seeded synthetic inputs for the five workload configurations.

The reference publishes no dataset for this path and no model weights are
available, so every tensor is synthetic, drawn with numpy's PCG64 generator
from the seeds below (the seeds the workload description leaves open are
``1000 * config + tensor_index``). "N(mu, s)" is read as mean / standard
deviation. fp16 fields are rounded to nearest from float32.

Quantised tables use the GGUF block layouts of the reference
(src/ds3_reference.c:65-70 Q4_K 144 B, :119-124 Q6_K 210 B): raw random block
fields (fp16 d/dmin ~U(0, 0.02), uniform scale bytes, uniform quant bytes),
which covers every bit pattern the decoders accept.
"""

from __future__ import annotations

import numpy as np

N_EMBD = 2048
N_HEAD = 32
N_HEAD_KV = 4
HEAD_DIM = 128
N_EXPERT = 128
N_EXPERT_USED = 8
N_FF_EXP = 768
N_VOCAB = 151936
ROPE_THETA = 1e6
NORM_EPS = 1e-6

Q4K_BLOCK = 144
Q6K_BLOCK = 210


def rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def normal(seed: int, shape, mean=0.0, std=1.0) -> np.ndarray:
    return (rng(seed).standard_normal(shape, dtype=np.float32) * np.float32(std) + np.float32(mean)).astype(
        np.float32)


def q4k_table(n_rows: int, n_cols: int, seed: int) -> np.ndarray:
    """[n_rows, n_cols/256 * 144] uint8 random Q4_K rows."""
    nb = n_cols // 256
    g = rng(seed)
    t = g.integers(0, 256, size=(n_rows, nb, Q4K_BLOCK), dtype=np.uint8)
    dd = g.uniform(0.0, 0.02, size=(n_rows, nb, 2)).astype(np.float16)
    t[:, :, 0:4] = dd.view(np.uint8).reshape(n_rows, nb, 4)
    return t.reshape(n_rows, nb * Q4K_BLOCK)


def q6k_table(n_rows: int, n_cols: int, seed: int) -> np.ndarray:
    """[n_rows, n_cols/256 * 210] uint8 random Q6_K rows."""
    nb = n_cols // 256
    g = rng(seed)
    t = g.integers(0, 256, size=(n_rows, nb, Q6K_BLOCK), dtype=np.uint8)  # ql, qh, int8 scales
    d = g.uniform(0.0, 0.02, size=(n_rows, nb, 1)).astype(np.float16)
    t[:, :, 208:210] = d.view(np.uint8).reshape(n_rows, nb, 2)
    return t.reshape(n_rows, nb * Q6K_BLOCK)


def token_ids(n: int, seed: int, vocab: int = N_VOCAB) -> np.ndarray:
    return rng(seed).integers(0, vocab, size=n, dtype=np.int64).astype(np.int32)


def gamma(n: int, seed: int) -> np.ndarray:
    return normal(seed, (n,), 1.0, 0.1)
