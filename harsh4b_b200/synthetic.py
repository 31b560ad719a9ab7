"""Seeded synthetic checkpoints for the Qwen3-4B LATTICE architecture.

The real ``model.lat.pt`` is not distributable, so every measurement and
parity check runs on random weights drawn the same way each time:

* body projections: int4 codes ``rint(clip(N(0, 2.5), -7, 7))``, packed two
  per byte along K, with fp32 row scales ``lognormal(mean=-6, sigma=0.3)``;
* the tied embedding / LM head: the same recipe, shape ``[vocab, hidden]``;
* norm vectors: ``1 + N(0, 0.02)`` in fp32.

Each tensor draws from its own ``numpy.random.default_rng([seed, index])``,
so the bytes do not depend on thread scheduling.
"""
from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from .cache import Checkpoint, norm_names, projection_names

# Qwen3-4B hyper-parameters (the reference's configs/qwen3-4b.json).
QWEN3_4B = {
    "num_hidden_layers": 36, "hidden_size": 2560, "intermediate_size": 9728,
    "num_attention_heads": 32, "num_key_value_heads": 8, "head_dim": 128,
    "vocab_size": 151936, "max_position_embeddings": 40960, "rope_theta": 1000000,
    "rms_norm_eps": 1e-06, "tie_word_embeddings": True,
}


def qwen3_4b_config(**overrides) -> dict:
    return dict(QWEN3_4B, **overrides)


def tiny_config(**overrides) -> dict:
    """A 2-layer model with the real head_dim and GQA grouping, for parity tests.

    Like Qwen3-4B it keeps intermediate_size >= q heads * head_dim: the
    reference sizes its int8 activation scratch by intermediate_size
    (cpu_lightspark.py:294) and quantises the attention output into it."""
    config = dict(QWEN3_4B, num_hidden_layers=2, hidden_size=256, intermediate_size=1024,
                  num_attention_heads=8, num_key_value_heads=2, vocab_size=2048,
                  max_position_embeddings=512)
    config.update(overrides)
    return config


_CHUNK = 1 << 22


def int4_matrix(rng: np.random.Generator, rows: int, cols: int) -> np.ndarray:
    """Packed uint8[rows, cols/2] of codes rint(clip(N(0, 2.5), -7, 7))."""
    packed = np.empty((rows, cols // 2), dtype=np.uint8)
    step = max(1, _CHUNK // cols)
    for start in range(0, rows, step):
        stop = min(rows, start + step)
        block = rng.standard_normal((stop - start, cols), dtype=np.float32)
        block *= np.float32(2.5)
        np.clip(block, -7.0, 7.0, out=block)
        np.rint(block, out=block)
        codes = block.astype(np.int8).view(np.uint8)
        packed[start:stop] = (codes[:, 0::2] & np.uint8(0x0F)) | (codes[:, 1::2] << np.uint8(4))
    return packed


def row_scales(rng: np.random.Generator, rows: int) -> np.ndarray:
    return rng.lognormal(mean=-6.0, sigma=0.3, size=rows).astype(np.float32)


def synthetic_checkpoint(config: dict | None = None, seed: int = 0, threads: int | None = None) -> Checkpoint:
    config = dict(config or QWEN3_4B)
    checkpoint = Checkpoint(config=config)
    shapes = checkpoint.expected_shapes()
    names = projection_names(config)
    vocab, hidden = int(config["vocab_size"]), int(config["hidden_size"])

    def make_projection(index: int):
        rows, cols = shapes[names[index]]
        rng = np.random.default_rng([seed, index])
        return names[index], (int4_matrix(rng, rows, cols), row_scales(rng, rows))

    def make_embedding_part(part: int, parts: int):
        start, stop = part * vocab // parts, (part + 1) * vocab // parts
        rng = np.random.default_rng([seed, len(names), part])
        return start, stop, int4_matrix(rng, stop - start, hidden), row_scales(rng, stop - start)

    workers = threads or min(32, os.cpu_count() or 1)
    parts = 64 if vocab >= 65536 else 1
    checkpoint.embedding = np.empty((vocab, hidden // 2), dtype=np.uint8)
    checkpoint.embedding_scales = np.empty(vocab, dtype=np.float32)
    with ThreadPoolExecutor(max_workers=workers) as pool:
        embedding_jobs = [pool.submit(make_embedding_part, p, parts) for p in range(parts)]
        for name, value in pool.map(make_projection, range(len(names))):
            checkpoint.projections[name] = value
        for job in embedding_jobs:
            start, stop, weights, scales = job.result()
            checkpoint.embedding[start:stop] = weights
            checkpoint.embedding_scales[start:stop] = scales
    rng = np.random.default_rng([seed, len(names) + 1])
    for name in norm_names(config):
        size = int(config["head_dim"]) if ("q_norm" in name or "k_norm" in name) else hidden
        checkpoint.norms[name] = (1.0 + 0.02 * rng.standard_normal(size)).astype(np.float32)
    return checkpoint


def synthetic_prompt(config: dict | None = None, length: int = 128, seed: int = 0) -> list[int]:
    """Uniform random token ids in [0, vocab)."""
    vocab = int((config or QWEN3_4B)["vocab_size"])
    rng = np.random.default_rng([seed, 0x70726F6D])
    return [int(t) for t in rng.integers(0, vocab, size=length)]


def outlier_activation(size: int, seed: int = 0, fraction: float = 0.005, factor: float = 20.0) -> np.ndarray:
    """fp32 N(0,1) activation with a seeded ``fraction`` of channels scaled by
    ``factor``; the input distribution of the body-GEMV microbenchmark."""
    rng = np.random.default_rng([seed, size, 0x6F7574])
    x = rng.standard_normal(size, dtype=np.float32)
    count = max(1, int(round(size * fraction)))
    x[rng.choice(size, size=count, replace=False)] *= np.float32(factor)
    return x
