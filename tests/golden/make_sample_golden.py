"""Generates tests/golden/sample_cases.npz: tokens drawn by the reference's
own CPU-runtime sampler (inference_runtime.sample_numpy,
inference_runtime.py:144-163) on seeded random logits, with the draw u that
numpy's legacy global generator produced for each case. Run here, where the
reference tree is importable:

    python tests/golden/make_sample_golden.py /path/to/reference
"""
import sys
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent / "sample_cases.npz"
VOCAB = 1024
CASES = 48


def main(reference: str) -> None:
    sys.path.insert(0, reference)
    import inference_runtime

    rng = np.random.default_rng(2024)
    logits = rng.normal(0.0, 3.0, (CASES, VOCAB)).astype(np.float32)
    generated = np.full((CASES, 16), -1, dtype=np.int64)
    params = np.zeros((CASES, 4), dtype=np.float64)  # temperature, top_p, top_k, penalty
    uniform = np.zeros(CASES, dtype=np.float64)
    tokens = np.zeros(CASES, dtype=np.int64)
    for i in range(CASES):
        n = int(rng.integers(0, 17))
        generated[i, :n] = rng.integers(0, VOCAB, n)
        temperature = float(rng.choice([0.0, 0.4, 0.7, 1.3]))
        top_p = float(rng.choice([0.5, 0.9, 1.0]))
        top_k = int(rng.choice([1, 8, 40, 50, 64]))
        penalty = float(rng.choice([1.0, 1.08, 1.15]))
        params[i] = (temperature, top_p, top_k, penalty)
        gen = [int(t) for t in generated[i, :n]]
        np.random.seed(1000 + i)
        tokens[i] = inference_runtime.sample_numpy(np, logits[i], gen, temperature, top_p, top_k, penalty)
        np.random.seed(1000 + i)
        uniform[i] = np.random.random_sample() if temperature > 0.01 else 0.0
    np.savez_compressed(OUT, logits=logits, generated=generated, params=params, uniform=uniform, tokens=tokens)
    print("wrote", OUT)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_sample_golden.py /path/to/reference")
    main(sys.argv[1])
