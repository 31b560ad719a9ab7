#!/usr/bin/env python3
"""Generate the LATTICE -> int4 conversion fixtures from the reference's own
functions: ``MLX.lattice_model.expand_t1`` (MLX/lattice_model.py:160-185),
``cpu_lightspark._convert_projection`` (cpu_lightspark.py:149-201) and
``cpu_lightspark._convert_embedding`` (:204-229), run unmodified on seeded
synthetic projections.

Usage (needs a checkout of the reference project; not run by the tests):

    python tests/golden/make_lattice_golden.py <path-to-reference-checkout>

Writes ``tests/golden/lattice_cases.npz``.
"""
from __future__ import annotations

import sys
import tempfile
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))

from oracle.lattice import orthogonal, synthetic_projection  # noqa: E402

# (rows, width, blocksize, dim_l, dim_r, fp16 scale planes, o2 modes)
CASES = [(24, 96, 32, 8, 12, True, (0, 1)), (16, 160, 64, 10, 16, False, (0, 1)),
         (12, 256, 128, 16, 16, True, (1,)), (7, 72, 16, 6, 12, True, (0, 1))]
EMBEDDINGS = [(40, 64, np.float32), (33, 128, np.float16)]


class Tensor:
    """The ``.numpy()`` face the reference's checkpoint reader gives tensors."""

    def __init__(self, value):
        self.value = value

    def numpy(self):
        return self.value


def main(reference: str) -> None:
    sys.path.insert(0, str(Path(reference).resolve()))
    import cpu_lightspark
    from MLX.lattice_model import expand_t1

    rng = np.random.default_rng(2024)
    out = {}
    with tempfile.TemporaryDirectory() as tmp:
        for i, (rows, width, blocksize, dl, dr, half, o2) in enumerate(CASES):
            packed = synthetic_projection(rng, rows, width, blocksize, o2=o2, half=half)
            left, right = orthogonal(rng, dl), orthogonal(rng, dr)
            wrapped = {k: (Tensor(v) if isinstance(v, np.ndarray) else v) for k, v in packed.items()}
            t1 = expand_t1(wrapped)
            wpath, spath = Path(tmp) / f"w{i}.npy", Path(tmp) / f"s{i}.npy"
            cpu_lightspark._convert_projection(wrapped, left, right, wpath, spath)
            for key, value in packed.items():
                out[f"p{i}_{key}"] = np.asarray(value)
            out[f"p{i}_left"], out[f"p{i}_right"] = left, right
            out[f"p{i}_t1_dense"] = t1
            out[f"p{i}_packed"] = np.load(wpath)
            out[f"p{i}_scales"] = np.load(spath)
        for i, (rows, width, dtype) in enumerate(EMBEDDINGS):
            source = (rng.standard_normal((rows, width)) * 0.05).astype(dtype)
            source[0, 3] = 0.0
            source[1] = 0.0  # an all-zero row takes the 1e-8 floor
            wpath, spath = Path(tmp) / f"e{i}.npy", Path(tmp) / f"es{i}.npy"
            cpu_lightspark._convert_embedding(source, wpath, spath)
            out[f"e{i}_source"] = source
            out[f"e{i}_packed"] = np.load(wpath)
            out[f"e{i}_scales"] = np.load(spath)
    out["n_projections"] = np.array(len(CASES))
    out["n_embeddings"] = np.array(len(EMBEDDINGS))
    target = Path(__file__).resolve().parent / "lattice_cases.npz"
    np.savez_compressed(target, **out)
    print("wrote", target)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_lattice_golden.py /path/to/reference")
    main(sys.argv[1])
