#!/usr/bin/env python3
"""Generate the golden decode fixtures from the reference's own code.

Runs the reference's ``cpu_lightspark.LiteSparkQwen.forward_token``
(cpu_lightspark.py:424-468) unmodified, built directly from a seeded
synthetic checkpoint (bypassing ``load_checkpoint``), and records its logits
and greedy tokens. The reference needs three stand-ins on an x86 host:

* ``int4_kernel`` -> the C oracle's ``oracle_int4_i8_gemv``, which has the
  ctypes signature of ``litespark_int4_i8_gemv`` (cpu_lightspark.py:71-79);
* ``kernel`` -> ``oracle.OracleKernel``, restating the absent third-party
  ``litespark_inference`` kernel object;
* ``attention_kernel = None`` -> the reference's own numpy einsum attention
  (cpu_lightspark.py:408-422).

Usage (needs a checkout of the reference project; not run by the tests):

    python tests/golden/make_golden.py --reference <path-to-reference-checkout>

Writes ``tests/golden/tiny_decode.npz``.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import sys
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))

import oracle  # noqa: E402
from harsh4b_b200.synthetic import synthetic_checkpoint, synthetic_prompt, tiny_config  # noqa: E402

SEED = 7
PROMPT = 12
DECODE = 20


def checkpoint_digest(checkpoint) -> str:
    digest = hashlib.sha256()
    for name in sorted(checkpoint.projections):
        for array in checkpoint.projections[name]:
            digest.update(np.ascontiguousarray(array).tobytes())
    digest.update(checkpoint.embedding.tobytes())
    digest.update(checkpoint.embedding_scales.tobytes())
    for name in sorted(checkpoint.norms):
        digest.update(checkpoint.norms[name].tobytes())
    return digest.hexdigest()


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", type=Path, required=True, help="reference project root")
    parser.add_argument("--out", type=Path, default=Path(__file__).resolve().parent / "tiny_decode.npz")
    args = parser.parse_args()
    sys.path.insert(0, str(args.reference.resolve()))
    import cpu_lightspark as reference

    config = tiny_config()
    checkpoint = synthetic_checkpoint(config, seed=SEED)
    layers = []
    for index in range(config["num_hidden_layers"]):
        qkv, o, gate_up, down, input_norm, post_norm, q_norm, k_norm = checkpoint.layer(index)
        layers.append(reference.QwenLayer(
            qkv=reference.LiteSparkProjection(*qkv), o=reference.LiteSparkProjection(*o),
            gate_up=reference.LiteSparkProjection(*gate_up), down=reference.LiteSparkProjection(*down),
            input_norm=input_norm, post_norm=post_norm, q_norm=q_norm, k_norm=k_norm))
    model = reference.LiteSparkQwen(config, layers, checkpoint.embedding, checkpoint.embedding_scales,
                                    checkpoint.norms["model.norm.weight"], oracle.OracleKernel())
    model.int4_kernel = oracle.int4_gemv_function()
    model.attention_kernel = None

    prompt = synthetic_prompt(config, PROMPT, seed=SEED)
    state = model.new_state(PROMPT + DECODE)
    logits, tokens = [], []
    for token in prompt:
        logits.append(model.forward_token(token, state).copy())
    for _ in range(DECODE):
        token = int(logits[-1].argmax())  # the --argmax policy, cpu_lightspark.py:704-705
        tokens.append(token)
        logits.append(model.forward_token(token, state).copy())
    np.savez_compressed(
        args.out, config=json.dumps(config), seed=SEED, prompt=np.asarray(prompt, dtype=np.int64),
        tokens=np.asarray(tokens, dtype=np.int64), logits=np.stack(logits).astype(np.float32),
        digest=checkpoint_digest(checkpoint))
    print(f"wrote {args.out}: {len(prompt)} prompt + {len(tokens)} greedy steps")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
