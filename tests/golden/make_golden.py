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

Writes ``tests/golden/tiny_decode.npz`` (a 2-layer toy shape, every logit
of every step) and, with ``--qwen-shape``, ``tests/golden/qwen_shape_decode.npz``:
two layers of Qwen3-4B's exact shapes (hidden 2560, 32 / 8 heads of 128,
SwiGLU 9728, the full 151936-row tied vocabulary), a 16-token prompt and 64
greedy steps. That fixture keeps, per step after the prompt, the greedy
token, the top-1 / top-2 margin, the 32 largest logits with their ids and the
logits at 1024 fixed random ids (the full rows would be 39 MB), and how far
the reference's own two attention paths (native kernel vs numpy) move the
logits on those steps (``reference_path_drift``).
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
from harsh4b_b200.synthetic import qwen3_4b_config, synthetic_checkpoint, synthetic_prompt, tiny_config  # noqa: E402

SEED = 7
PROMPT = 12
DECODE = 20
QWEN_SEED = 11
QWEN_PROMPT = 16
QWEN_DECODE = 64
QWEN_SAMPLE = 1024
QWEN_TOP = 32


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
    parser.add_argument("--out", type=Path, default=None)
    parser.add_argument("--qwen-shape", action="store_true", help="two layers of Qwen3-4B shapes, full vocabulary")
    args = parser.parse_args()
    here = Path(__file__).resolve().parent
    if args.out is None:
        args.out = here / ("qwen_shape_decode.npz" if args.qwen_shape else "tiny_decode.npz")
    sys.path.insert(0, str(args.reference.resolve()))
    import cpu_lightspark as reference

    seed = QWEN_SEED if args.qwen_shape else SEED
    config = qwen3_4b_config(num_hidden_layers=2) if args.qwen_shape else tiny_config()
    checkpoint = synthetic_checkpoint(config, seed=seed)
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

    prompt_len, decode = (QWEN_PROMPT, QWEN_DECODE) if args.qwen_shape else (PROMPT, DECODE)
    prompt = synthetic_prompt(config, prompt_len, seed=seed)
    state = model.new_state(prompt_len + decode)
    logits, tokens = [], []
    for token in prompt:
        logits.append(model.forward_token(token, state).copy())
    for _ in range(decode):
        token = int(logits[-1].argmax())  # the --argmax policy, cpu_lightspark.py:704-705
        tokens.append(token)
        logits.append(model.forward_token(token, state).copy())
    if args.qwen_shape:
        rows = np.stack(logits[prompt_len - 1:])  # the row after the prompt, then one per greedy step
        # The reference's other attention path -- its native kernel
        # (litespark_gqa_decode, as restated by the oracle's C code) instead of
        # numpy -- on the same tokens: how far its own two paths disagree.
        import ctypes

        native = oracle.library().oracle_gqa_decode
        native.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int] * 5
        native.restype = None
        model.attention_kernel = native
        state = model.new_state(prompt_len + decode)
        other = []
        for token in prompt:
            last = model.forward_token(token, state).copy()
        other.append(last)
        for token in tokens:
            other.append(model.forward_token(token, state).copy())
        path_drift = float(np.abs(np.stack(other) - rows).max())
        sample_ids = np.sort(np.random.default_rng([seed, 0x5A4D]).choice(config["vocab_size"], QWEN_SAMPLE,
                                                                         replace=False))
        top_ids = np.argsort(-rows, axis=1, kind="stable")[:, :QWEN_TOP]
        part = np.partition(rows, -2, axis=1)
        np.savez_compressed(
            args.out, config=json.dumps(config), seed=seed, prompt=np.asarray(prompt, dtype=np.int64),
            tokens=np.asarray(tokens, dtype=np.int64), sample_ids=sample_ids.astype(np.int64),
            sample_logits=rows[:, sample_ids].astype(np.float32), top_ids=top_ids.astype(np.int64),
            top_logits=np.take_along_axis(rows, top_ids, axis=1).astype(np.float32),
            margin=(part[:, -1] - part[:, -2]).astype(np.float32), digest=checkpoint_digest(checkpoint),
            reference_path_drift=np.float32(path_drift))
        print(f"wrote {args.out}: {len(prompt)} prompt + {len(tokens)} greedy steps; "
              f"min top-2 margin {float((part[:, -1] - part[:, -2]).min()):.4g}; the reference's native vs "
              f"numpy attention paths differ by {path_drift:.4g} max-abs")
        return 0
    np.savez_compressed(
        args.out, config=json.dumps(config), seed=SEED, prompt=np.asarray(prompt, dtype=np.int64),
        tokens=np.asarray(tokens, dtype=np.int64), logits=np.stack(logits).astype(np.float32),
        digest=checkpoint_digest(checkpoint))
    print(f"wrote {args.out}: {len(prompt)} prompt + {len(tokens)} greedy steps")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
