"""Phase timeline of the persistent decode kernel (a profiling tool).

Builds an instrumented copy of the library (``-DH4B_PHASE_TRACE``: every CTA
stamps ``%globaltimer`` at the start of each GEMV segment of layer 2, after
its prologue, after its ring tiles and after its epilogue, at the attention
steps, and at the same points of the LM-head segment), decodes config 0 on
it and prints, per segment, the median / max CTA durations and the rate at
which the GEMV tiles consume weight bytes:

* ``tile-phase GB/s``: the segment's weight + scale bytes over the longest
  CTA's tile phase (the ring is filled ahead by the producer warp, so this
  is the GEMV's compute-side rate, not an HBM rate);
* ``segment GB/s``: the same bytes over the time from the first CTA's
  segment start to the last CTA's tiles done (handoff, prologue and tiles).

The instrumented build is slower than the normal one (every stamp is a
global store); ratios between phases are what it is for.

    python -m harsh4b_b200.phase_trace [--layers 36] [--json out.json]
"""
from __future__ import annotations

import argparse
import ctypes
import json
import tempfile
from pathlib import Path

import numpy as np

SEGMENTS = {"qkv": 0, "o": 4, "gate_up": 8, "down": 12}
ATTENTION = {16: "attention entered", 17: "q/k/v polled", 18: "first sub-tile staged", 19: "attention math done",
             20: "splits merged", 21: "attended heads published", 22: "split partial published"}


def segment_bytes(model) -> dict:
    """Weight + row-scale bytes of one layer's segments and of the LM head."""
    H, I, Q, KV = model.hidden, model.intermediate, model.q_size, model.kv_size
    rows = {"qkv": (Q + 2 * KV, H), "o": (H, Q), "gate_up": (2 * I, H), "down": (H, I), "lm_head": (model.vocab, H)}
    return {k: r * (w // 2) + 4 * r for k, (r, w) in rows.items()}


def run(layers: int = 36, library: Path | None = None, tokens: int = 30) -> dict:
    from . import _lib, build

    if library is None:
        library = Path(tempfile.mkdtemp()) / "libharsh4b_b200_trace.so"
        build.build(output=library, defines=("H4B_PHASE_TRACE",))
    _lib.LIBRARY = Path(library)
    import torch

    from .model import CudaQwen
    from .synthetic import qwen3_4b_config, synthetic_checkpoint, synthetic_prompt

    config = qwen3_4b_config(num_hidden_layers=layers)
    model = CudaQwen.from_checkpoint(synthetic_checkpoint(config, seed=0), kv_dtype="float16", mode="persistent")
    state = model.new_state(128 + tokens + 2)
    for token in synthetic_prompt(config, 128, seed=0):
        model.forward_token(token, state)
    model.generate_greedy(state.next_token_host(), state, tokens)
    torch.cuda.synchronize()
    lib = _lib.load_library(str(library))
    lib.h4b_phase_trace_ctas.argtypes = [ctypes.c_void_p]
    stamps = np.zeros((1024, 32), dtype=np.uint64)
    _lib.check(lib.h4b_phase_trace_ctas(stamps.ctypes.data), "h4b_phase_trace_ctas")
    n = model.sm_count
    t = stamps[:n].astype(np.int64)
    t0 = t[:, 0].min()
    us = (t - t0) / 1000.0
    sizes = segment_bytes(model)
    out = {"layers": layers, "context": 128 + tokens, "ctas": n, "segments": {}, "attention": {}}

    def describe(name, base):
        start, pro, tiles, epi = (us[:, base + k] for k in range(4))
        tile_phase = tiles - pro
        seg = {"prologue_us_med": float(np.median(pro - start)), "tiles_us_med": float(np.median(tile_phase)),
               "tiles_us_max": float(tile_phase.max()), "epilogue_us_med": float(np.median(epi - tiles)),
               "span_us": float(tiles.max() - start.min()), "bytes": int(sizes[name])}
        seg["tile_phase_gbs"] = sizes[name] / (seg["tiles_us_max"] * 1e3)
        seg["segment_gbs"] = sizes[name] / (seg["span_us"] * 1e3)
        out["segments"][name] = {k: round(v, 3) if isinstance(v, float) else v for k, v in seg.items()}

    for name, base in SEGMENTS.items():
        describe(name, base)
    describe("lm_head", 23)
    # the layer's period: one segment start to the same segment a layer later
    # is not stamped; use the span from qkv start to down epilogue done
    out["layer_us"] = round(float(np.median(us[:, 15] - us[:, 0])), 3)
    valid = [c for c in range(n) if t[c, 16] > 0]
    for ev, label in ATTENTION.items():
        vals = [us[c, ev] - us[c, 0] for c in valid if t[c, ev] >= t0]
        if vals:
            out["attention"][label] = round(float(np.median(vals)), 3)
    out["status"] = model.status()
    state.close()
    return out


def main(argv=None) -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--layers", type=int, default=36)
    parser.add_argument("--library", type=Path, default=None, help="an already built trace library")
    parser.add_argument("--json", type=Path, default=None)
    args = parser.parse_args(argv)
    result = run(args.layers, args.library)
    print(f"layer 2 of {result['layers']}, context {result['context']}, {result['ctas']} CTAs; "
          f"qkv start -> down epilogue (median CTA) {result['layer_us']} us")
    print(f"{'segment':8s} {'prologue':>9s} {'tiles med':>10s} {'tiles max':>10s} {'epilogue':>9s} "
          f"{'span':>7s} {'MB':>7s} {'tile GB/s':>10s} {'seg GB/s':>9s}")
    for name, s in result["segments"].items():
        print(f"{name:8s} {s['prologue_us_med']:9.2f} {s['tiles_us_med']:10.2f} {s['tiles_us_max']:10.2f} "
              f"{s['epilogue_us_med']:9.2f} {s['span_us']:7.2f} {s['bytes'] / 1e6:7.2f} "
              f"{s['tile_phase_gbs']:10.0f} {s['segment_gbs']:9.0f}")
    print("attention (median over attention CTAs, us after the qkv segment start):", result["attention"])
    if args.json:
        args.json.write_text(json.dumps(result, indent=2))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
