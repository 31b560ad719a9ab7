"""The reference's benchmark suite on the B200 backend.

The reference measures its runtimes with ``benchmarks/bench_latency.py``
(a TTFT / TPOT grid over prompt x decode lengths) and
``benchmarks/bench_energy.py`` (one generation with board power sampled,
Joules per token); both take any runtime from ``create_runtime`` and already
handle ``device == "cuda"`` (bench_energy.py:269-273, NVML sampler
:181-197). With "cuda" routed to :class:`harsh4b_b200.runtime.CudaBackend`
they run unchanged. This module restates their measurements for machines
without the reference checkout:

* :func:`timed_generate` -- one generation: TTFT = prefill + first sample,
  then per-token latencies (decode + device sync + sample) until
  ``max_new_tokens`` or an end-of-turn id (bench_energy.py:276-305);
* :func:`latency_grid` -- the bench_latency cells: TTFT median/min/max,
  prefill tok/s, TPOT median / p95, decode and end-to-end tok/s per
  (prompt, decode) length (bench_latency.py:93-142);
* :func:`energy_per_token` -- the NVML board-power integral over one
  generation (reading power only; nothing on the GPU is changed).

``python -m harsh4b_b200.benchsuite --model <LATTICE file or cache dir>``
prints the grid and writes JSON / CSV like bench_latency.py.
"""
from __future__ import annotations

import argparse
import csv
import json
import statistics
import threading
import time
from pathlib import Path


def percentile(values: list[float], pct: float) -> float:
    """Linear-interpolated percentile, as the reference's benchmarks compute it."""
    if not values:
        return 0.0
    ordered = sorted(values)
    rank = (len(ordered) - 1) * pct / 100.0
    low, high = int(rank), min(int(rank) + 1, len(ordered) - 1)
    return ordered[low] * (1 - (rank - low)) + ordered[high] * (rank - low)


def _sync(backend) -> None:
    backend.torch.cuda.synchronize()


def timed_generate(backend, prompt_ids: list[int], max_new_tokens: int, temperature: float,
                   stop_ids=None) -> dict:
    """One measured generation; returns TTFT, the inter-token latencies, the
    generated ids and the prefill / decode wall times."""
    stop_ids = stop_ids if stop_ids is not None else getattr(backend.tokenizer, "stop_ids", set())
    itls, generated = [], []
    t_start = time.perf_counter()
    logits, session = backend.prefill(prompt_ids, max_new_tokens)
    _sync(backend)
    token = backend.sample(logits, generated, temperature)
    ttft = time.perf_counter() - t_start
    if token in stop_ids:
        return dict(ttft=ttft, itls=[], generated=generated, prefill_s=ttft, decode_s=0.0)
    generated.append(token)
    t_dec0 = time.perf_counter()
    while len(generated) < max_new_tokens:
        t0 = time.perf_counter()
        logits = backend.decode(token, session)
        _sync(backend)
        token = backend.sample(logits, generated, temperature)
        itls.append(time.perf_counter() - t0)
        if token in stop_ids:
            break
        generated.append(token)
    return dict(ttft=ttft, itls=itls, generated=generated, prefill_s=ttft, decode_s=time.perf_counter() - t_dec0)


def latency_grid(backend, prompt_lens, decode_lens, repeats: int = 3, warmup: int = 1, temperature: float = 0.0,
                 prompt_for=None, stop_ids=None, out=print) -> list[dict]:
    """bench_latency's grid: one cell per (prompt length, decode length)."""
    med = statistics.median
    cells = []
    for prompt_len in prompt_lens:
        prompt_ids = prompt_for(prompt_len) if prompt_for else [(7 * i + 13) % 1000 for i in range(prompt_len)]
        for decode_len in decode_lens:
            for _ in range(warmup):
                timed_generate(backend, prompt_ids, decode_len, temperature, stop_ids)
            ttfts, prefills, tpot_med, tpot_p95, dec_tps, e2e_tps = [], [], [], [], [], []
            n_gen = 0
            for _ in range(repeats):
                t0 = time.perf_counter()
                result = timed_generate(backend, prompt_ids, decode_len, temperature, stop_ids)
                wall_s = time.perf_counter() - t0
                n_gen, itls = len(result["generated"]), result["itls"]
                ttfts.append(result["ttft"])
                prefills.append(len(prompt_ids) / result["prefill_s"] if result["prefill_s"] else 0.0)
                tpot_med.append(med(itls) * 1000 if itls else 0.0)
                tpot_p95.append(percentile(itls, 95) * 1000 if itls else 0.0)
                dec_tps.append(len(itls) / result["decode_s"] if result["decode_s"] else 0.0)
                e2e_tps.append(n_gen / wall_s if wall_s else 0.0)
            cell = dict(prompt_tokens=prompt_len, decode_tokens=decode_len, generated_tokens=n_gen,
                        ttft_med_s=round(med(ttfts), 4), ttft_min_s=round(min(ttfts), 4),
                        ttft_max_s=round(max(ttfts), 4), prefill_med_tok_s=round(med(prefills), 2),
                        tpot_med_ms=round(med(tpot_med), 3), tpot_p95_ms=round(med(tpot_p95), 3),
                        decode_med_tok_s=round(med(dec_tps), 2), e2e_med_tok_s=round(med(e2e_tps), 2))
            cells.append(cell)
            out(f"[p={prompt_len:5d} d={decode_len:4d}] TTFT med {cell['ttft_med_s']:.4f}s prefill "
                f"{cell['prefill_med_tok_s']:.0f}tok/s | TPOT med/p95 {cell['tpot_med_ms']:.2f}/"
                f"{cell['tpot_p95_ms']:.2f}ms decode {cell['decode_med_tok_s']:.1f}tok/s")
    return cells


class NvmlPower:
    """Board power of one GPU sampled by a thread through NVML (read only)."""

    def __init__(self, index: int = 0, interval_s: float = 0.01):
        import pynvml

        pynvml.nvmlInit()
        self._nvml, self.interval = pynvml, interval_s
        self._handle = pynvml.nvmlDeviceGetHandleByIndex(index)
        self._samples: list[tuple[float, float]] = []
        self._stop = threading.Event()
        self._thread = None

    def _run(self) -> None:
        while not self._stop.is_set():
            try:
                watts = self._nvml.nvmlDeviceGetPowerUsage(self._handle) / 1000.0
                self._samples.append((time.perf_counter(), watts))
            except Exception:
                pass
            time.sleep(self.interval)

    def __enter__(self):
        self._samples.clear()
        self._stop.clear()
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        self._thread.join()

    def joules(self) -> float:
        """Trapezoidal integral of the sampled power."""
        s = self._samples
        return sum(0.5 * (s[i][1] + s[i - 1][1]) * (s[i][0] - s[i - 1][0]) for i in range(1, len(s)))

    def mean_watts(self) -> float:
        return statistics.fmean(w for _, w in self._samples) if self._samples else 0.0


def energy_per_token(backend, prompt_ids, max_new_tokens: int, temperature: float = 0.0, index: int = 0,
                     stop_ids=None) -> dict:
    """One generation with the GPU's board power sampled: Joules per
    generated token and the mean power (bench_energy's measurement)."""
    with NvmlPower(index) as power:
        result = timed_generate(backend, prompt_ids, max_new_tokens, temperature, stop_ids)
    n = max(1, len(result["generated"]))
    joules = power.joules()
    return dict(tokens=len(result["generated"]), joules=round(joules, 3), joules_per_token=round(joules / n, 4),
                mean_watts=round(power.mean_watts(), 1), ttft_s=round(result["ttft"], 4),
                decode_tok_s=round(len(result["itls"]) / result["decode_s"], 2) if result["decode_s"] else 0.0)


def main(argv=None) -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--model", type=Path, required=True, help="LATTICE checkpoint file or packed cache directory")
    parser.add_argument("--prompt-lens", default="32,128,512")
    parser.add_argument("--decode-lens", default="32")
    parser.add_argument("--repeats", type=int, default=3)
    parser.add_argument("--warmup", type=int, default=1)
    parser.add_argument("--temperature", type=float, default=0.0)
    parser.add_argument("--energy", action="store_true", help="also one NVML-sampled generation (J/token)")
    parser.add_argument("--json-out", type=Path)
    parser.add_argument("--csv-out", type=Path)
    args = parser.parse_args(argv)
    from .runtime import CudaBackend

    backend = CudaBackend(args.model)
    print(f"runtime: {backend.device} ({backend.description})\nhardware: {backend.hardware}", flush=True)
    cells = latency_grid(backend, [int(v) for v in args.prompt_lens.split(",")],
                         [int(v) for v in args.decode_lens.split(",")], args.repeats, args.warmup, args.temperature,
                         stop_ids=set())
    summary = dict(runtime=backend.device, hardware=backend.hardware, repeats=args.repeats, cells=cells)
    if args.energy:
        summary["energy"] = energy_per_token(backend, [(7 * i + 13) % 1000 for i in range(128)], 64,
                                             args.temperature, stop_ids=set())
        print("energy:", summary["energy"], flush=True)
    if args.json_out:
        args.json_out.parent.mkdir(parents=True, exist_ok=True)
        args.json_out.write_text(json.dumps(summary, indent=2))
    if args.csv_out:
        args.csv_out.parent.mkdir(parents=True, exist_ok=True)
        with open(args.csv_out, "w", newline="") as fh:
            writer = csv.DictWriter(fh, fieldnames=list(cells[0].keys()))
            writer.writeheader()
            writer.writerows(cells)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
