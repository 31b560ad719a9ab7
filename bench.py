#!/usr/bin/env python3
"""Batch-1 Qwen3-4B int4 decode benchmark on B200.

A step is one decode token at batch 1 through the whole model (36 layers +
LM head + greedy argmax), on the seeded synthetic checkpoint, after a
128-token prompt. ``value`` times K steps with every input resident in HBM
(one CUDA graph replay per token, the next token fed back on the device);
``e2e`` times the same K steps through the public API with a host round trip
per token (pinned H2D of the token id, D2H of the greedy result).

Under torchrun each rank decodes its own sequence on its own GPU
(independent replicas, no collective on the data path); ``value`` is the
sum over ranks of tokens / max-over-ranks time.

``--impl reference`` times the reference's CPU path instead: the oracle's
restatement of cpu_lightspark.LiteSparkQwen.forward_token with the C GEMV
(OpenMP over all host cores), since the reference's native kernel is ARM
NEON only and its litespark-inference dependency is not installable.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "batch-1 decode tok/s Qwen3-4B int4; body-GEMV HBM GB/s vs ~8 TB/s"
PROMPT = 128
# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) per algorithmic
# byte, from ncu captures: the persistent decode kernel on a 4-layer
# Qwen3-4B-shaped model (weights + LM head + KV,
# profiles/decode_persistent_full_4layer.md; traffic grows in proportion to
# the bytes streamed, so the ratio scales a launch of the full model), and
# the body GEMV kernel on the gate_up shape
# (profiles/gemv_kernel_gate_up_lm_head_config1.md).
NCU_TRAFFIC_PER_BYTE = {"persistent": 1.0550, "gemv": 1.001}
# The persistent kernel's phases from the phase-trace build
# (profiles/decode_persistent_phases_config0.md): per segment, weight + scale
# bytes over the longest CTA's tile phase (GB/s), and over the segment span.
PERSISTENT_PHASES = {"qkv": (5136, 1031), "o": (3731, 356), "gate_up": (4703, 2518), "down": (4099, 1396),
                     "lm_head": (4989, 4440)}


def parse_args():
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=64)
    parser.add_argument("--warmup", type=int, default=8)
    parser.add_argument("--impl", choices=("ours", "reference"), default="ours")
    parser.add_argument("--kv-dtype", choices=("float16", "float32"), default="float16")
    parser.add_argument("--seed", type=int, default=0)
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--workload", choices=("decode", "gemv", "batch", "prefill", "gemm", "attention", "tp"),
                        default="decode",
                        help="decode: config 0 (the headline); gemv: config 1 body GEMV; attention: config 2; "
                             "batch: config 3 batched decode; prefill / tp: config 4; gemm: the a13 GEMM")
    parser.add_argument("--shapes", default="q,k,v,o,gate,up,down",
                        help="gemv workload: comma-separated projection names")
    parser.add_argument("--iters", type=int, default=200, help="gemv workload: timed launches per shape")
    parser.add_argument("--mode", choices=("persistent", "chain"), default="persistent",
                        help="decode step: one persistent kernel per token, or the PDL kernel chain")
    parser.add_argument("--gemm-shapes", default="qkv,o,gate_up,down,lm_head", help="gemm workload: shapes")
    parser.add_argument("--gemm-m", default="64,2048", help="gemm workload: token counts")
    parser.add_argument("--attn-cases", default="1x512,1x4096,1x32768,32x512,32x4096,32x32768",
                        help="attention workload: batch x context [x splits] cases")
    parser.add_argument("--batch", type=int, default=64, help="batch workload: sequences")
    parser.add_argument("--prompt-len", type=int, default=2048, help="batch / prefill workloads: prompt tokens")
    parser.add_argument("--prefill-attention", choices=("tensor", "exact"), default="tensor",
                        help="prefill workload: tcgen05 attention (tolerance) or the decode-order fp32 kernel")
    parser.add_argument("--batch-attention", choices=("tensor", "exact"), default="tensor",
                        help="batch workload: the tcgen05 attention (tolerance) or the decode-order fp32 one")
    parser.add_argument("--batch-splits", type=int, default=16,
                        help="batch workload: attention splits per sequence (the tensor kernel: at most this)")
    parser.add_argument("--kernel-shares", action="store_true",
                        help="batch workload: add the per-kernel device-time shares of 2 more steps (torch "
                             "profiler, CUDA activity), taken after the timed regions")
    parser.add_argument("--context", type=int, default=4096, help="tp workload: context before decoding")
    parser.add_argument("--layers", type=int, default=None,
                        help="override the layer count (a smaller model for profiling captures; not the headline)")
    return parser.parse_args()


def measured_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm_gbs": float(data["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML in a thread."""

    def __init__(self, index: int):
        self.index, self.samples, self.reasons = index, [], set()
        self._stop = threading.Event()
        self._thread = None
        self.max_mhz = None

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._handle = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM)
        except Exception as exc:  # NVML missing: report no clocks rather than fail
            self._nvml = None
            self.error = str(exc)
            return self
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()
        return self

    def _run(self):
        n = self._nvml
        names = {
            "hw_slowdown": getattr(n, "nvmlClocksEventReasonHwSlowdown", 0x8),
            "hw_thermal_slowdown": getattr(n, "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
            "sw_thermal_slowdown": getattr(n, "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
            "sw_power_cap": getattr(n, "nvmlClocksEventReasonSwPowerCap", 0x4),
            "hw_power_brake_slowdown": getattr(n, "nvmlClocksEventReasonHwPowerBrakeSlowdown", 0x80),
        }
        while not self._stop.is_set():
            try:
                self.samples.append(n.nvmlDeviceGetClockInfo(self._handle, n.NVML_CLOCK_SM))
                mask = n.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
                self.reasons.update(name for name, bit in names.items() if mask & bit)
            except Exception:
                pass
            time.sleep(0.005)

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread:
            self._thread.join()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def body_gemv_roofline(torch, model, state, peak_gbs) -> dict:
    """Average duration of the body GEMV kernel over all 144 launches of a
    token, each launched alone (no programmatic overlap) and timed with CUDA
    events on the stream they run on, after a sleep kernel so the host has
    queued every launch before the first event."""
    import ctypes

    from harsh4b_b200._lib import check, lib

    stream = state.stream
    body_bytes = sum(t.numel() * t.element_size() for t in (
        model.w_qkv, model.s_qkv, model.w_o, model.s_o, model.w_gate_up, model.s_gate_up, model.w_down,
        model.s_down))
    head_bytes = model.embedding.numel() + model.embedding_scales.numel() * 4
    start, mid, end = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        torch.cuda._sleep(50_000_000)
        start.record(stream)
        for layer in range(model.n_layers):
            for stage in (1, 3, 4, 5):
                check(lib().h4b_decode_stage(ctypes.byref(model.desc), ctypes.byref(state.desc), stage, layer,
                                             stream.cuda_stream), "h4b_decode_stage")
        mid.record(stream)
        check(lib().h4b_decode_stage(ctypes.byref(model.desc), ctypes.byref(state.desc), 6, 0,
                                     stream.cuda_stream), "h4b_decode_stage")
        end.record(stream)
    stream.synchronize()
    body_s = start.elapsed_time(mid) / 1000.0
    head_s = mid.elapsed_time(end) / 1000.0
    launches = 4 * model.n_layers
    achieved = body_bytes / body_s / 1e9
    traffic = None
    if NCU_TRAFFIC_PER_BYTE["gemv"] is not None:
        traffic = round(body_bytes / launches * NCU_TRAFFIC_PER_BYTE["gemv"])
    return {"bound": "hbm", "kernel": "gemv_kernel (body: qkv, o, gate/up, down)",
            "achieved": round(achieved, 1), "peak": peak_gbs, "unit": "GB/s", "frac": round(achieved / peak_gbs, 4),
            "traffic": traffic, "bytes_per_launch": round(body_bytes / launches),
            "avg_launch_us": round(body_s / launches * 1e6, 3), "launches": launches,
            "lm_head_gbs": round(head_bytes / head_s / 1e9, 1), "lm_head_us": round(head_s * 1e6, 2)}


def oracle_decode_timing(checkpoint, prompt, warmup: int, steps: int) -> dict:
    """The reference's CPU decode as restated by the oracle, on all host
    cores: the prompt fed untimed (all of it unless that would take more
    than ~90 s here), `warmup` untimed greedy tokens, then `steps` timed
    greedy tokens -- the same contexts as the GPU arm's timed steps."""
    import oracle

    threads = oracle.configure_threads(os.cpu_count())
    sys.path.insert(0, str(ROOT / "tests"))
    from _models import oracle_model

    model = oracle_model(checkpoint)
    state = model.new_state(len(prompt) + warmup + steps + 1)
    t0 = time.perf_counter()
    logits = model.forward_token(int(prompt[0]), state)
    per_token = time.perf_counter() - t0
    prefill = min(len(prompt), max(1, int(90.0 / max(per_token, 1e-3))))
    for token in prompt[1:prefill]:
        logits = model.forward_token(int(token), state)
    token = int(logits.argmax())
    for _ in range(warmup):
        token = int(model.forward_token(token, state).argmax())
    started = time.perf_counter()
    for _ in range(steps):
        token = int(model.forward_token(token, state).argmax())
    elapsed = time.perf_counter() - started
    return {"value": round(steps / elapsed, 3), "elapsed": elapsed, "prefill": prefill, "threads": threads,
            "cores": oracle.max_threads(),
            "sample": f"{steps} greedy decode tokens at batch 1 after a {prefill}-token prefill and {warmup} "
                      f"warm-up tokens (context {prefill + warmup + 1}..{prefill + warmup + steps}), "
                      f"config-0 weights, {threads} OpenMP threads"}


def cpu_baseline(checkpoint, prompt, warmup: int, steps: int) -> dict:
    """The oracle on this host's cores over the GPU arm's own timed steps."""
    t = oracle_decode_timing(checkpoint, prompt, warmup, steps)
    return {"value": t["value"], "unit": "tok/s", "cores": t["cores"], "kind": "port", "sample": t["sample"],
            "cpu": cpu_model()}


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference(args, rank) -> int:
    if rank != 0:
        return 0
    from harsh4b_b200.synthetic import qwen3_4b_config, synthetic_checkpoint, synthetic_prompt

    config = qwen3_4b_config()
    checkpoint = synthetic_checkpoint(config, seed=args.seed)
    prompt = synthetic_prompt(config, PROMPT, seed=args.seed)
    t = oracle_decode_timing(checkpoint, prompt, args.warmup, args.steps)
    value, elapsed, prefill, sample = t["value"], t["elapsed"], t["prefill"], t["sample"]
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(elapsed / args.steps * 1000, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int4xint8", "data": "synthetic", "impl": "reference",
        "config": {"workload": "config0: Qwen3-4B int4 synthetic checkpoint, 128-token random prompt, "
                               "batch-1 greedy decode", "prompt": prefill, "kv_dtype": "float32",
                   "parallelism": "replicas"},
        "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": t["cores"], "kind": "port",
                         "sample": sample, "cpu": cpu_model()},
        "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args, rank, world, local_rank, dist) -> int:
    import torch

    from harsh4b_b200.model import CudaQwen
    from harsh4b_b200.synthetic import qwen3_4b_config, synthetic_checkpoint, synthetic_prompt

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    config = qwen3_4b_config(**({"num_hidden_layers": args.layers} if args.layers else {}))
    checkpoint = synthetic_checkpoint(config, seed=args.seed)
    # every replica decodes its own random prompt
    prompt = synthetic_prompt(config, PROMPT, seed=args.seed + rank)
    model = CudaQwen.from_checkpoint(checkpoint, kv_dtype=args.kv_dtype, device=device, mode=args.mode)
    capacity = PROMPT + args.warmup + args.steps + 1

    def barrier():
        if dist is not None:
            dist.barrier(device_ids=[local_rank])

    # ---- value: device-resident decode ----
    state = model.new_state(capacity)
    for token in prompt:
        model.forward_token(token, state)
    first = state.next_token_host()
    model.generate_greedy(first, state, args.warmup)
    token = state.next_token_host()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clocks:
        with torch.cuda.stream(state.stream):
            start.record(state.stream)
        model.generate_greedy(token, state, args.steps)
        with torch.cuda.stream(state.stream):
            end.record(state.stream)
        torch.cuda.synchronize()
    barrier()
    elapsed = start.elapsed_time(end) / 1000.0
    last_token = state.next_token_host()
    status = model.status()

    # ---- e2e: host round trip per token (token id in from pinned host memory,
    # greedy id out) through CudaQwen.decode_greedy ----
    e2e_state = model.new_state(capacity)
    for token_id in prompt:
        model.forward_token(token_id, e2e_state)
    token = e2e_state.next_token_host()
    for _ in range(args.warmup):
        token = model.decode_greedy(token, e2e_state)
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    e_start.record(e2e_state.stream)
    for _ in range(args.steps):
        token = model.decode_greedy(token, e2e_state)
    e_end.record(e2e_state.stream)
    torch.cuda.synchronize()
    barrier()
    e2e_elapsed = e_start.elapsed_time(e_end) / 1000.0

    # ---- roofline of the dominant kernel ----
    peaks = measured_peaks()
    roof_state = model.new_state(capacity)
    for token_id in prompt[:4]:
        model.forward_token(token_id, roof_state)
    gemv_alone = body_gemv_roofline(torch, model, roof_state, peaks["hbm_gbs"])
    state.close(); e2e_state.close(); roof_state.close()

    times = torch.tensor([elapsed, e2e_elapsed], dtype=torch.float64, device=device)
    if dist is not None:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    elapsed, e2e_elapsed = float(times[0]), float(times[1])
    tp_record = tp_subrecord(args, checkpoint, rank, world, local_rank, dist) if world > 1 else None
    if rank != 0:
        return 0
    value = world * args.steps / elapsed
    kv_bytes = 2 if args.kv_dtype == "float16" else 4
    bytes_per_token = model.weight_bytes + model.n_layers * 2 * model.kv_size * kv_bytes * (
        PROMPT + args.warmup + args.steps // 2)
    if args.mode == "persistent":
        # One kernel launch per token: its algorithmic bytes over its event-timed duration.
        achieved = bytes_per_token * args.steps / elapsed / 1e9
        ratio = NCU_TRAFFIC_PER_BYTE["persistent"]
        roofline = {"bound": "hbm", "kernel": "decode_persistent_kernel (whole token)", "achieved": round(achieved, 1),
                    "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                    "traffic": round(bytes_per_token * ratio) if ratio else None, "bytes_per_launch": bytes_per_token,
                    "avg_launch_us": round(elapsed / args.steps * 1e6, 2), "launches": args.steps,
                    "peak_source": peaks["source"], "gemv_isolated": gemv_alone,
                    "gemv_phases": {"source": "phase-trace build, profiles/decode_persistent_phases_config0.md",
                                    "unit": "GB/s", **{k: {"tile_phase": v[0], "segment": v[1],
                                                           "tile_phase_frac": round(v[0] / peaks["hbm_gbs"], 3)}
                                                       for k, v in PERSISTENT_PHASES.items()}}}
    else:
        roofline = dict(gemv_alone, peak_source=peaks["source"])
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(elapsed / args.steps * 1000, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int4xint8", "data": "synthetic",
        "config": {"workload": "config0: Qwen3-4B int4 synthetic checkpoint (seed 0), 128-token random prompt, "
                               "batch-1 greedy decode", "prompt": PROMPT, "kv_dtype": args.kv_dtype,
                   "layers": model.n_layers, "decode_step": args.mode,
                   "context": [PROMPT + args.warmup, PROMPT + args.warmup + args.steps],
                   "l2": "inputs larger than L2 (1.82 GB of weights streamed per token)",
                   "parallelism": f"replicas x{world}"},
        "e2e": {"value": round(world * args.steps / e2e_elapsed, 2), "unit": "tok/s", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 4},
        "gpu_launches": args.steps * (1 if args.mode == "persistent" else 5 * model.n_layers + 3),
        "step_roofline": {"bytes_per_token": bytes_per_token,
                          "achieved_gbs": round(bytes_per_token * args.steps / elapsed / 1e9, 1),
                          "frac": round(bytes_per_token * args.steps / elapsed / 1e9 / peaks["hbm_gbs"], 4)},
        "roofline": roofline,
        "clocks": clocks.summary(),
        "device_status": status,
        "last_token": last_token,
    }
    if tp_record is not None:
        line["tp"] = tp_record
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(checkpoint, prompt, args.warmup, args.steps)
    print(json.dumps(line), flush=True)
    return 0


def tp_subrecord(args, checkpoint, rank, world, local_rank, dist, context: int = 4096,
                 steps: int = 20, warmup: int = 3) -> dict:
    """Config 4 on the same N GPUs, reported beside the replica line:
    tensor-parallel batch-1 decode (tp = N) from a context of `context`
    positions (K/V filled with N(0,1) values), the token captured in one
    CUDA graph with the one-shot P2P exchanges. p50 latency per token (wall
    and device), the communication alone (the token's collectives issued
    without the kernels; this path does not overlap them, so it is exposed),
    and whether 8 greedy tokens after a real 16-token prompt equal those of
    the single-GPU decode with the same attention splits (the chain kernels,
    16 splits), which the sharding must reproduce bit for bit."""
    import numpy as np
    import torch

    from harsh4b_b200.model import CudaQwen
    from harsh4b_b200.synthetic import synthetic_prompt
    from harsh4b_b200.tp import TensorParallelQwen

    device = torch.device("cuda", local_rank)
    prompt = synthetic_prompt(checkpoint.config, 16, seed=args.seed)  # the same on every rank
    tp = TensorParallelQwen(checkpoint, kv_dtype=args.kv_dtype, device=device)
    # greedy tokens after a real prompt, against one GPU
    check_state = tp.new_state(32)
    token = None
    for t in prompt[:16]:
        token, _ = tp.forward_token(int(t), check_state, graph=False)
    tp_tokens = [token]
    for _ in range(7):
        token, _ = tp.forward_token(token, check_state, graph=False)
        tp_tokens.append(token)
    match = None
    if rank == 0:
        single = CudaQwen.from_checkpoint(checkpoint, kv_dtype=args.kv_dtype, device=device, mode="chain",
                                          attn_splits=16)
        st = single.new_state(32)
        for t in prompt[:16]:
            single.forward_token(int(t), st)
        one = [st.next_token_host()]
        for _ in range(7):
            single.forward_token(one[-1], st)
            one.append(st.next_token_host())
        match = one == tp_tokens
        st.close()
        del single
    # every rank waits for rank 0's single-GPU check: the P2P exchanges poll
    # for their peers with a bounded wait
    torch.cuda.synchronize()
    dist.barrier(device_ids=[local_rank])
    # latency from a long context
    state = tp.new_state(context + warmup + steps + 1)
    g = torch.Generator(device=device).manual_seed(args.seed + rank)
    state.k_cache.normal_(generator=g)
    state.v_cache.normal_(generator=g)
    state.position_dev.fill_(context)
    state.position = context
    token = int(np.random.default_rng(args.seed).integers(0, tp.vocab))
    for _ in range(warmup):
        token, _ = tp.forward_token(token, state, graph=True)
    walls, device_ms = [], []
    dist.barrier(device_ids=[local_rank])
    torch.cuda.synchronize()
    for _ in range(steps):
        start, end = _event_pair(torch)
        t0 = time.perf_counter()
        start.record()
        token, _ = tp.forward_token(token, state, graph=True)
        end.record()
        torch.cuda.synchronize()
        walls.append(time.perf_counter() - t0)
        device_ms.append(start.elapsed_time(end))
    tp.release_graphs()
    # config 4's prefill on the same ranks: a 2048-token prompt, sharded GEMMs
    # with the [M] absmax and [M][H] int32 all-reduces between them
    prefill_ids = [int(t) for t in np.random.default_rng([args.seed, 2048]).integers(0, tp.vocab, 2048)]
    pre_state = tp.new_state(2048 + 1)
    tp.prefill(prefill_ids, pre_state)  # warm-up (scratch, communicators)
    pre_state.close()
    pre_state = tp.new_state(2048 + 1)
    dist.barrier(device_ids=[local_rank])
    torch.cuda.synchronize()
    p_start, p_end = _event_pair(torch)
    p_start.record()
    tp.prefill(prefill_ids, pre_state)
    p_end.record()
    torch.cuda.synchronize()
    prefill_ms = p_start.elapsed_time(p_end)
    pre_state.close()
    tp.model._prefill_scratch = None
    H, L = tp.model.hidden, tp.model.n_layers
    amax = torch.zeros(1, device=device)
    acc = torch.zeros(H, dtype=torch.int32, device=device)
    pairs = [torch.zeros(2, dtype=torch.float64, device=device) for _ in range(world)]

    def comm_token():
        for _ in range(2 * L):
            dist.all_reduce(amax, op=dist.ReduceOp.MAX)
            dist.all_reduce(acc, op=dist.ReduceOp.SUM)
        dist.all_gather(pairs, pairs[rank].clone())

    comm_token()
    torch.cuda.synchronize()
    c_start, c_end = _event_pair(torch)
    c_start.record()
    for _ in range(5):
        comm_token()
    c_end.record()
    torch.cuda.synchronize()
    stats = torch.tensor([statistics.median(walls) * 1000, statistics.median(device_ms),
                          c_start.elapsed_time(c_end) / 5, prefill_ms], dtype=torch.float64, device=device)
    dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    status = tp.model.status()
    tp.close()
    p50, dev, comm, pre = (round(float(v), 4) for v in stats.cpu())
    return {"parallelism": f"tp{world}", "context": context, "p50_ms": p50, "device_ms_p50": dev,
            "exposed_comm_ms": comm, "tok_s": round(1000.0 / p50, 2), "steps": steps,
            "exchange": "one-shot P2P kernels over NVLink peer memory, token in one CUDA graph",
            "greedy_match_single_gpu": match,
            "prefill_2048": {"ms": pre, "tok_s": round(2048 / pre * 1000, 1),
                             "exchange": "NCCL all-reduce of [M] absmax (MAX) and [M][H] int32 sums (SUM)"},
            "device_status": status}


GEMV_SHAPES = {"q": (4096, 2560), "k": (1024, 2560), "v": (1024, 2560), "o": (2560, 4096),
               "gate": (9728, 2560), "up": (9728, 2560), "down": (2560, 9728), "qkv": (6144, 2560),
               "gate_up": (19456, 2560), "lm_head": (151936, 2560)}


def run_gemv(args) -> int:
    """Config 1: the fused quantise + int4 GEMV alone, per projection shape.
    Weight copies rotate so the bytes read per launch come from HBM (the
    copies together exceed the 126 MB L2); launches are queued behind a
    sleep kernel and timed with CUDA events on their stream. `us`/`gbs`: each
    launch waits for the previous one to finish; `pdl_chain`: the same launches
    with programmatic dependent launch (as the decode chain runs them), so a
    launch streams its weights while the previous one finishes."""
    import numpy as np
    import torch

    import oracle
    from harsh4b_b200 import ops
    from harsh4b_b200.synthetic import int4_matrix, outlier_activation, row_scales

    peaks = measured_peaks()
    results = {}
    stream = torch.cuda.current_stream()
    for name in args.shapes.split(","):
        rows, width = GEMV_SHAPES[name]
        rng = np.random.default_rng([1, rows, width])
        packed, scales = int4_matrix(rng, rows, width), row_scales(rng, rows)
        x = outlier_activation(width, seed=rows)
        weights, scale_t = torch.from_numpy(packed).cuda(), torch.from_numpy(scales).cuda()
        bytes_per_launch = rows * width // 2 + 4 * rows + 4 * width
        copies = max(1, -(-300_000_000 // bytes_per_launch))
        ws = [weights] + [weights.clone() for _ in range(copies - 1)]
        ss = [scale_t] + [scale_t.clone() for _ in range(copies - 1)]
        xt = torch.from_numpy(x).cuda()
        out = torch.empty(rows, dtype=torch.float32, device="cuda")
        acc = torch.empty(rows, dtype=torch.int32, device="cuda")
        ops.int4_gemv_fused_quant(xt, ws[0], ss[0], out=out, acc=acc)
        q = np.empty(width, dtype=np.int8)
        _, want_acc = oracle.int4_gemv(q, packed, scales, oracle.quantize_activation(x, q))
        got_acc = acc.cpu().numpy()
        exact = bool(np.array_equal(got_acc, want_acc))
        mismatch = np.nonzero(got_acc != want_acc)[0]
        scale_slot = torch.empty(1, dtype=torch.float32, device="cuda")

        def timed(pdl: bool) -> float:
            for i in range(min(3, args.iters)):
                ops.int4_gemv_fused_quant(xt, ws[i % copies], ss[i % copies], out=out, scale=scale_slot, pdl=pdl)
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            torch.cuda._sleep(20_000_000)
            start.record(stream)
            for i in range(args.iters):
                ops.int4_gemv_fused_quant(xt, ws[i % copies], ss[i % copies], out=out, scale=scale_slot, pdl=pdl)
            end.record(stream)
            torch.cuda.synchronize()
            return start.elapsed_time(end) * 1000.0 / args.iters

        us, us_pdl = timed(False), timed(True)
        gbs, gbs_pdl = bytes_per_launch / us / 1e3, bytes_per_launch / us_pdl / 1e3
        from harsh4b_b200._lib import device_status
        results[name] = {"rows": rows, "width": width, "us": round(us, 3), "gbs": round(gbs, 1),
                         "frac": round(gbs / peaks["hbm_gbs"], 4),
                         "pdl_chain": {"us": round(us_pdl, 3), "gbs": round(gbs_pdl, 1),
                                       "frac": round(gbs_pdl / peaks["hbm_gbs"], 4)},
                         "int32_bit_exact": exact, "device_status": device_status()}
        if not exact:
            results[name]["mismatched_rows"] = int(mismatch.size)
            results[name]["first_mismatches"] = mismatch[:6].tolist()
            results[name]["diffs"] = (got_acc[mismatch[:6]].astype(np.int64) - want_acc[mismatch[:6]]).tolist()
        del ws, ss
    line = {"metric": "body GEMV HBM GB/s (fused int8 quantisation + int4 GEMV), batch 1",
            "unit": "GB/s", "peak": peaks["hbm_gbs"], "peak_source": peaks["source"], "iters": args.iters,
            "config": {"workload": "config1: body projections, fp32 N(0,1) activation with 0.5% x20 outliers",
                       "l2": "rotating weight copies > 300 MB per shape"}, "shapes": results}
    print(json.dumps(line), flush=True)
    return 0


def _event_pair(torch):
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def run_batch(args, rank=0, world=1, local_rank=0, dist=None) -> int:
    """Config 3: batched greedy decode of B sequences (default 64) after a
    prompt of --prompt-len random ids each, body projections on the tcgen05
    GEMM. `value` = B x K tokens over K device-fed steps (generate_batch);
    `e2e` = the same K steps through forward_batch with the B token ids
    copied in and the B greedy ids read back every step. The prompts are fed
    through forward_batch before timing (not timed). Under torchrun every
    rank runs its own batch of B sequences (data-parallel replicas, no
    collective on the data path); `value` sums the ranks' tokens over the
    max-over-ranks time."""
    import numpy as np
    import torch

    torch.cuda.set_device(local_rank)

    def barrier():
        if dist is not None:
            dist.barrier(device_ids=[local_rank])

    from harsh4b_b200.model import CudaQwen
    from harsh4b_b200.synthetic import qwen3_4b_config, synthetic_checkpoint

    peaks = measured_peaks()
    B, P = args.batch, args.prompt_len
    config = qwen3_4b_config(**({"num_hidden_layers": args.layers} if args.layers else {}))
    model = CudaQwen.from_checkpoint(synthetic_checkpoint(config, seed=args.seed), kv_dtype=args.kv_dtype,
                                     mode="chain")
    rng = np.random.default_rng([args.seed, B, P, rank])
    prompts = rng.integers(0, model.vocab, size=(B, P))
    capacity = P + 2 * (args.warmup + args.steps) + 2 + (2 if args.kernel_shares else 0)
    splits = args.batch_splits
    state = model.new_batch_state(B, capacity, attn_splits=splits, attention=args.batch_attention)
    t0 = time.perf_counter()
    for i in range(P):
        model.forward_batch(prompts[:, i], state)
    torch.cuda.synchronize()
    prompt_s = time.perf_counter() - t0
    model.generate_batch(state, args.warmup)
    start, end = _event_pair(torch)
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clocks:
        start.record()
        model.generate_batch(state, args.steps)
        end.record()
        torch.cuda.synchronize()
    barrier()
    elapsed = start.elapsed_time(end) / 1000.0
    ctx0 = P + args.warmup
    # e2e: host ids in, host greedy ids out, every step
    host_next = torch.empty(B, dtype=torch.int32).pin_memory()
    tokens = state.next_tokens.cpu().numpy()
    for _ in range(args.warmup):
        model.forward_batch(tokens, state)
        host_next.copy_(state.next_tokens)
        tokens = host_next.numpy().copy()
    e_start, e_end = _event_pair(torch)
    barrier()
    torch.cuda.synchronize()
    e_start.record()
    for _ in range(args.steps):
        model.forward_batch(tokens, state)
        host_next.copy_(state.next_tokens)
        tokens = host_next.numpy().copy()
    e_end.record()
    torch.cuda.synchronize()
    barrier()
    e2e_elapsed = e_start.elapsed_time(e_end) / 1000.0
    times = torch.tensor([elapsed, e2e_elapsed], dtype=torch.float64, device="cuda")
    if dist is not None:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    elapsed, e2e_elapsed = float(times[0]), float(times[1])
    status = model.status()
    if rank != 0:
        return 0
    shares = kernel_shares(torch, lambda: model.generate_batch(state, 2), 2) if args.kernel_shares else None
    kv_bytes = 2 if args.kv_dtype == "float16" else 4
    per_pos = model.n_layers * 2 * model.kv_size * kv_bytes
    mean_ctx = ctx0 + (args.steps + 1) / 2
    bytes_per_step = model.weight_bytes + B * per_pos * mean_ctx
    achieved = bytes_per_step * args.steps / elapsed / 1e9
    line = {
        "metric": "batched decode tok/s Qwen3-4B int4 (config 3)",
        "value": round(world * B * args.steps / elapsed, 1),
        "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(elapsed / args.steps * 1000, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int4xint8", "data": "synthetic",
        "config": {"workload": f"config3: batch {B}, {P}-token random prompts, greedy decode, tcgen05 GEMM body",
                   "batch": B, "prompt": P, "kv_dtype": args.kv_dtype, "layers": model.n_layers,
                   "context": [ctx0, ctx0 + args.steps], "l2": "inputs larger than L2",
                   "prompt_feed_s": round(prompt_s, 2), "parallelism": f"replicas x{world}",
                   "attention": args.batch_attention, "attn_splits": splits},
        "e2e": {"value": round(world * B * args.steps / e2e_elapsed, 1), "unit": "tok/s",
                "h2d_bytes_per_step": 4 * B, "d2h_bytes_per_step": 4 * B},
        "roofline": {"bound": "hbm", "kernel": "whole batched step (weights + every sequence's K/V)",
                     "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4), "bytes_per_step": int(bytes_per_step),
                     "peak_source": peaks["source"]},
        "clocks": clocks.summary(), "device_status": status,
    }
    if shares is not None:
        line["kernel_shares"] = shares
    print(json.dumps(line), flush=True)
    return 0


def kernel_shares(torch, fn, steps: int) -> dict:
    """Per-kernel device time of `fn` (torch profiler, CUDA activity): per
    kernel name its launches and microseconds per step and its share of all
    the kernels' time. Taken under a profiler, so only the shares are read;
    the bench's timings come from CUDA events."""
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    totals = {}
    for event in prof.events():
        if event.device_type != torch.autograd.DeviceType.CUDA:
            continue
        name = event.name.split("(")[0].replace("void ", "").strip()
        if "int4_gemm_tc" not in name:
            name = name.split("<")[0]
        entry = totals.setdefault(name, [0, 0.0])
        entry[0] += 1
        entry[1] += event.device_time_total
    whole = sum(t for _, t in totals.values()) or 1.0
    return {name: {"launches_per_step": n / steps, "us_per_step": round(t / steps, 1), "share": round(t / whole, 4)}
            for name, (n, t) in sorted(totals.items(), key=lambda kv: -kv[1][1])}


def run_prefill(args) -> int:
    """Config 4's prefill: one --prompt-len-token prompt (default 2048) fed in
    one CudaQwen.prefill call (tcgen05 GEMMs over all prompt rows). A step is
    one whole prefill into a fresh session; `value` is prompt tok/s. The
    roofline is the tensor pipe: 2 x body MACs per prompt row (int8 ops)."""
    import numpy as np
    import torch

    from harsh4b_b200.model import CudaQwen
    from harsh4b_b200.synthetic import qwen3_4b_config, synthetic_checkpoint

    P = args.prompt_len
    config = qwen3_4b_config(**({"num_hidden_layers": args.layers} if args.layers else {}))
    model = CudaQwen.from_checkpoint(synthetic_checkpoint(config, seed=args.seed), kv_dtype=args.kv_dtype,
                                     mode="chain")
    ids = np.random.default_rng([args.seed, P]).integers(0, model.vocab, size=P)
    state = model.new_state(P + 1)
    for _ in range(args.warmup):
        state.reset()
        model.prefill(ids, state, max_tokens=P, attention=args.prefill_attention)
    times = []
    with ClockSampler(torch.cuda.current_device()) as clocks:
        for _ in range(args.steps):
            state.reset()
            start, end = _event_pair(torch)
            with torch.cuda.stream(state.stream):
                start.record(state.stream)
            model.prefill(ids, state, max_tokens=P, attention=args.prefill_attention)
            with torch.cuda.stream(state.stream):
                end.record(state.stream)
            torch.cuda.synchronize()
            times.append(start.elapsed_time(end) / 1000.0)
    elapsed = sum(times)
    attention = prefill_attention_record(model, state, P, args.prefill_attention)
    H, I, Q, KV = model.hidden, model.intermediate, model.q_size, model.kv_size
    body_macs = model.n_layers * (H * (Q + 2 * KV) + Q * H + H * 2 * I + I * H)
    ops_per_prefill = 2 * body_macs * P + 2 * model.vocab * H
    achieved = ops_per_prefill * args.steps / elapsed / 1e12
    int8_peak = 2 * measured_bf16_tflops()
    line = {
        "metric": "prefill tok/s Qwen3-4B int4 (config 4 prefill)", "value": round(P * args.steps / elapsed, 1),
        "unit": "tok/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(elapsed / args.steps * 1000, 3), "p50_ms": round(statistics.median(times) * 1000, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int4xint8", "data": "synthetic",
        "config": {"workload": f"config4 prefill: {P}-token random prompt, one h4b_prefill call",
                   "prompt": P, "kv_dtype": args.kv_dtype, "layers": model.n_layers,
                   "attention": args.prefill_attention, "l2": "inputs larger than L2"},
        "roofline": {"bound": "tensor", "kernel": "whole prefill (int8 ops of every GEMM)",
                     "achieved": round(achieved, 1), "peak": round(int8_peak, 1), "unit": "TOP/s",
                     "frac": round(achieved / int8_peak, 4), "ops_per_step": int(ops_per_prefill),
                     "peak_source": "2 x measured bf16 dense (int8 dense rate is twice bf16 on B200)"},
        "attention": attention, "clocks": clocks.summary(), "device_status": model.status(),
    }
    print(json.dumps(line), flush=True)
    return 0


def prefill_attention_record(model, state, P: int, attention: str, reps: int = 20) -> dict:
    """The prompt attention kernel alone (h4b_prefill_attention on the last
    layer, after a prefill of P tokens from position 0), CUDA-event timed on
    the state's stream: algorithmic flops = 2 products x 2 flops x head_dim
    x sum of the rows' contexts x q heads."""
    import ctypes

    import torch

    from harsh4b_b200._lib import check, lib

    scratch = model._prefill_scratch
    call = lambda: check(lib().h4b_prefill_attention(ctypes.byref(model.desc), ctypes.byref(state.desc),
                                                     ctypes.byref(scratch.desc), P, model.n_layers - 1,
                                                     state.stream.cuda_stream), "h4b_prefill_attention")
    with torch.cuda.stream(state.stream):
        for _ in range(3):
            call()
        start, end = _event_pair(torch)
        start.record(state.stream)
        for _ in range(reps):
            call()
        end.record(state.stream)
    torch.cuda.synchronize()
    us = start.elapsed_time(end) * 1000.0 / reps
    flops = 4 * model.head_dim * (P * (P + 1) // 2) * model.heads
    peak = measured_bf16_tflops()
    achieved = flops / us / 1e6
    tensor = attention == "tensor"
    kernel = "prefill_attention_tc_kernel" if tensor else "prefill_attention_block_kernel"
    return {"kernel": kernel, "bound": "tensor" if tensor else "fp32 FMA (CUDA cores, the decode order)",
            "us_per_layer": round(us, 2), "flops_per_layer": flops,
            "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
            "peak_source": "measured bf16 dense burst (fp16 runs at the bf16 rate)",
            "note": "algorithmic flops; the tensor kernel issues twice as many MMA flops (q and p as hi + lo fp16)"}


def measured_bf16_tflops() -> float:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return float(json.loads(path.read_text())["bf16_tflops"])
    return 1590.0


def _graph_time(torch, fn, reps: int, warmup: int = 3) -> float:
    """Seconds per call of `fn`, captured `reps` times in one CUDA graph."""
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(reps):
            fn()
    graph.replay()
    torch.cuda.synchronize()
    start, end = _event_pair(torch)
    start.record()
    graph.replay()
    end.record()
    torch.cuda.synchronize()
    del graph
    return start.elapsed_time(end) / 1000.0 / reps


GEMM_SHAPES = {"qkv": (6144, 2560), "o": (2560, 4096), "gate_up": (19456, 2560), "down": (2560, 9728),
               "lm_head": (151936, 2560)}


def run_gemm(args) -> int:
    """a13: the batched int4 x int8 GEMM per body shape at M = 64 (batched
    decode, HBM-bound) and M = 2048 (prefill, tensor-bound), tcgen05 kernel
    and the mma.sync kernel, each launch captured in a CUDA graph. Weight
    copies rotate so M = 64 reads come from HBM; outputs are checked equal
    between the kernels."""
    import torch

    from harsh4b_b200 import ops

    peaks = measured_peaks()
    int8_peak = 2 * measured_bf16_tflops()
    results = []
    g = torch.Generator(device="cuda").manual_seed(args.seed)
    for M in (int(m) for m in args.gemm_m.split(",")):
        for name in args.gemm_shapes.split(","):
            N, K = GEMM_SHAPES[name]
            if name == "lm_head" and M > 64:
                continue
            copies = max(1, -(-300_000_000 // (N * K // 2)))
            ws = [torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device="cuda", generator=g)
                  for _ in range(copies)]
            scales = torch.rand(N, device="cuda", generator=g)
            x8 = torch.randint(-127, 128, (M, K), dtype=torch.int8, device="cuda", generator=g)
            act = torch.rand(M, device="cuda", generator=g) * 1e-2
            sums = x8.to(torch.int32).sum(1, dtype=torch.int32)
            outs = {k: torch.empty(M, N, device="cuda") for k in ("tcgen05", "mma_sync")}
            row = {"M": M, "shape": name, "N": N, "K": K}
            for kern in ("tcgen05", "mma_sync"):
                state = {"i": 0}

                def launch(kern=kern, state=state):
                    ops.int4_gemm(x8, act, sums, ws[state["i"] % copies], scales, out=outs[kern], kernel=kern)
                    state["i"] += 1

                sec = _graph_time(torch, launch, reps=max(copies, 8))
                ops_ = 2 * M * N * K
                row[kern] = {"us": round(sec * 1e6, 2), "tops": round(ops_ / sec / 1e12, 1),
                             "gbs": round((N * K // 2 + 4 * N + M * K + 4 * M * N) / sec / 1e9, 1)}
            if M <= 64:
                # the batched decode's form: K split over one CTA per SM (stream-K)
                # through a zeroed int32 buffer, finalised into out
                acc = torch.zeros(M * N, dtype=torch.int32, device="cuda")
                outs["split"] = torch.empty(M, N, device="cuda")
                state = {"i": 0}

                def launch_acc(state=state):
                    ops.int4_gemm_acc(x8, act, sums, ws[state["i"] % copies], scales, acc, out=outs["split"])
                    state["i"] += 1

                sec = _graph_time(torch, launch_acc, reps=max(copies, 8))
                row["tcgen05_acc"] = {"us": round(sec * 1e6, 2), "tops": round(2 * M * N * K / sec / 1e12, 1),
                                      "gbs": round((N * K // 2 + 4 * N + M * K + 4 * M * N) / sec / 1e9, 1)}
                row["equal_acc"] = bool(torch.equal(outs["split"], outs["tcgen05"]))
            row["equal"] = bool(torch.equal(outs["tcgen05"], outs["mma_sync"]))
            tc = row["tcgen05"]
            row["frac"] = (round(tc["gbs"] / peaks["hbm_gbs"], 4) if M <= 64 else round(tc["tops"] / int8_peak, 4))
            if M <= 64:
                row["frac_acc"] = round(row["tcgen05_acc"]["gbs"] / peaks["hbm_gbs"], 4)
            results.append(row)
            del ws
    line = {"metric": "batched int4 x int8 GEMM (a13): tcgen05 vs mma.sync", "unit": "us",
            "peaks": {"hbm_gbs": peaks["hbm_gbs"], "int8_tops": round(int8_peak, 1),
                      "int8_source": "2 x measured bf16 dense"},
            "config": {"workload": "a13 shapes at M = 64 (HBM-bound frac) and M = 2048 (tensor-bound frac)",
                       "l2": "rotating weight copies > 300 MB at M = 64"},
            "shapes": results}
    print(json.dumps(line), flush=True)
    return 0


def run_attention(args) -> int:
    """Config 2: the decode attention kernel (qk-RMSNorm, RoPE, KV append,
    split-K GQA over an fp16 cache) for 32 q / 8 kv heads at contexts 512,
    4096, 32768 and batch 1 and 32; the cache is filled with N(0,1) values.
    Batch 1 is the decode stage (h4b_decode_stage 2) of a session at the
    given position, batch 32 the batched kernel (h4b_batch_attention), both
    the exact fp32 kernels; every case also carries a `tensor` record, the
    tcgen05 batched kernel (h4b_batch_attention with attention="tensor") on
    the same shapes, batch 1 as a one-sequence batch."""
    import ctypes

    import torch

    from harsh4b_b200._lib import check, lib
    from harsh4b_b200.model import CudaQwen
    from harsh4b_b200.synthetic import qwen3_4b_config, synthetic_checkpoint

    peaks = measured_peaks()
    model = CudaQwen.from_checkpoint(synthetic_checkpoint(qwen3_4b_config(num_hidden_layers=1), seed=args.seed),
                                     kv_dtype="float16", mode="chain")
    results = []
    for case in args.attn_cases.split(","):
        fields = [int(v) for v in case.split("x")]
        batch, ctx = fields[0], fields[1]
        if len(fields) > 2:  # batch x context x splits
            splits = fields[2]
        else:  # enough CTAs for five per SM, at least 64 tokens per split
            splits = max(1, min(64, -(-5 * 148 // (model.kv_heads * batch)), ctx // 64))
        if batch == 1:
            st = model.new_state(ctx, attn_splits=splits)
            st.k_cache.normal_(); st.v_cache.normal_(); st.qkv.normal_()
            st.position_dev.fill_(ctx - 1)

            def launch(st=st):
                check(lib().h4b_decode_stage(ctypes.byref(model.desc), ctypes.byref(st.desc), 2, 0,
                                             torch.cuda.current_stream().cuda_stream), "h4b_decode_stage")
        else:
            st = model.new_batch_state(batch, ctx, attn_splits=splits, attention="exact")
            st.k_cache.normal_(); st.v_cache.normal_(); st.qkv.normal_()
            st.positions.fill_(ctx - 1)

            def launch(st=st):
                check(lib().h4b_batch_attention(ctypes.byref(model.desc), ctypes.byref(st.desc), 0,
                                                torch.cuda.current_stream().cuda_stream), "h4b_batch_attention")
        sec = _graph_time(torch, launch, reps=20)
        kv_bytes = batch * 2 * ctx * model.kv_size * 2
        case_line = {"batch": batch, "ctx": ctx, "splits": splits, "us": round(sec * 1e6, 2),
                     "gbs": round(kv_bytes / sec / 1e9, 1), "frac": round(kv_bytes / sec / 1e9 / peaks["hbm_gbs"], 4),
                     "kv_bytes": kv_bytes}
        del st
        torch.cuda.empty_cache()
        # the tcgen05 batched kernel on the same case (qk-norm / RoPE / append kernel + attention + merge;
        # batch 1 as a one-sequence batch)
        st = model.new_batch_state(batch, ctx, attn_splits=64, attention="tensor")
        st.k_cache.normal_(); st.v_cache.normal_(); st.qkv.normal_()
        st.positions.fill_(ctx - 1)

        def launch_tc(st=st):
            check(lib().h4b_batch_attention(ctypes.byref(model.desc), ctypes.byref(st.desc), 0,
                                            torch.cuda.current_stream().cuda_stream), "h4b_batch_attention")
        sec_tc = _graph_time(torch, launch_tc, reps=20)
        case_line["tensor"] = {"us": round(sec_tc * 1e6, 2), "gbs": round(kv_bytes / sec_tc / 1e9, 1),
                               "frac": round(kv_bytes / sec_tc / 1e9 / peaks["hbm_gbs"], 4)}
        del st
        torch.cuda.empty_cache()
        results.append(case_line)
    line = {"metric": "GQA decode attention GB/s of K/V read (config 2)", "unit": "GB/s",
            "peak": peaks["hbm_gbs"], "peak_source": peaks["source"],
            "config": {"workload": "config2: 32 q / 8 kv heads, d 128, fp16 KV N(0,1), RoPE + qk-norm in kernel",
                       "l2": "K/V of 1-32 sequences; 512-context batch-1 rows fit in L2 (graph replays reuse them)"},
            "cases": results, "device_status": model.status()}
    print(json.dumps(line), flush=True)
    return 0


def run_tp(args, rank, world, local_rank, dist) -> int:
    """Config 4 decode: tensor-parallel batch-1 decode on `world` GPUs from a
    context of --context tokens (the K/V cache is filled with N(0,1) values;
    the prefill is not part of this line). A step is one token through
    TensorParallelQwen.forward_token (all ranks, NCCL all-reduces of the o /
    down int32 sums and their scales, all-gather of the greedy candidates).
    Reports the p50 wall latency per token with the token captured in one
    CUDA graph (and, under "eager", dispatched call by call), the device time
    per token (max over ranks) and the communication alone: the same
    collectives issued without the kernels (exposed, since this path does not
    overlap them)."""
    import numpy as np
    import torch

    from harsh4b_b200.synthetic import qwen3_4b_config, synthetic_checkpoint
    from harsh4b_b200.tp import TensorParallelQwen

    device = torch.device("cuda", local_rank)
    config = qwen3_4b_config(**({"num_hidden_layers": args.layers} if args.layers else {}))
    model = TensorParallelQwen(synthetic_checkpoint(config, seed=args.seed), kv_dtype=args.kv_dtype, device=device)
    C = args.context
    state = model.new_state(C + 3 * (args.warmup + args.steps) + 1)  # three timed rounds
    g = torch.Generator(device=device).manual_seed(args.seed + rank)
    state.k_cache.normal_(generator=g)
    state.v_cache.normal_(generator=g)
    state.position_dev.fill_(C)
    state.position = C
    token = int(np.random.default_rng(args.seed).integers(0, model.vocab))

    def run(graph: bool):
        nonlocal token
        for _ in range(args.warmup):
            token, _ = model.forward_token(token, state, graph=graph)
        walls, device_ms = [], []
        dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize()
        for _ in range(args.steps):
            start, end = _event_pair(torch)
            t0 = time.perf_counter()
            start.record()
            token, _ = model.forward_token(token, state, graph=graph)
            end.record()
            torch.cuda.synchronize()
            walls.append(time.perf_counter() - t0)
            device_ms.append(start.elapsed_time(end))
        return statistics.median(walls) * 1000, statistics.median(device_ms)

    eager_wall, eager_dev = run(graph=False)
    model.comm = "nccl"  # the same token with NCCL collectives, for comparison
    nccl_wall, nccl_dev = run(graph=True)
    model.release_graphs()
    model.comm = "p2p"
    with ClockSampler(local_rank) as clocks:
        graph_wall, graph_dev = run(graph=True)
    model.release_graphs()
    # the collectives of one token alone
    H, L = model.model.hidden, model.model.n_layers
    amax = torch.zeros(1, device=device)
    acc = torch.zeros(H, dtype=torch.int32, device=device)
    pair = torch.zeros(2, dtype=torch.float64, device=device)
    pairs = [torch.zeros(2, dtype=torch.float64, device=device) for _ in range(world)]

    def comm_token():
        for _ in range(2 * L):
            dist.all_reduce(amax, op=dist.ReduceOp.MAX)
            dist.all_reduce(acc, op=dist.ReduceOp.SUM)
        dist.all_gather(pairs, pair)

    for _ in range(3):
        comm_token()
    torch.cuda.synchronize()
    c_start, c_end = _event_pair(torch)
    c_start.record()
    for _ in range(args.steps):
        comm_token()
    c_end.record()
    torch.cuda.synchronize()
    comm_ms = c_start.elapsed_time(c_end) / args.steps
    stats = torch.tensor([graph_wall, graph_dev, comm_ms, eager_wall, eager_dev, nccl_wall, nccl_dev],
                         dtype=torch.float64, device=device)
    dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    status = model.model.status()
    model.close()
    if rank != 0:
        return 0
    p50, dev, comm, eager_p50, eager_dev_p50, nccl_p50, nccl_dev_p50 = (float(v) for v in stats.cpu())
    line = {
        "metric": "tensor-parallel batch-1 decode latency Qwen3-4B int4 (config 4)", "value": round(1000.0 / p50, 2),
        "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(p50, 4),
        "p50_ms": round(p50, 4), "device_ms_p50": round(dev, 4),
        "exchange": "one-shot P2P kernels over NVLink peer memory, token captured in a CUDA graph",
        "eager": {"p50_ms": round(eager_p50, 4), "device_ms_p50": round(eager_dev_p50, 4)},
        "nccl_graph": {"p50_ms": round(nccl_p50, 4), "device_ms_p50": round(nccl_dev_p50, 4),
                       "collectives_alone_ms": round(comm, 4)},
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int4xint8",
        "data": "synthetic",
        "config": {"workload": f"config4 TP: batch 1 from context {C} (K/V filled with N(0,1) values)",
                   "context": C, "kv_dtype": args.kv_dtype, "layers": L, "parallelism": f"tp{world}",
                   "collectives_per_token": 4 * L + 1},
        "clocks": clocks.summary(), "device_status": status,
    }
    print(json.dumps(line), flush=True)
    return 0


def main() -> int:
    args = parse_args()
    single = {"gemv": run_gemv, "prefill": run_prefill, "gemm": run_gemm, "attention": run_attention}
    if args.workload in single:
        return single[args.workload](args)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank)
    dist = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as torch_dist

        torch.cuda.set_device(local_rank)
        torch_dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                      device_id=torch.device("cuda", local_rank))
        dist = torch_dist
    if args.workload == "tp" and dist is None:  # one rank: a process group of one
        import datetime

        import torch
        import torch.distributed as torch_dist

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29531")
        torch.cuda.set_device(local_rank)
        torch_dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=300),
                                      device_id=torch.device("cuda", local_rank))
        dist = torch_dist
    try:
        if args.workload == "tp":
            return run_tp(args, rank, world, local_rank, dist)
        if args.workload == "batch":
            return run_batch(args, rank, world, local_rank, dist)
        return run_ours(args, rank, world, local_rank, dist)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    raise SystemExit(main())
