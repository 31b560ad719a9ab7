"""``test.py --runtime cuda``: the reference's command-line generation run
(test.py:281-333, ``run_cpu``) on the B200 backend.

The reference's test.py parses the arguments, builds the prompt token ids
and then calls the runtime's generation loop; a maintainer adds ``"cuda"`` to
its ``--runtime`` choices (test.py:57) and routes it here::

    if args.runtime == "cuda":
        from harsh4b_b200.cli import run_test_py
        run_test_py(args, tokens, tokenizer, MODEL_PATH)
        return

The loop is the reference's: the prompt, then up to ``--max-new-tokens``
sampled tokens with its temperature / top-p / top-k / repetition-penalty
policy and ``--seed``, stopping at an end-of-turn id; the first
``--warmup-tokens`` decode steps are left out of the decode rate, and, as
there, a decode step's time is the forward pass alone (here including its
device synchronisation), not the sampling. The prompt goes through one
prefill pass and sampling runs on the device.
"""
from __future__ import annotations

import time

STOP_IDS = {151_643, 151_645}  # test.py:144-151 without a tokenizer


def stop_ids_of(tokenizer) -> set[int]:
    if tokenizer is None:
        return set(STOP_IDS)
    ids = {tokenizer.token_to_id(s) for s in ("<|endoftext|>", "<|im_end|>")}
    return {i for i in ids if i is not None}


def run_test_py(args, tokens, tokenizer, model_path, *, model=None, out=print) -> dict:
    """Generate from ``tokens`` as test.py's CPU runtime does; returns the
    generated ids and the timings it prints."""
    import torch

    from .runtime import CudaBackend, load_model

    out("[CUDA] Loading the LATTICE model on the B200 backend...", flush=True)
    started = time.perf_counter()
    if model is None:
        model = load_model(model_path, verbose=True)
    backend = CudaBackend(model=model, tokenizer=tokenizer, seed=args.seed, top_p=args.top_p, top_k=args.top_k,
                          repetition_penalty=args.repetition_penalty)
    out(f"[CUDA] Model ready in {time.perf_counter() - started:.1f}s on {backend.hardware}", flush=True)
    stop_ids = stop_ids_of(tokenizer)
    decoder = None
    if tokenizer is not None:
        from tokenizers.decoders import DecodeStream

        decoder = DecodeStream(skip_special_tokens=True)
    generated, decode_times = [], []
    started = time.perf_counter()
    logits, session = backend.prefill(list(tokens), args.max_new_tokens)
    torch.cuda.synchronize(model.device)
    token = backend.sample(logits, generated, args.temperature)
    prefill_seconds = time.perf_counter() - started
    out(f"[CUDA] First token ready in {prefill_seconds:.3f}s\n\n--- OUTPUT (streaming) ---", flush=True)
    for _ in range(args.max_new_tokens):
        if token in stop_ids:
            break
        generated.append(token)
        piece = decoder.step(tokenizer, token) if decoder else f"{token},"
        if piece:
            out(piece, end="", flush=True)
        if len(generated) >= args.max_new_tokens:
            break
        started = time.perf_counter()
        logits = backend.decode(token, session)
        torch.cuda.synchronize(model.device)
        decode_times.append(time.perf_counter() - started)
        token = backend.sample(logits, generated, args.temperature)
    measured = decode_times[min(args.warmup_tokens, len(decode_times)):]
    out("\n--------------")
    out(f"model: {getattr(model_path, 'name', model_path)}")
    out("runtime: cuda (B200 packed int4)")
    stop = "end-of-turn token" if token in stop_ids else f"{args.max_new_tokens}-token limit (output may be truncated)"
    out(f"stop: {stop}")
    out(f"prefill: {len(tokens)} tokens in {prefill_seconds:.3f}s ({len(tokens) / prefill_seconds:.2f} tok/s)")
    rate = len(measured) / sum(measured) if measured else None
    out(f"decode: {rate:.2f} tok/s" if rate else "decode: no non-EOS tokens were available to benchmark")
    return {"generated": generated, "prefill_seconds": prefill_seconds, "decode_tok_s": rate}
