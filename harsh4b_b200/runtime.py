"""Runtime entry for the B200 backend: the ``Runtime`` contract of the
reference's chat server (inference_runtime.py:71-122) and a ``CudaRuntime``
that serves it from :class:`harsh4b_b200.model.CudaQwen`.

The reference picks its backend in ``create_runtime`` (inference_runtime.py:
349-356); ``select_runtime`` already answers "cuda" when torch sees a GPU
(:16-32). A maintainer routes "cuda" to :class:`CudaRuntime` (see
INTEGRATION.md). Methods keep the reference's names and meaning:

* ``prefill(ids, max_tokens) -> (logits, session)``: a fresh decode state
  sized for the prompt plus the output, the prompt fed in one pass through
  the batched GEMMs (the reference's CPU runtime loops over the tokens,
  :124-128; the resulting state and logits are the same);
* ``decode(token, session) -> logits``;
* ``sample(logits, generated, temperature) -> int``: sample_numpy's policy
  (:144-163; top-p 0.9, top-k 50, repetition penalty 1.15) on the device,
  with the draw taken from this runtime's numpy generator;
* ``memory_gib()``, ``status()``, ``stream(...)`` and the attributes
  ``device``, ``hardware``, ``description``, ``tokenizer``, ``torch``.
"""
from __future__ import annotations

import time
from pathlib import Path

import numpy as np

MODEL_ID = "Qwen/Qwen3-4B"


class Runtime:
    """Backend-independent part of a runtime (inference_runtime.py:71-122)."""

    max_context = 2048

    def status(self) -> dict:
        return dict(model=MODEL_ID, device=self.device, runtime=self.device, hardware=self.hardware,
                    quant=self.description, ready=True, vram_gb=round(self.memory_gib(), 2),
                    max_context=self.max_context)

    def memory_gib(self) -> float:
        return 0.0

    def stream(self, prompt_ids, max_tokens, temperature, stopped=lambda: False):
        """One fresh session per request; no forward pass after the last token.
        Yields {"token": text, "done": False} per decoded piece, then
        {"done": True, "stats": {...}} (the reference's stream contract)."""
        from tokenizers.decoders import DecodeStream

        if not prompt_ids or len(prompt_ids) + max_tokens > self.max_context:
            raise ValueError("Prompt and output exceed the runtime context budget")
        generated: list[int] = []
        decoder = DecodeStream(skip_special_tokens=True)
        prefill_seconds = decode_seconds = 0.0
        decode_steps = 0
        if not stopped():
            t0 = time.perf_counter()
            logits, session = self.prefill(prompt_ids, max_tokens)
            token = self.sample(logits, generated, temperature)
            prefill_seconds = time.perf_counter() - t0
            while not stopped() and token not in self.tokenizer.stop_ids:
                generated.append(token)
                text = decoder.step(self.tokenizer.backend, token)
                if text:
                    yield {"token": text, "done": False}
                if len(generated) >= max_tokens or stopped():
                    break
                t0 = time.perf_counter()
                logits = self.decode(token, session)
                token = self.sample(logits, generated, temperature)
                decode_seconds += time.perf_counter() - t0
                decode_steps += 1
        yield {"done": True, "stats": {
            "tokens": len(generated), "time": round(prefill_seconds + decode_seconds, 3),
            "prefill_time": round(prefill_seconds, 3), "decode_time": round(decode_seconds, 3),
            "decode_steps": decode_steps,
            "tok_per_sec": round(decode_steps / decode_seconds, 2) if decode_seconds else 0.0,
            "vram_gb": round(self.memory_gib(), 2), "runtime": self.device,
        }}


class CudaRuntime(Runtime):
    """The reference's runtime contract on the B200 decode path."""

    device = "cuda"

    def __init__(self, path=None, tokenizer=None, *, model=None, kv_dtype: str = "float16", mode: str = "persistent",
                 seed: int | None = None, top_p: float = 0.9, top_k: int = 50, repetition_penalty: float = 1.15,
                 **_):
        import torch

        from .model import CudaQwen

        if not torch.cuda.is_available():
            raise RuntimeError("CUDA is unavailable; harsh4b_b200 has no CPU fallback")
        self.torch, self.tokenizer = torch, tokenizer
        if model is None:
            if path is None:
                raise ValueError("CudaRuntime needs a LiteSpark cache directory or a CudaQwen model")
            model = CudaQwen.from_cache(Path(path), kv_dtype=kv_dtype, mode=mode)
        self.model = model
        self.hardware = torch.cuda.get_device_name(model.device)
        self.description = f"CUDA · B200 packed int4 ({getattr(model, 'mode', mode)} decode, {model.kv_dtype} KV)"
        self.top_p, self.top_k, self.repetition_penalty = float(top_p), int(top_k), float(repetition_penalty)
        self.generator = np.random.default_rng(seed)
        self._work = torch.empty(model.vocab, dtype=torch.float32, device=model.device)
        self._token = torch.empty(1, dtype=torch.int32, device=model.device)
        self._seen = torch.empty(self.max_context, dtype=torch.int32, device=model.device)
        from ._lib import lib

        nbytes = int(lib().h4b_sample_scratch_bytes(model.vocab, self.top_k))
        if nbytes < 0:
            raise ValueError(f"top_k {self.top_k} is not supported by the device sampler")
        self._scratch = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=model.device)

    def prefill(self, ids, max_tokens):
        """A fresh session with the prompt fed in one CudaQwen.prefill pass (the
        reference's CPU runtime feeds it token by token, :124-128; the state
        ends the same, with the prompt's attention split count fixed per
        session)."""
        state = self.model.new_state(len(ids) + max_tokens)
        logits = self.model.prefill([int(t) for t in ids], state)
        return logits, state

    def decode(self, token, session):
        return self.model.forward_token(int(token), session)

    def sample(self, logits, generated, temperature):
        """sample_numpy's policy on the device; the logits are not modified."""
        from . import ops

        torch = self.torch
        values = logits.reshape(-1)
        if values.dtype != torch.float32 or not values.is_cuda:
            values = torch.as_tensor(values, dtype=torch.float32, device=self.model.device)
        with torch.cuda.stream(torch.cuda.current_stream(self.model.device)):
            self._work.copy_(values)
            seen = sorted(set(int(t) for t in generated)) if self.repetition_penalty != 1.0 else []
            gen = None
            if seen:
                if len(seen) > self._seen.numel():
                    self._seen = torch.empty(len(seen), dtype=torch.int32, device=self.model.device)
                gen = self._seen[:len(seen)]
                gen.copy_(torch.tensor(seen, dtype=torch.int32))
            uniform = float(self.generator.random()) if temperature > 0.01 else 0.0
            ops.sample(self._work, gen, uniform, temperature=temperature, top_k=self.top_k, top_p=self.top_p,
                       repetition_penalty=self.repetition_penalty, out=self._token, scratch=self._scratch)
            return int(self._token.item())

    def memory_gib(self) -> float:
        return self.torch.cuda.memory_allocated(self.model.device) / 2**30


def select_runtime(requested: str = "auto") -> str:
    """inference_runtime.select_runtime restricted to this backend: "cuda"
    when a GPU is visible (raises otherwise -- there is no CPU path here)."""
    if requested not in ("auto", "cuda"):
        raise ValueError(f"harsh4b_b200 serves only the cuda runtime, not {requested!r}")
    import torch

    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is unavailable; harsh4b_b200 has no CPU fallback")
    return "cuda"


def create_runtime(name: str = "auto", model_path=None, tokenizer=None, **options) -> CudaRuntime:
    """create_runtime (inference_runtime.py:349-356) for the cuda runtime:
    `model_path` is a LiteSpark cache directory (build_litespark_cpu layout),
    `tokenizer` an object with `.stop_ids` and `.backend` (the reference's
    ChatTokenizer)."""
    select_runtime(name)
    return CudaRuntime(model_path, tokenizer, **options)
