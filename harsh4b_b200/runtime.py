"""The B200 backend of the reference chat server's runtime contract.

The reference defines ``Runtime`` (inference_runtime.py:71-122: ``status``,
``stream`` and the context budget) and one subclass per backend that
supplies ``prefill``, ``decode``, ``sample``, ``memory_gib`` and the
attributes ``device``, ``hardware``, ``description``, ``tokenizer`` (and
``torch``, read by benchmarks/bench_energy.py:269-273). This module ships
only that backend half, :class:`CudaBackend`; the reference side composes it
with its own base class::

    from harsh4b_b200.runtime import CudaBackend

    class CudaRuntime(CudaBackend, Runtime):
        pass

and ``create_runtime`` (inference_runtime.py:349-356) picks ``CudaRuntime``
for ``"cuda"``, as ``select_runtime`` (:16-32) already answers ``"cuda"``
when torch sees a GPU. ``stream()`` is the reference's, unchanged.

Methods keep the reference's names and meaning:

* ``prefill(ids, max_tokens) -> (logits, session)``: a fresh decode state
  sized for the prompt plus the output, the prompt fed in one pass through
  the batched GEMMs (the reference's CPU runtime loops over the tokens,
  inference_runtime.py:177-181; the resulting state and logits are the same);
* ``decode(token, session) -> logits``;
* ``sample(logits, generated, temperature) -> int``: sample_numpy's policy
  (inference_runtime.py:144-163; top-p 0.9, top-k 50, repetition penalty
  1.15) on the device, the draw taken from this runtime's numpy generator;
* ``memory_gib()``.

``create_runtime(model_path, ...)`` hands the backend the LATTICE checkpoint
path (``checkpoint_path``, inference_runtime.py:35-43); a directory holding a
packed cache (``manifest.json``) with its norms is accepted as well.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np


def load_model(path, *, kv_dtype: str = "float16", mode: str = "persistent", cache_dir=None, verbose: bool = False):
    """A :class:`CudaQwen` from a LATTICE checkpoint file (converted on the
    GPU into the shared packed cache) or from a self-contained cache
    directory."""
    from .model import CudaQwen

    path = Path(path)
    if path.is_dir():
        return CudaQwen.from_cache(path, kv_dtype=kv_dtype, mode=mode)
    from .lattice import build_b200_model

    return build_b200_model(path, cache_dir=cache_dir, verbose=verbose, kv_dtype=kv_dtype, mode=mode)


class CudaBackend:
    """prefill / decode / sample / memory_gib of the reference's runtime
    contract on the B200 decode path (combine with the reference's
    ``Runtime`` for ``status`` and ``stream``).

    ``model`` and ``sampler`` let a caller hand in its own model object
    (``new_state`` / ``prefill`` / ``forward_token``) or sampling policy
    ``sampler(logits, generated, temperature) -> int``; without them the
    backend builds the CUDA model from ``path`` and samples on the device,
    and raises when no GPU is visible (there is no CPU fallback)."""

    device = "cuda"

    def __init__(self, path=None, tokenizer=None, *, model=None, sampler=None, kv_dtype: str = "float16",
                 mode: str = "persistent", seed: int | None = None, top_p: float = 0.9, top_k: int = 50,
                 repetition_penalty: float = 1.15, cache_dir=None, verbose: bool = False, **_):
        import torch

        if model is None:
            if not torch.cuda.is_available():
                raise RuntimeError("CUDA is unavailable; harsh4b_b200 has no CPU fallback")
            if path is None:
                raise ValueError("CudaBackend needs a LATTICE checkpoint, a packed cache directory or a model")
            model = load_model(path, kv_dtype=kv_dtype, mode=mode, cache_dir=cache_dir, verbose=verbose)
        self.torch, self.tokenizer, self.model = torch, tokenizer, model
        on_gpu = torch.device(getattr(model, "device", "cpu")).type == "cuda"
        self.hardware = torch.cuda.get_device_name(model.device) if on_gpu else str(getattr(model, "device", "cpu"))
        self.description = (f"CUDA · B200 packed int4 ({getattr(model, 'mode', mode)} decode, "
                            f"{getattr(model, 'kv_dtype', kv_dtype)} KV)")
        self.top_p, self.top_k, self.repetition_penalty = float(top_p), int(top_k), float(repetition_penalty)
        self.generator = np.random.default_rng(seed)
        self._sampler = sampler
        if sampler is None:
            from ._lib import lib

            self._work = torch.empty(model.vocab, dtype=torch.float32, device=model.device)
            self._token = torch.empty(1, dtype=torch.int32, device=model.device)
            self._seen = torch.empty(2048, dtype=torch.int32, device=model.device)
            nbytes = int(lib().h4b_sample_scratch_bytes(model.vocab, self.top_k))
            if nbytes < 0:
                raise ValueError(f"top_k {self.top_k} is not supported by the device sampler")
            self._scratch = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=model.device)

    def prefill(self, ids, max_tokens):
        """A fresh session with the prompt fed in one CudaQwen.prefill pass
        (the state ends as after feeding the prompt token by token, with the
        prompt's attention split count fixed per session)."""
        state = self.model.new_state(len(ids) + max_tokens)
        logits = self.model.prefill([int(t) for t in ids], state)
        return logits, state

    def decode(self, token, session):
        return self.model.forward_token(int(token), session)

    def sample(self, logits, generated, temperature):
        """sample_numpy's policy on the device; the logits are not modified."""
        if self._sampler is not None:
            return int(self._sampler(logits, generated, temperature))
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
        if self.torch.device(getattr(self.model, "device", "cpu")).type != "cuda":
            return 0.0
        return self.torch.cuda.memory_allocated(self.model.device) / 2**30
