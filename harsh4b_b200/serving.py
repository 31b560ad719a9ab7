"""Continuous batching for the chat server: concurrent requests share one
batched decode on the GPU.

The reference's server (web_ui.py:706-802) runs one request at a time: each
POST /api/chat takes a model lock and iterates ``runtime.stream()``. Here one
engine thread owns a :class:`harsh4b_b200.model.CudaBatchState` of ``slots``
sequences. Requests join a free slot between steps -- the prompt goes
through the one-pass prefill (h4b_prefill) straight into that slot's K/V --
and every step advances all active slots by one token with one batched
decode (h4b_decode_batch: tensor-core GEMMs over the batch, per-sequence
attention). A request leaves its slot at an end-of-turn id, at its token
limit or when its caller cancels; the slot is reused at once.

Per request the token policy is the reference stream()'s
(inference_runtime.py:90-122): the first token is sampled from the prefill
logits, then each decoded token is sampled with the runtime's policy (greedy
at temperature <= 0.01, else sample_numpy's top-k / top-p / repetition
penalty on the device), stopping at a stop id (not emitted) or after
``max_tokens`` tokens. Idle slots decode a dummy token at position 0, which
touches nothing of the other slots (every row of the batched step is
independent).

:class:`BatchedCudaBackend` exposes this through the runtime contract with a
thread-safe ``stream()`` (``concurrent = True``), so a server that drops its
model lock for such runtimes batches its concurrent requests.
"""
from __future__ import annotations

import queue
import threading
import time
from dataclasses import dataclass, field

import numpy as np

from .runtime import CudaBackend


@dataclass
class Request:
    prompt_ids: list
    max_tokens: int
    temperature: float
    stopped: object = None                     # callable -> bool (cancellation)
    events: queue.Queue = field(default_factory=queue.Queue)  # ("token", id) ... ("done", stats)
    generated: list = field(default_factory=list)
    slot: int = -1
    t_submit: float = 0.0
    prefill_s: float = 0.0
    t_decode0: float = 0.0
    decode_steps: int = 0


class ContinuousBatcher:
    """The engine: one thread, `slots` decode sessions advanced together."""

    def __init__(self, model, slots: int = 8, capacity: int = 2048, attn_splits: int = 16, sampler=None,
                 stop_ids=(), seed: int | None = None, top_p: float = 0.9, top_k: int = 50,
                 repetition_penalty: float = 1.15, attention: str = "tensor"):
        import torch

        from .model import CudaDecodeState

        self.torch, self.model = torch, model
        self.slots, self.capacity = int(slots), int(capacity)
        self.attention = attention  # the prompt and the batched-decode attention kernels
        self.batch = model.new_batch_state(self.slots, self.capacity, attn_splits, attention)
        self.slot_states = [CudaDecodeState(model, self.capacity, kv=(self.batch.k_cache[b], self.batch.v_cache[b]))
                            for b in range(self.slots)]
        self.sampler = sampler or CudaBackend(model=model, seed=seed, top_p=top_p, top_k=top_k,
                                              repetition_penalty=repetition_penalty).sample
        self.stop_ids = set(stop_ids)
        self.active: list[Request | None] = [None] * self.slots
        self.positions = np.zeros(self.slots, dtype=np.int32)
        self.tokens = np.zeros(self.slots, dtype=np.int32)
        self._positions_h = torch.zeros(self.slots, dtype=torch.int32).pin_memory()
        self._tokens_h = torch.zeros(self.slots, dtype=torch.int32).pin_memory()
        self._next_h = torch.zeros(self.slots, dtype=torch.int32).pin_memory()
        self.pending: queue.Queue = queue.Queue()
        self.steps = 0
        self._wake = threading.Event()
        self._stop = threading.Event()
        self._thread = None
        self.error = None

    # -- requests ----------------------------------------------------------
    def submit(self, prompt_ids, max_tokens: int, temperature: float = 0.0, stopped=None) -> Request:
        ids = [int(t) for t in prompt_ids]
        if not ids or max_tokens < 1 or len(ids) + max_tokens > self.capacity:
            raise ValueError("Prompt and output exceed the engine's context budget")
        if min(ids) < 0 or max(ids) >= self.model.vocab:
            raise ValueError("token ID outside the vocabulary")
        request = Request(ids, int(max_tokens), float(temperature), stopped, t_submit=time.perf_counter())
        self.pending.put(request)
        self._wake.set()
        return request

    # -- engine ------------------------------------------------------------
    def start(self) -> "ContinuousBatcher":
        self._thread = threading.Thread(target=self._loop, name="h4b-batcher", daemon=True)
        self._thread.start()
        return self

    def close(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join()
            self._thread = None
        for state in self.slot_states:
            state.close()

    def _loop(self) -> None:
        torch = self.torch
        torch.cuda.set_device(self.model.device)
        try:
            while not self._stop.is_set():
                self.admit()
                if any(r is not None for r in self.active):
                    self.step()
                elif self.pending.empty():
                    self._wake.wait(0.05)  # idle until a request arrives
                    self._wake.clear()
        except Exception as exc:  # surface to every waiting caller
            self.error = exc
            for request in self.active:
                if request is not None:
                    request.events.put(("error", str(exc)))
            while not self.pending.empty():
                self.pending.get().events.put(("error", str(exc)))

    def _cancelled(self, request: Request) -> bool:
        return bool(request.stopped and request.stopped())

    def _finish(self, request: Request) -> None:
        decode_s = time.perf_counter() - request.t_decode0 if request.decode_steps else 0.0
        request.events.put(("done", {"tokens": len(request.generated), "prefill_time": request.prefill_s,
                                     "decode_time": decode_s, "decode_steps": request.decode_steps,
                                     "slot": request.slot}))
        if request.slot >= 0:
            self.active[request.slot] = None
            self.positions[request.slot] = 0
            self.tokens[request.slot] = 0

    def _accept(self, request: Request, token: int) -> bool:
        """The reference stream()'s per-token rule; True while the request goes on."""
        if token in self.stop_ids:
            return False
        request.generated.append(token)
        request.events.put(("token", token))
        return len(request.generated) < request.max_tokens and not self._cancelled(request)

    def admit(self) -> None:
        """Prefill waiting requests into free slots."""
        while not self.pending.empty() and None in self.active:
            request = self.pending.get()
            if self._cancelled(request):
                self._finish(request)
                continue
            b = self.active.index(None)
            request.slot = b
            state = self.slot_states[b]
            state.reset()
            t0 = time.perf_counter()
            logits = self.model.prefill(request.prompt_ids, state, attention=self.attention)
            token = self.sampler(logits, request.generated, request.temperature)
            request.prefill_s = time.perf_counter() - t0
            request.t_decode0 = time.perf_counter()
            self.active[b] = request
            if not self._accept(request, int(token)):
                self._finish(request)
                continue
            self.positions[b] = len(request.prompt_ids)
            self.tokens[b] = int(token)

    def step(self) -> None:
        """One batched decode token for every active slot."""
        import ctypes

        from ._lib import check, lib

        torch, batch = self.torch, self.batch
        self._positions_h.copy_(torch.from_numpy(self.positions))
        self._tokens_h.copy_(torch.from_numpy(self.tokens))
        batch.positions.copy_(self._positions_h, non_blocking=True)
        batch.tokens.copy_(self._tokens_h, non_blocking=True)
        check(lib().h4b_decode_batch(ctypes.byref(self.model.desc), ctypes.byref(batch.desc),
                                     torch.cuda.current_stream(self.model.device).cuda_stream), "h4b_decode_batch")
        self._next_h.copy_(batch.next_tokens)  # synchronises (the pinned inputs are free again)
        greedy = self._next_h.numpy()
        self.steps += 1
        for b, request in enumerate(self.active):
            if request is None:
                continue
            request.decode_steps += 1
            self.positions[b] += 1
            if request.temperature <= 0.01:
                token = int(greedy[b])
            else:
                token = int(self.sampler(batch.logits[b], request.generated, request.temperature))
            if self._accept(request, token):
                self.tokens[b] = token
            else:
                self._finish(request)


class BatchedCudaBackend(CudaBackend):
    """The runtime contract on the continuous batcher: ``stream()`` may be
    called from several threads at once; each call is one request in the
    shared batch. Events follow the reference's stream contract:
    {"token": text, "done": False} per decoded piece, then
    {"done": True, "stats": {...}}."""

    concurrent = True

    def __init__(self, path=None, tokenizer=None, *, slots: int = 8, capacity: int = 2048, **options):
        super().__init__(path, tokenizer, **options)
        stop_ids = getattr(tokenizer, "stop_ids", ()) if tokenizer is not None else ()
        self.engine = ContinuousBatcher(self.model, slots=slots, capacity=capacity, sampler=self.sample,
                                        stop_ids=stop_ids).start()
        self.description += f", continuous batching over {slots} slots"

    def stream(self, prompt_ids, max_tokens, temperature, stopped=lambda: False):
        from tokenizers.decoders import DecodeStream

        request = self.engine.submit(prompt_ids, max_tokens, temperature, stopped)
        decoder = DecodeStream(skip_special_tokens=True)
        while True:
            kind, value = request.events.get()
            if kind == "token":
                text = decoder.step(self.tokenizer.backend, value)
                if text:
                    yield {"token": text, "done": False}
            elif kind == "error":
                raise RuntimeError(value)
            else:
                decode_s, steps = value["decode_time"], value["decode_steps"]
                yield {"done": True, "stats": {
                    "tokens": value["tokens"], "time": round(value["prefill_time"] + decode_s, 3),
                    "prefill_time": round(value["prefill_time"], 3), "decode_time": round(decode_s, 3),
                    "decode_steps": steps, "tok_per_sec": round(steps / decode_s, 2) if decode_s else 0.0,
                    "vram_gb": round(self.memory_gib(), 2), "runtime": self.device}}
                return

    def close(self) -> None:
        self.engine.close()
