"""Device-resident Qwen3 decode model: the ``cuda`` counterpart of the
reference's ``cpu_lightspark.LiteSparkQwen`` (cpu_lightspark.py:312-553).

``CudaQwen`` keeps the reference object's surface -- ``new_state(capacity)``,
``forward_token(token_id, state)`` returning next-token logits,
``profile_forward_token`` returning ``(logits, timings, counts, total)`` with
the same category names -- and runs each token as one CUDA graph replay of
the C-ABI decode step. Logits are returned as a CUDA tensor view of the
state's buffer (overwritten by the next call, like ``state.logits`` in the
reference).
"""
from __future__ import annotations

import ctypes
import time

import numpy as np
import torch

from ._lib import (BatchStateDesc, ModelDesc, PrefillScratchDesc, StateDesc, check, device_status, lib,
                   STATUS_WAIT_TIMEOUT)
from .cache import Checkpoint, norm_names, read_cache

KV_DTYPES = {"float32": (0, torch.float32), "float16": (1, torch.float16)}
MODES = ("persistent", "chain")
# prefill attention kernels (h4b_prefill_scratch.attn_kernel)
PREFILL_ATTENTION = {"exact": 0, "tensor": 1}
# batched-decode attention kernels (h4b_batch_state.attn_kernel)
BATCH_ATTENTION = {"exact": 0, "tensor": 1}
PERSISTENT_ATTN_CHUNK = 32  # tokens per attention split in the persistent step (persistent.cu)
SWIGLU_BLOCK = 4  # rows per gate/up interleave block (matches the kernel)

PROFILE_CATEGORIES = (
    "ternary/int4 GEMV",
    "activation quantization",
    "embedding / LM head",
    "attention",
    "RMSNorm",
    "packing/depacking",
)


def rope_tables(config) -> tuple[np.ndarray, np.ndarray]:
    """fp32 cos/sin tables [max_position, head_dim/2], computed the way the
    reference computes them (cpu_lightspark.py:329-336)."""
    head_dim = int(config["head_dim"])
    exponent = np.arange(0, head_dim, 2, dtype=np.float32) / np.float32(head_dim)
    inv_freq = np.float32(1.0) / np.float32(config["rope_theta"]) ** exponent
    positions = np.arange(int(config["max_position_embeddings"]), dtype=np.float32)
    angles = positions[:, None] * inv_freq[None, :]
    return np.cos(angles).astype(np.float32), np.sin(angles).astype(np.float32)


def interleave_gate_up(rows: np.ndarray, intermediate: int) -> np.ndarray:
    """[gate; up] rows -> blocks of SWIGLU_BLOCK gate rows then the matching up rows."""
    gate, up = rows[:intermediate], rows[intermediate:]
    tail = gate.shape[1:]
    blocks = intermediate // SWIGLU_BLOCK
    return np.stack([gate.reshape(blocks, SWIGLU_BLOCK, *tail), up.reshape(blocks, SWIGLU_BLOCK, *tail)],
                    axis=1).reshape(2 * intermediate, *tail)


def _as_layer_tuple(layer):
    """Accept a reference-style QwenLayer-like object or a Checkpoint.layer tuple."""
    if isinstance(layer, tuple):
        return layer
    return ((layer.qkv.weights, layer.qkv.scales), (layer.o.weights, layer.o.scales),
            (layer.gate_up.weights, layer.gate_up.scales), (layer.down.weights, layer.down.scales),
            layer.input_norm, layer.post_norm, layer.q_norm, layer.k_norm)


class CudaDecodeState:
    """Caller-owned KV cache and scratch on the device (QwenDecodeState,
    cpu_lightspark.py:275-309). One CUDA graph per state replays a token."""

    def __init__(self, model: "CudaQwen", capacity: int, attn_splits: int | None = None, kv=None):
        if capacity < 1:
            raise ValueError("decode capacity must be positive")
        if capacity > model.max_pos:
            raise ValueError("decode capacity exceeds max_position_embeddings")
        self.model = model
        self.capacity = int(capacity)
        self.position = 0
        dev = model.device
        code, kv_torch = KV_DTYPES[model.kv_dtype]
        shape = (model.n_layers, model.kv_heads, self.capacity, model.head_dim)
        if kv is None:
            self.k_cache = torch.zeros(shape, dtype=kv_torch, device=dev)
            self.v_cache = torch.zeros(shape, dtype=kv_torch, device=dev)
        else:
            # K/V held elsewhere (e.g. one sequence slot of a batch state)
            self.k_cache, self.v_cache = kv
            for t in kv:
                if tuple(t.shape) != shape or t.dtype != kv_torch or t.device != dev or not t.is_contiguous():
                    raise ValueError("external K/V buffers must be contiguous [layers][kv_heads][capacity][head_dim] "
                                     "in the model's KV dtype on its device")
        self.splits = int(attn_splits or model.attn_splits)
        partial_splits = self.splits
        i32 = dict(dtype=torch.int32, device=dev)
        f32 = dict(dtype=torch.float32, device=dev)
        self.position_dev = torch.zeros(1, **i32)
        self.token_dev = torch.zeros(1, **i32)
        self.next_token_dev = torch.zeros(1, **i32)
        self.x = torch.zeros(model.hidden, **f32)
        self.qkv = torch.zeros(model.q_size + 2 * model.kv_size, **f32)
        self.attended = torch.zeros(model.q_size, **f32)
        self.act = torch.zeros(model.intermediate, **f32)
        self.logits = torch.zeros(model.vocab, **f32)
        self.absmax = torch.zeros(2 * model.n_layers, **f32)
        self.argmax_key = torch.zeros(1, dtype=torch.int64, device=dev)
        self.partials = torch.zeros(model.kv_heads * partial_splits * model.groups * (model.head_dim + 4), **f32)
        self.counters = torch.zeros(model.kv_heads, **i32)
        words = lib().h4b_persistent_exchange_words(ctypes.byref(model.desc))
        if words < 0:
            check(int(words), "h4b_persistent_exchange_words")
        self.exchange = torch.zeros(int(words), dtype=torch.int64, device=dev)
        self.desc = StateDesc(self.capacity, code, self.splits, *[t.data_ptr() for t in (
            self.k_cache, self.v_cache, self.position_dev, self.token_dev, self.next_token_dev, self.x, self.qkv,
            self.attended, self.act, self.logits, self.absmax, self.argmax_key, self.partials, self.counters,
            self.exchange)])
        check(lib().h4b_validate(ctypes.byref(model.desc), ctypes.byref(self.desc)), "h4b_validate")
        self.stream = torch.cuda.Stream(device=dev)
        self._token_host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self._next_host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self._copied = torch.cuda.Event()
        self._graph = None

    # -- graph management -------------------------------------------------
    def _ensure_graph(self) -> None:
        if self._graph is None:
            handle = ctypes.c_void_p()
            create = (lib().h4b_graph_create_persistent if self.model.mode == "persistent"
                      else lib().h4b_graph_create)
            with torch.cuda.device(self.model.device):
                check(create(ctypes.byref(self.model.desc), ctypes.byref(self.desc), self.stream.cuda_stream,
                             ctypes.byref(handle)), "h4b_graph_create")
            self._graph = handle

    def close(self) -> None:
        if self._graph is not None:
            lib().h4b_graph_destroy(self._graph)
            self._graph = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- one step ---------------------------------------------------------
    def set_token(self, token_id: int) -> None:
        """Queue the host -> device copy of the next input token (pinned)."""
        self._copied.synchronize()  # the pinned slot may still feed an earlier copy
        self._token_host[0] = int(token_id)
        with torch.cuda.stream(self.stream):
            self.token_dev.copy_(self._token_host, non_blocking=True)
            self._copied.record(self.stream)

    def replay(self, steps: int = 1) -> None:
        """Run `steps` decode tokens back to back; after the first, each step
        consumes the previous step's greedy token (device-side feedback)."""
        self._ensure_graph()
        for _ in range(steps):
            check(lib().h4b_graph_launch(self._graph, self.stream.cuda_stream), "h4b_graph_launch")
        self.position += steps

    def greedy_token(self, token_id: int) -> int:
        """One decode step fed `token_id` from the host, returning its greedy
        token to the host (h4b_graph_token: one call for the pinned copy in,
        the graph launch, the copy out and the wait)."""
        self._ensure_graph()
        self._copied.synchronize()  # a set_token copy may still read the pinned slot
        self._token_host[0] = int(token_id)
        check(lib().h4b_graph_token(self._graph, self._token_host.data_ptr(), self.token_dev.data_ptr(),
                                    self.next_token_dev.data_ptr(), self._next_host.data_ptr(),
                                    self.stream.cuda_stream), "h4b_graph_token")
        self.position += 1
        return int(self._next_host[0])

    def next_token_host(self) -> int:
        """Device -> host read of the greedy token of the last step."""
        with torch.cuda.stream(self.stream):
            self._next_host.copy_(self.next_token_dev, non_blocking=True)
        self.stream.synchronize()
        return int(self._next_host[0])

    def reset(self) -> None:
        """Start a new sequence in the same buffers."""
        self.stream.synchronize()
        self.position = 0
        self.position_dev.zero_()
        self.exchange.zero_()  # also recovers the persistent step after a failed token
        torch.cuda.synchronize(self.model.device)


class CudaBatchState:
    """B independent decode sessions advanced together (one token each per
    step). KV cache [B][L][kv_heads][capacity][head_dim]; every sequence keeps
    its own position. Scratch sized for the batch; nothing allocates per step.

    attention="exact": the fp32 split kernel with `attn_splits` splits, each
    row bit-identical to a decode step. attention="tensor" (the default; fp16
    cache, head_dim 128, 4 q heads per kv head, otherwise as "exact"): tcgen05
    attention with split fp16 operands over whole 128-key tiles (one wave of
    CTAs for small batches, about two per SM otherwise, at most `attn_splits`
    splits), within the 1e-3 relative
    tolerance of the fp32 path."""

    def __init__(self, model: "CudaQwen", batch: int, capacity: int, attn_splits: int = 16,
                 attention: str = "tensor"):
        if batch < 1 or capacity < 1:
            raise ValueError("batch and capacity must be positive")
        if attention not in BATCH_ATTENTION:
            raise ValueError(f"attention must be one of {sorted(BATCH_ATTENTION)}")
        if capacity > model.max_pos:
            raise ValueError(f"capacity {capacity} exceeds the model's {model.max_pos} positions")
        self.model, self.batch, self.capacity, self.splits = model, batch, capacity, int(attn_splits)
        dev = model.device
        code, kv_torch = KV_DTYPES[model.kv_dtype]
        shape = (batch, model.n_layers, model.kv_heads, capacity, model.head_dim)
        self.k_cache = torch.zeros(shape, dtype=kv_torch, device=dev)
        self.v_cache = torch.zeros(shape, dtype=kv_torch, device=dev)
        i32 = dict(dtype=torch.int32, device=dev)
        f32 = dict(dtype=torch.float32, device=dev)
        H, I, Q, KV = model.hidden, model.intermediate, model.q_size, model.kv_size
        self.positions = torch.zeros(batch, **i32)
        self.tokens = torch.zeros(batch, **i32)
        self.next_tokens = torch.zeros(batch, **i32)
        self.x = torch.zeros(batch, H, **f32)
        self.x8 = torch.zeros(batch, max(H, Q, I), dtype=torch.int8, device=dev)
        self.act_scale = torch.zeros(batch, **f32)
        self.act_sum = torch.zeros(batch, **i32)
        self.qkv = torch.zeros(batch, Q + 2 * KV, **f32)
        self.attended = torch.zeros(batch, Q, **f32)
        self.proj = torch.zeros(batch, H, **f32)
        self.gate_up = torch.zeros(batch, 2 * I, **f32)
        self.act = torch.zeros(batch, I, **f32)
        self.logits = torch.zeros(batch, model.vocab, **f32)
        self.partials = torch.zeros(batch * model.kv_heads * self.splits * model.groups * (model.head_dim + 4), **f32)
        self.counters = torch.zeros(batch * model.kv_heads, **i32)
        # int32 sums of the split-K / stream-K GEMMs (every body projection),
        # zero between GEMMs
        acc_width = max(Q + 2 * KV, H, 2 * I)
        self.gemm_acc = torch.zeros(batch * acc_width, **i32)
        self.desc = BatchStateDesc(batch, capacity, code, self.splits, *[t.data_ptr() for t in (
            self.k_cache, self.v_cache, self.positions, self.tokens, self.next_tokens, self.x, self.x8,
            self.act_scale, self.act_sum, self.qkv, self.attended, self.proj, self.gate_up, self.act, self.logits,
            self.partials, self.counters, self.gemm_acc)])
        self.desc.attn_kernel = BATCH_ATTENTION[attention]
        self.desc.gemm_acc_width = acc_width
        check(lib().h4b_validate_batch(ctypes.byref(model.desc), ctypes.byref(self.desc)), "h4b_validate_batch")
        self.position = np.zeros(batch, dtype=np.int64)  # host copy of every sequence's position
        self._steps = 0
        self._graph = None

    def step(self) -> None:
        """One h4b_decode_batch step on the current stream. The first runs
        eagerly (it does the once-per-device kernel set-up); later ones replay
        a CUDA graph of the step captured on the second call: every input the
        step reads (tokens, positions, caches, scratch) is a device buffer of
        this state, so the one capture serves every later step."""
        model = self.model
        if self._steps == 0:
            check(lib().h4b_decode_batch(ctypes.byref(model.desc), ctypes.byref(self.desc),
                                         torch.cuda.current_stream(model.device).cuda_stream), "h4b_decode_batch")
        else:
            if self._graph is None:
                graph, stream = torch.cuda.CUDAGraph(), torch.cuda.Stream(model.device)
                stream.wait_stream(torch.cuda.current_stream(model.device))
                with torch.cuda.graph(graph, stream=stream):
                    check(lib().h4b_decode_batch(ctypes.byref(model.desc), ctypes.byref(self.desc),
                                                 stream.cuda_stream), "h4b_decode_batch")
                self._graph = graph
            self._graph.replay()
        self._steps += 1


class PrefillScratch:
    """Device buffers for h4b_prefill: up to `max_tokens` prompt rows per call,
    attention over `attn_queries` queries per launch with `splits` splits."""

    def __init__(self, model: "CudaQwen", max_tokens: int, splits: int, attn_queries: int = 512):
        dev = model.device
        i32 = dict(dtype=torch.int32, device=dev)
        f32 = dict(dtype=torch.float32, device=dev)
        H, I, Q, KV = model.hidden, model.intermediate, model.q_size, model.kv_size
        self.max_tokens, self.splits = int(max_tokens), int(splits)
        self.attn_queries = max(1, min(int(attn_queries), self.max_tokens))
        M = self.max_tokens
        self.x = torch.zeros(M, H, **f32)
        self.x8 = torch.zeros(M, max(H, Q, I), dtype=torch.int8, device=dev)
        self.act_scale = torch.zeros(M, **f32)
        self.act_sum = torch.zeros(M, **i32)
        self.qkv = torch.zeros(M, Q + 2 * KV, **f32)
        self.attended = torch.zeros(M, Q, **f32)
        self.gate_up = torch.zeros(M, 2 * I, **f32)
        self.act = torch.zeros(M, I, **f32)
        self.proj = torch.zeros(M, H, **f32)
        self.tokens = torch.zeros(M, **i32)
        self.positions = torch.zeros(M, **i32)
        if not 1 <= self.splits <= 64:
            raise ValueError("prefill attention splits must be in 1..64")
        parts = self.attn_queries * model.kv_heads * self.splits if self.splits > 1 else 1
        self.partials = torch.zeros(parts * model.groups * (model.head_dim + 4), **f32)
        self.counters = torch.zeros(max(1, self.attn_queries * model.kv_heads if self.splits > 1 else 1), **i32)
        self.desc = PrefillScratchDesc(M, self.attn_queries, self.splits, *[t.data_ptr() for t in (
            self.x, self.x8, self.act_scale, self.act_sum, self.qkv, self.attended, self.gate_up, self.act,
            self.proj, self.tokens, self.positions, self.partials, self.counters)])


class CudaQwen:
    """Qwen3 decode on one B200 from the packed int4 cache layout."""

    def __init__(self, config, layers, embedding, embedding_scales, final_norm, *, kv_dtype: str = "float16",
                 device=None, attn_splits: int = 16, mode: str = "persistent"):
        if kv_dtype not in KV_DTYPES:
            raise ValueError(f"kv_dtype must be one of {sorted(KV_DTYPES)}")
        if mode not in MODES:
            raise ValueError(f"mode must be one of {MODES}")
        lib()  # raises without a usable device or library
        self.mode = mode
        self._prefill_scratch = None
        self.config = dict(config)
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.kv_dtype = kv_dtype
        self.attn_splits = attn_splits
        c = self.config
        self.n_layers = int(c["num_hidden_layers"])
        self.hidden = int(c["hidden_size"])
        self.intermediate = int(c["intermediate_size"])
        self.heads = int(c["num_attention_heads"])
        self.kv_heads = int(c["num_key_value_heads"])
        self.head_dim = int(c["head_dim"])
        self.vocab = int(c["vocab_size"])
        self.max_pos = int(c["max_position_embeddings"])
        self.eps = float(c["rms_norm_eps"])
        self.groups = self.heads // self.kv_heads
        self.q_size = self.heads * self.head_dim
        self.kv_size = self.kv_heads * self.head_dim
        sms = ctypes.c_int(0)
        with torch.cuda.device(self.device):
            check(lib().h4b_device_info(ctypes.byref(sms), None, None), "h4b_device_info")
        self.sm_count = sms.value
        self.max_persistent_splits = max(1, min(64, self.sm_count // self.kv_heads))
        layers = [_as_layer_tuple(layer) for layer in layers]
        if len(layers) != self.n_layers:
            raise ValueError("layer count does not match the config")
        H, I, Q, KV = self.hidden, self.intermediate, self.q_size, self.kv_size
        qkv_rows = Q + 2 * KV

        def upload(parts, shape, dtype):
            buffer = torch.empty(shape, dtype=dtype, device=self.device)
            for index, part in enumerate(parts):
                buffer[index].copy_(torch.from_numpy(np.ascontiguousarray(part)))
            return buffer

        def pick(i):
            return [layer[i] for layer in layers]

        self.w_qkv = upload([p[0] for p in pick(0)], (self.n_layers, qkv_rows, H // 2), torch.uint8)
        self.s_qkv = upload([p[1] for p in pick(0)], (self.n_layers, qkv_rows), torch.float32)
        self.w_o = upload([p[0] for p in pick(1)], (self.n_layers, H, Q // 2), torch.uint8)
        self.s_o = upload([p[1] for p in pick(1)], (self.n_layers, H), torch.float32)
        self.w_gate_up = upload([interleave_gate_up(np.asarray(p[0]), I) for p in pick(2)],
                                (self.n_layers, 2 * I, H // 2), torch.uint8)
        self.s_gate_up = upload([interleave_gate_up(np.asarray(p[1]), I) for p in pick(2)],
                                (self.n_layers, 2 * I), torch.float32)
        self.w_down = upload([p[0] for p in pick(3)], (self.n_layers, H, I // 2), torch.uint8)
        self.s_down = upload([p[1] for p in pick(3)], (self.n_layers, H), torch.float32)
        self.norm_in = upload(pick(4), (self.n_layers, H), torch.float32)
        self.norm_post = upload(pick(5), (self.n_layers, H), torch.float32)
        self.norm_q = upload(pick(6), (self.n_layers, self.head_dim), torch.float32)
        self.norm_k = upload(pick(7), (self.n_layers, self.head_dim), torch.float32)
        self.embedding = torch.from_numpy(np.ascontiguousarray(embedding)).to(self.device)
        self.embedding_scales = torch.from_numpy(np.ascontiguousarray(embedding_scales, dtype=np.float32)).to(self.device)
        self.final_norm = torch.from_numpy(np.ascontiguousarray(final_norm, dtype=np.float32)).to(self.device)
        cos, sin = rope_tables(self.config)
        self.rope_cos = torch.from_numpy(cos).to(self.device)
        self.rope_sin = torch.from_numpy(sin).to(self.device)
        if self.embedding.shape != (self.vocab, H // 2):
            raise ValueError("embedding shape does not match the config")
        self.desc = ModelDesc(self.n_layers, H, I, self.heads, self.kv_heads, self.head_dim, self.vocab,
                              self.max_pos, self.eps, *[t.data_ptr() for t in (
                                  self.w_qkv, self.s_qkv, self.w_o, self.s_o, self.w_gate_up, self.s_gate_up,
                                  self.w_down, self.s_down, self.embedding, self.embedding_scales, self.norm_in,
                                  self.norm_post, self.norm_q, self.norm_k, self.final_norm, self.rope_cos,
                                  self.rope_sin)])
        torch.cuda.synchronize(self.device)

    @classmethod
    def from_checkpoint(cls, checkpoint: Checkpoint, **kwargs) -> "CudaQwen":
        checkpoint.validate()
        missing = [n for n in norm_names(checkpoint.config) if n not in checkpoint.norms]
        if missing:
            raise ValueError(f"no norm vectors for {missing[0]} (and {len(missing) - 1} more): a cache built by the "
                             "reference keeps them in the LATTICE checkpoint -- build the model with "
                             "harsh4b_b200.lattice.build_b200_model(checkpoint) or fill Checkpoint.norms")
        layers = [checkpoint.layer(i) for i in range(int(checkpoint.config["num_hidden_layers"]))]
        return cls(checkpoint.config, layers, checkpoint.embedding, checkpoint.embedding_scales,
                   checkpoint.norms["model.norm.weight"], **kwargs)

    @classmethod
    def from_cache(cls, directory, config: dict | None = None, **kwargs) -> "CudaQwen":
        """Load the reference's packed cache directory (cpu_lightspark.py:571-676)."""
        return cls.from_checkpoint(read_cache(directory, config), **kwargs)

    @property
    def weight_bytes(self) -> int:
        """Bytes of packed weights + row scales one token streams (body + LM head)."""
        tensors = (self.w_qkv, self.s_qkv, self.w_o, self.s_o, self.w_gate_up, self.s_gate_up, self.w_down,
                   self.s_down, self.embedding, self.embedding_scales)
        return sum(t.numel() * t.element_size() for t in tensors)

    def new_state(self, capacity: int, attn_splits: int | None = None) -> CudaDecodeState:
        return CudaDecodeState(self, capacity, attn_splits)

    def attention_split_rule(self, state: CudaDecodeState | None = None):
        """How many context splits the attention of a token with context `ctx`
        uses: fixed per state in the kernel chain, chosen per token in the
        persistent step. Returns a function ctx -> splits (the CPU oracle takes
        it to repeat the device's summation order)."""
        if self.mode == "chain":
            fixed = state.splits if state is not None else self.attn_splits
            return lambda ctx: fixed
        cap = self.max_persistent_splits
        return lambda ctx: max(1, min(cap, -(-ctx // PERSISTENT_ATTN_CHUNK)))

    def _check(self, token_id: int, state: CudaDecodeState) -> None:
        if state.model is not self:
            raise ValueError("decode state belongs to another model")
        if state.position >= state.capacity:
            raise ValueError("decode state capacity exhausted")
        if not 0 <= int(token_id) < self.vocab:
            raise ValueError(f"token ID {token_id} is outside the vocabulary")

    def forward_token(self, token_id: int, state: CudaDecodeState) -> torch.Tensor:
        """Consume one token and return its next-token logits (cpu_lightspark.py:424-468)."""
        self._check(token_id, state)
        current = torch.cuda.current_stream(self.device)
        state.stream.wait_stream(current)
        state.set_token(token_id)
        state.replay()
        current.wait_stream(state.stream)
        return state.logits

    def decode_greedy(self, token_id: int, state: CudaDecodeState) -> int:
        """forward_token + argmax with the token ids on the host: consumes
        `token_id` and returns the greedy next token (the logits stay in
        state.logits), in one library call per token."""
        self._check(token_id, state)
        state.stream.wait_stream(torch.cuda.current_stream(self.device))
        return state.greedy_token(token_id)

    def prefill(self, token_ids, state: CudaDecodeState, max_tokens: int = 2048,
                attn_splits: int = 1, attention: str = "tensor") -> torch.Tensor:
        """Feed a prompt in one pass per `max_tokens` rows (h4b_prefill): the
        body projections run as tensor-core GEMMs over the prompt rows, each
        prompt query's attention in `attn_splits` context splits. Returns the
        last token's logits.

        attention="exact": the state then stands where forward_token over the
        same ids with that split count leaves it, bit for bit.
        attention="tensor" (one split, fp16 cache, head_dim 128, 4 q heads
        per kv head; otherwise as "exact"): tcgen05 attention with split fp16
        operands, within the 1e-3 relative tolerance of the fp32 path."""
        if attention not in PREFILL_ATTENTION:
            raise ValueError(f"attention must be one of {sorted(PREFILL_ATTENTION)}")
        ids = np.asarray([int(t) for t in token_ids], dtype=np.int32)
        if ids.size == 0:
            raise ValueError("empty prompt")
        if state.model is not self:
            raise ValueError("decode state belongs to another model")
        if state.position + ids.size > state.capacity:
            raise ValueError("decode state capacity exhausted")
        if ids.min() < 0 or ids.max() >= self.vocab:
            raise ValueError("token ID outside the vocabulary")
        rows = min(int(max_tokens), int(ids.size))
        scratch = self._prefill_scratch
        if scratch is None or scratch.max_tokens < rows or scratch.splits != int(attn_splits):
            scratch = self._prefill_scratch = PrefillScratch(self, rows, int(attn_splits))
        scratch.desc.attn_kernel = PREFILL_ATTENTION[attention]
        current = torch.cuda.current_stream(self.device)
        state.stream.wait_stream(current)
        with torch.cuda.stream(state.stream):
            for start in range(0, ids.size, scratch.max_tokens):
                part = ids[start:start + scratch.max_tokens]
                scratch.tokens[:part.size].copy_(torch.from_numpy(part), non_blocking=False)
                check(lib().h4b_prefill(ctypes.byref(self.desc), ctypes.byref(state.desc), ctypes.byref(scratch.desc),
                                        int(part.size), state.stream.cuda_stream), "h4b_prefill")
                state.position += int(part.size)
        current.wait_stream(state.stream)
        return state.logits

    def new_batch_state(self, batch: int, capacity: int, attn_splits: int = 16,
                        attention: str = "tensor") -> CudaBatchState:
        return CudaBatchState(self, batch, capacity, attn_splits, attention)

    def forward_batch(self, token_ids, state: CudaBatchState) -> torch.Tensor:
        """One token for each of the state's B sequences; returns the [B, V]
        logits (a view, overwritten by the next call). Row b equals what
        forward_token gives sequence b with the same attention splits."""
        ids = [int(t) for t in token_ids]
        if len(ids) != state.batch:
            raise ValueError(f"expected {state.batch} token ids, got {len(ids)}")
        if any(not 0 <= t < self.vocab for t in ids):
            raise ValueError("token ID outside the vocabulary")
        if int(state.position.max()) >= state.capacity:
            raise ValueError("decode state capacity exhausted")
        state.tokens.copy_(torch.tensor(ids, dtype=torch.int32), non_blocking=False)
        state.step()
        state.position += 1
        return state.logits

    def generate_batch(self, state: CudaBatchState, steps: int) -> None:
        """`steps` greedy tokens for every sequence, each fed back on the device
        (state.tokens holds the last tokens; call forward_batch first)."""
        if int(state.position.max()) + steps > state.capacity:
            raise ValueError("decode state capacity exhausted")
        for _ in range(steps):
            state.step()
        state.position += steps

    def generate_greedy(self, token_id: int, state: CudaDecodeState, steps: int) -> None:
        """Feed `token_id`, then `steps - 1` more greedy tokens, with no host
        round trip between steps (the graph feeds its own argmax back)."""
        self._check(token_id, state)
        if state.position + steps > state.capacity:
            raise ValueError("decode state capacity exhausted")
        current = torch.cuda.current_stream(self.device)
        state.stream.wait_stream(current)
        state.set_token(token_id)
        state.replay(steps)
        current.wait_stream(state.stream)

    def profile_forward_token(self, token_id: int, state: CudaDecodeState):
        """Time one real token by category with CUDA events, launching each
        stage separately (cpu_lightspark.py:470-553). Returns
        (logits, timings seconds, counts, total seconds)."""
        self._check(token_id, state)
        torch.cuda.synchronize(self.device)
        state.set_token(token_id)
        state.stream.synchronize()
        timings = {name: 0.0 for name in PROFILE_CATEGORIES}
        counts = {name: 0 for name in PROFILE_CATEGORIES}
        plan = [(0, 0, "embedding / LM head")]
        for layer in range(self.n_layers):
            plan += [(1, layer, "ternary/int4 GEMV"), (2, layer, "attention"), (3, layer, "ternary/int4 GEMV"),
                     (4, layer, "ternary/int4 GEMV"), (5, layer, "ternary/int4 GEMV")]
        plan += [(6, 0, "embedding / LM head"), (7, 0, None)]
        events = [torch.cuda.Event(enable_timing=True) for _ in range(len(plan) + 1)]
        started = time.perf_counter()
        with torch.cuda.stream(state.stream):
            events[0].record(state.stream)
            for index, (stage, layer, _) in enumerate(plan):
                check(lib().h4b_decode_stage(ctypes.byref(self.desc), ctypes.byref(state.desc), stage, layer,
                                             state.stream.cuda_stream), "h4b_decode_stage")
                events[index + 1].record(state.stream)
        state.stream.synchronize()
        total = time.perf_counter() - started
        for index, (_, _, name) in enumerate(plan):
            if name is None:
                continue
            timings[name] += events[index].elapsed_time(events[index + 1]) / 1000.0
            counts[name] += 1
        state.position += 1
        return state.logits, timings, counts, total

    def status(self) -> int:
        """Read and clear the device status word; raises on a wait timeout."""
        value = device_status()
        if value & STATUS_WAIT_TIMEOUT:
            raise RuntimeError("a device-side wait timed out (status word %d)" % value)
        return value
