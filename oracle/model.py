"""Numpy restatement of ``cpu_lightspark.LiteSparkQwen`` -- TEST INFRASTRUCTURE ONLY.

Each method cites the reference lines it restates (paths relative to the
reference project root). Heavy arithmetic goes through the C oracle
(``litespark_oracle.c``); the orchestration is plain numpy.

``kv_dtype=np.float16`` rounds every stored key/value through fp16, which
mirrors the device cache's precision; the default fp32 is the reference's
own cache (cpu_lightspark.py:290).

RMSNorm, qk-norm, attention and SiLU run in the device kernels' reduction
order with the shared exp (see litespark_oracle.c); ``attn_splits`` (an int,
or a function of the context length) must follow the device's split choice
for bit-exact comparisons.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import OracleKernel, gqa_splitk, library, _ptr


@dataclass(frozen=True)
class OracleProjection:
    """One row-scaled packed int4 matrix (cpu_lightspark.py:246-260)."""

    weights: np.ndarray  # uint8[N, K/2]; low nibble = even k
    scales: np.ndarray   # float32[N]

    @property
    def input_size(self) -> int:
        return self.weights.shape[1] * 2

    @property
    def output_size(self) -> int:
        return self.weights.shape[0]


@dataclass(frozen=True)
class OracleLayer:
    """Fused per-layer projections (cpu_lightspark.py:263-272, fused at :638-661)."""

    qkv: OracleProjection
    o: OracleProjection
    gate_up: OracleProjection
    down: OracleProjection
    input_norm: np.ndarray
    post_norm: np.ndarray
    q_norm: np.ndarray
    k_norm: np.ndarray


class OracleState:
    """Caller-owned KV cache and scratch (cpu_lightspark.py:275-309)."""

    def __init__(self, model: "OracleQwen", capacity: int):
        if capacity < 1:
            raise ValueError("decode capacity must be positive")
        c = model.config
        self.capacity = capacity
        self.position = 0
        shape = (model.n_layers, capacity, model.kv_heads, model.head_dim)
        self.keys = np.zeros(shape, dtype=np.float32)
        self.values = np.zeros(shape, dtype=np.float32)
        self.x = np.empty(model.hidden, dtype=np.float32)
        self.normalized = np.empty(model.hidden, dtype=np.float32)
        self.quantized = np.empty(max(model.hidden, model.q_size, model.intermediate), dtype=np.int8)
        self.qkv = np.empty(model.q_size + 2 * model.kv_size, dtype=np.float32)
        self.attended = np.empty(model.q_size, dtype=np.float32)
        self.projected = np.empty(model.hidden, dtype=np.float32)
        self.gate_up = np.empty(2 * model.intermediate, dtype=np.float32)
        self.activated = np.empty(model.intermediate, dtype=np.float32)
        self.scores = np.empty((model.heads, capacity), dtype=np.float32)
        self.logits = np.empty(int(c["vocab_size"]), dtype=np.float32)


def rope_tables(config) -> tuple[np.ndarray, np.ndarray]:
    """fp32 cos/sin tables [max_position, head_dim/2] (cpu_lightspark.py:329-336)."""
    head_dim = int(config["head_dim"])
    exponent = np.arange(0, head_dim, 2, dtype=np.float32) / np.float32(head_dim)
    inv_freq = np.float32(1.0) / np.float32(config["rope_theta"]) ** exponent
    positions = np.arange(int(config["max_position_embeddings"]), dtype=np.float32)
    angles = positions[:, None] * inv_freq[None, :]
    return np.cos(angles).astype(np.float32), np.sin(angles).astype(np.float32)


class OracleQwen:
    """Torch-free Qwen3 single-token decode (cpu_lightspark.py:312-468)."""

    def __init__(self, config, layers, embedding, embedding_scales, final_norm, *, kv_dtype=np.float32,
                 attn_splits: int = 16):
        self.config = config
        self.layers = list(layers)
        self.embedding = embedding
        self.embedding_scales = embedding_scales
        self.lm_head = OracleProjection(embedding, embedding_scales)
        self.final_norm = final_norm
        self.kernel = OracleKernel()
        self.kv_dtype = np.dtype(kv_dtype)
        self.attn_splits = attn_splits
        self.n_layers = int(config["num_hidden_layers"])
        self.hidden = int(config["hidden_size"])
        self.intermediate = int(config["intermediate_size"])
        self.heads = int(config["num_attention_heads"])
        self.kv_heads = int(config["num_key_value_heads"])
        self.head_dim = int(config["head_dim"])
        self.groups = self.heads // self.kv_heads
        self.q_size = self.heads * self.head_dim
        self.kv_size = self.kv_heads * self.head_dim
        self.eps = float(config["rms_norm_eps"])
        self.rope_cos, self.rope_sin = rope_tables(config)
        library()  # fail early when the oracle library is missing

    def new_state(self, capacity: int) -> OracleState:
        return OracleState(self, capacity)

    # cpu_lightspark.py:341-349
    def embedding_into(self, token_id: int, out: np.ndarray) -> None:
        if not 0 <= token_id < self.embedding.shape[0]:
            raise ValueError(f"token ID {token_id} is outside the vocabulary")
        signed = self.embedding[token_id].view(np.int8)
        out[0::2] = (signed << 4) >> 4
        out[1::2] = signed >> 4
        out *= self.embedding_scales[token_id]

    # cpu_lightspark.py:351-371 (int4 layout, native-kernel branch)
    def project(self, projection: OracleProjection, quantized: np.ndarray, scale: float, out: np.ndarray):
        library().oracle_int4_i8_gemv(_ptr(quantized), _ptr(projection.weights), _ptr(projection.scales),
                                      scale, _ptr(out), projection.output_size, projection.input_size)

    def quantize(self, values: np.ndarray, state: OracleState) -> tuple[np.ndarray, float]:
        quantized = state.quantized[:values.size]
        return quantized, self.kernel.quantize_activation(values, quantized)

    # cpu_lightspark.py:373-379: divide by sqrt(mean(v^2) + eps), then scale.
    def qk_norm(self, values: np.ndarray, gamma: np.ndarray) -> None:
        library().oracle_qk_norm(_ptr(values), _ptr(gamma), values.shape[0], self.eps)

    # cpu_lightspark.py:381-387: half-split rotation at one position.
    def rope(self, values: np.ndarray, position: int) -> None:
        half = values.shape[1] // 2
        cosine, sine = self.rope_cos[position], self.rope_sin[position]
        x1 = values[:, :half].copy()
        x2 = values[:, half:].copy()
        values[:, :half] = x1 * cosine - x2 * sine
        values[:, half:] = x2 * cosine + x1 * sine

    # cpu_lightspark.py:389-422: softmax(q.k / sqrt(d)) v over t <= position.
    def attention(self, state: OracleState, layer_index: int, q: np.ndarray) -> None:
        context = state.position + 1
        splits = self.attn_splits(context) if callable(self.attn_splits) else self.attn_splits
        gqa_splitk(np.ascontiguousarray(q), state.keys[layer_index], state.values[layer_index], state.attended,
                   context, self.kv_heads, self.groups, int(splits))

    def _store(self, values: np.ndarray) -> np.ndarray:
        if self.kv_dtype == np.float32:
            return values
        return values.astype(self.kv_dtype).astype(np.float32)

    # cpu_lightspark.py:424-468
    def forward_token(self, token_id: int, state: OracleState) -> np.ndarray:
        if state.position >= state.capacity:
            raise ValueError("decode state capacity exhausted")
        q_end, k_end = self.q_size, self.q_size + self.kv_size
        self.embedding_into(token_id, state.x)
        for index, layer in enumerate(self.layers):
            self.kernel.rmsnorm_into(state.x, layer.input_norm, state.normalized, self.eps)
            quantized, scale = self.quantize(state.normalized, state)
            self.project(layer.qkv, quantized, scale, state.qkv)
            q = state.qkv[:q_end].reshape(self.heads, self.head_dim)
            k = state.qkv[q_end:k_end].reshape(self.kv_heads, self.head_dim)
            v = state.qkv[k_end:].reshape(self.kv_heads, self.head_dim)
            self.qk_norm(q, layer.q_norm)
            self.qk_norm(k, layer.k_norm)
            self.rope(q, state.position)
            self.rope(k, state.position)
            state.keys[index, state.position] = self._store(k)
            state.values[index, state.position] = self._store(v)
            self.attention(state, index, q)
            quantized, scale = self.quantize(state.attended, state)
            self.project(layer.o, quantized, scale, state.projected)
            self.kernel.add_inplace(state.x, state.projected)

            self.kernel.rmsnorm_into(state.x, layer.post_norm, state.normalized, self.eps)
            quantized, scale = self.quantize(state.normalized, state)
            self.project(layer.gate_up, quantized, scale, state.gate_up)
            gate = state.gate_up[:self.intermediate]
            up = state.gate_up[self.intermediate:]
            library().oracle_silu_mul(_ptr(gate), _ptr(up), _ptr(state.activated), self.intermediate)
            quantized, scale = self.quantize(state.activated, state)
            self.project(layer.down, quantized, scale, state.projected)
            self.kernel.add_inplace(state.x, state.projected)

        self.kernel.rmsnorm_into(state.x, self.final_norm, state.normalized, self.eps)
        quantized, scale = self.quantize(state.normalized, state)
        self.project(self.lm_head, quantized, scale, state.logits)
        state.position += 1
        return state.logits


def sample_logits(logits: np.ndarray, generated: list[int], *, argmax: bool, temperature: float = 0.7,
                  top_k: int = 40, top_p: float = 0.9, repetition_penalty: float = 1.08,
                  generator: np.random.Generator | None = None) -> int:
    """Restates cpu_lightspark.sample_logits (cpu_lightspark.py:700-726)."""
    if argmax:
        return int(np.asarray(logits).argmax())
    work = np.array(logits, dtype=np.float32, copy=True).reshape(-1)
    if generated and repetition_penalty != 1.0:
        seen = np.unique(np.asarray(generated, dtype=np.int64))
        old = work[seen]
        penalty = np.float32(repetition_penalty)
        work[seen] = np.where(old > 0, old / penalty, old * penalty)
    work /= np.float32(temperature)
    count = min(top_k, work.size)
    candidates = np.argpartition(-work, count - 1)[:count]
    candidates = candidates[np.argsort(-work[candidates])]
    chosen = work[candidates]
    chosen -= chosen.max()
    probabilities = np.exp(chosen, dtype=np.float32)
    probabilities /= probabilities.sum(dtype=np.float32)
    if top_p < 1.0:
        probabilities[(np.cumsum(probabilities) - probabilities) >= top_p] = 0
        probabilities /= probabilities.sum(dtype=np.float32)
    generator = generator or np.random.default_rng(0)
    return int(generator.choice(candidates, p=probabilities))


def choice_uniform(ids: np.ndarray, probabilities: np.ndarray, uniform: float) -> int:
    """numpy's Generator.choice(ids, p=probabilities) for a given draw
    u = generator.random(): the first index whose normalised float64
    cumulative probability exceeds u (searchsorted, side='right')."""
    cdf = np.asarray(probabilities, dtype=np.float64).cumsum()
    cdf /= cdf[-1]
    return int(ids[int(np.searchsorted(cdf, uniform, side="right"))])


def sample_runtime(logits: np.ndarray, generated: list[int], uniform: float, *, temperature: float = 0.7,
                   top_p: float = 0.9, top_k: int = 50, repetition_penalty: float = 1.15,
                   return_candidates: bool = False):
    """Restates inference_runtime.sample_numpy (inference_runtime.py:144-163),
    the CPU runtime's sampler, with the generator's draw passed in as
    `uniform` (see choice_uniform). top_k <= 0 means 50 (the CUDA and MLX
    samplers' rule, inference_runtime.py:243,180)."""
    values = np.array(logits, dtype=np.float32, copy=True).reshape(-1)
    if generated and repetition_penalty != 1.0:
        ids = np.array(sorted(set(generated)), dtype=np.int64)
        repeated = values[ids]
        values[ids] = np.where(repeated > 0, repeated / np.float32(repetition_penalty),
                               repeated * np.float32(repetition_penalty))
    if temperature <= 0.01:
        token = int(values.argmax())
        return (token, None, None) if return_candidates else token
    values /= np.float32(temperature)
    count = min(top_k if top_k > 0 else 50, values.size)
    ids = np.argpartition(-values, count - 1)[:count]
    ids = ids[np.lexsort((ids, -values[ids]))]  # descending; equal values by index (the reference leaves ties open)
    selected = values[ids]
    selected -= selected.max()
    probabilities = np.exp(selected, dtype=np.float32)
    probabilities /= probabilities.sum(dtype=np.float32)
    if top_p < 1.0:
        probabilities[(np.cumsum(probabilities) - probabilities) >= top_p] = 0
        probabilities /= probabilities.sum(dtype=np.float32)
    token = choice_uniform(ids, probabilities, uniform)
    return (token, ids, probabilities) if return_candidates else token
