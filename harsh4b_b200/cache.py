"""The packed int4 cache layout the reference's CPU runtime writes and reads.

Layout (``cpu_lightspark.build_litespark_cpu``, cpu_lightspark.py:571-676):

* ``manifest.json``: ``{"identity": ..., "complete": bool, "projections":
  {name: {"weights": file, "scales": file}}}``;
* ``<slug>.int4.npy``: ``uint8[N, K/2]``, two signed nibbles per byte, low
  nibble = even k (cpu_lightspark.py:139-146);
* ``<slug>.scales.npy``: ``float32[N]`` row scales;
* ``embedding.int4.npy`` / ``embedding.scales.npy``: the tied embedding / LM
  head in the same row-int4 format (cpu_lightspark.py:204-229).

The reference keeps the fp32 norm vectors in the LATTICE checkpoint; this
cache adds them as ``<slug>.npy`` files listed under ``manifest["norms"]`` so
a cache directory is self-contained.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

FORMAT = "lattice-to-row-int4-litespark"


def pack_int4(weights: np.ndarray) -> np.ndarray:
    """Pack signed [-7, +7] int8 values two per byte (cpu_lightspark.py:139-146)."""
    if weights.dtype != np.int8 or weights.ndim != 2 or weights.shape[1] % 2:
        raise ValueError("int4 matrix must be int8 with even width")
    if weights.size and (weights.min() < -7 or weights.max() > 7):
        raise ValueError("int4 values must be in [-7,+7]")
    even = weights[:, 0::2].view(np.uint8) & np.uint8(0x0F)
    odd = weights[:, 1::2].view(np.uint8) << np.uint8(4)
    return even | odd


def unpack_int4(packed: np.ndarray) -> np.ndarray:
    """Inverse of :func:`pack_int4` (cpu_lightspark.py:345-348, :616-625)."""
    signed = packed.view(np.int8)
    out = np.empty((packed.shape[0], packed.shape[1] * 2), dtype=np.int8)
    out[:, 0::2] = (signed << 4) >> 4
    out[:, 1::2] = signed >> 4
    return out


def quantize_rows_int4(weight: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Row-symmetric int4 quantisation of a dense fp32 matrix, the step that
    ends ``_convert_projection`` (cpu_lightspark.py:192-195)."""
    weight = np.asarray(weight, dtype=np.float32)
    scale = np.maximum(np.max(np.abs(weight), axis=1), np.float32(1e-8)) / np.float32(7.0)
    codes = np.rint(weight / scale[:, None]).clip(-7, 7).astype(np.int8)
    return pack_int4(codes), scale.astype(np.float32)


def projection_names(config) -> list[str]:
    """The 7 projections per layer in cache order (cpu_lightspark.py:585-595)."""
    names = []
    for index in range(int(config["num_hidden_layers"])):
        attn, mlp = f"model.layers.{index}.self_attn", f"model.layers.{index}.mlp"
        names += [f"{attn}.q_proj", f"{attn}.k_proj", f"{attn}.v_proj", f"{attn}.o_proj",
                  f"{mlp}.gate_proj", f"{mlp}.up_proj", f"{mlp}.down_proj"]
    return names


def norm_names(config) -> list[str]:
    names = []
    for index in range(int(config["num_hidden_layers"])):
        prefix = f"model.layers.{index}"
        names += [f"{prefix}.input_layernorm.weight", f"{prefix}.post_attention_layernorm.weight",
                  f"{prefix}.self_attn.q_norm.weight", f"{prefix}.self_attn.k_norm.weight"]
    return names + ["model.norm.weight"]


def slug(name: str) -> str:
    return name.replace(".", "_")  # cpu_lightspark.py:598


@dataclass
class Checkpoint:
    """A packed int4 model in host memory, keyed like the reference's state."""

    config: dict
    projections: dict = field(default_factory=dict)  # name -> (uint8[N,K/2], float32[N])
    embedding: np.ndarray | None = None              # uint8[V, H/2]
    embedding_scales: np.ndarray | None = None       # float32[V]
    norms: dict = field(default_factory=dict)        # name -> float32[n]

    def layer(self, index: int):
        """(qkv, o, gate_up, down, input_norm, post_norm, q_norm, k_norm), with q/k/v
        and gate/up rows concatenated as ``combine`` does (cpu_lightspark.py:638-667)."""
        attn, mlp, prefix = (f"model.layers.{index}.self_attn", f"model.layers.{index}.mlp",
                             f"model.layers.{index}")
        p = self.projections

        def cat(*names):
            return (np.concatenate([p[n][0] for n in names], axis=0),
                    np.concatenate([p[n][1] for n in names]))

        return (cat(f"{attn}.q_proj", f"{attn}.k_proj", f"{attn}.v_proj"), p[f"{attn}.o_proj"],
                cat(f"{mlp}.gate_proj", f"{mlp}.up_proj"), p[f"{mlp}.down_proj"],
                self.norms[f"{prefix}.input_layernorm.weight"],
                self.norms[f"{prefix}.post_attention_layernorm.weight"],
                self.norms[f"{attn}.q_norm.weight"], self.norms[f"{attn}.k_norm.weight"])

    def expected_shapes(self) -> dict:
        c = self.config
        h, i = int(c["hidden_size"]), int(c["intermediate_size"])
        q = int(c["num_attention_heads"]) * int(c["head_dim"])
        kv = int(c["num_key_value_heads"]) * int(c["head_dim"])
        per = {"q_proj": (q, h), "k_proj": (kv, h), "v_proj": (kv, h), "o_proj": (h, q),
               "gate_proj": (i, h), "up_proj": (i, h), "down_proj": (h, i)}
        return {name: per[name.rsplit(".", 1)[1]] for name in projection_names(c)}

    def validate(self) -> None:
        for name, (rows, width) in self.expected_shapes().items():
            weights, scales = self.projections[name]
            if weights.shape != (rows, width // 2) or weights.dtype != np.uint8:
                raise ValueError(f"invalid packed cache shape for {name}: {weights.shape}")
            if scales.shape != (rows,) or scales.dtype != np.float32:
                raise ValueError(f"invalid row scales for {name}")
        vocab, hidden = int(self.config["vocab_size"]), int(self.config["hidden_size"])
        if self.embedding.shape != (vocab, hidden // 2) or self.embedding_scales.shape != (vocab,):
            raise ValueError("invalid embedding cache shape")


def _atomic_save(path: Path, array: np.ndarray) -> None:
    temporary = path.with_suffix(".npy.tmp")
    with open(temporary, "wb") as handle:
        np.save(handle, array, allow_pickle=False)
    os.replace(temporary, path)


def _atomic_json(path: Path, value: dict) -> None:
    temporary = path.with_suffix(".tmp")
    temporary.write_text(json.dumps(value, indent=2, sort_keys=True))
    os.replace(temporary, path)


def write_cache(directory, checkpoint: Checkpoint, identity: dict | None = None) -> Path:
    """Write ``checkpoint`` in the reference's cache layout, atomically per file
    with the manifest updated after each projection (cpu_lightspark.py:597-607)."""
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    manifest = {"identity": identity or {"format": FORMAT, "source": "synthetic"},
                "complete": False, "projections": {}, "norms": {}, "config": checkpoint.config}
    manifest_path = directory / "manifest.json"
    _atomic_json(manifest_path, manifest)
    for name in projection_names(checkpoint.config):
        weights, scales = checkpoint.projections[name]
        files = {"weights": f"{slug(name)}.int4.npy", "scales": f"{slug(name)}.scales.npy"}
        _atomic_save(directory / files["weights"], weights)
        _atomic_save(directory / files["scales"], scales)
        manifest["projections"][name] = files
        _atomic_json(manifest_path, manifest)
    _atomic_save(directory / "embedding.int4.npy", checkpoint.embedding)
    _atomic_save(directory / "embedding.scales.npy", checkpoint.embedding_scales)
    for name, value in checkpoint.norms.items():
        manifest["norms"][name] = f"{slug(name)}.npy"
        _atomic_save(directory / manifest["norms"][name], np.asarray(value, dtype=np.float32))
    manifest["complete"] = True
    _atomic_json(manifest_path, manifest)
    return directory


def read_cache(directory, config: dict | None = None, *, mmap: bool = True) -> Checkpoint:
    """Load a cache directory written by :func:`write_cache` or by the reference
    (the reference cache carries no norms; pass them in ``Checkpoint.norms``)."""
    directory = Path(directory)
    manifest = json.loads((directory / "manifest.json").read_text())
    if not manifest.get("complete"):
        raise ValueError(f"packed cache is incomplete: {directory}")
    config = config or manifest.get("config")
    if config is None:
        raise ValueError("cache has no config; pass the model config")
    mode = "r" if mmap else None
    load = lambda file: np.load(directory / file, mmap_mode=mode, allow_pickle=False)  # noqa: E731
    checkpoint = Checkpoint(config=config)
    for name in projection_names(config):
        files = manifest["projections"][name]
        checkpoint.projections[name] = (load(files["weights"]), load(files["scales"]))
    checkpoint.embedding = load("embedding.int4.npy")
    checkpoint.embedding_scales = load("embedding.scales.npy")
    for name, file in manifest.get("norms", {}).items():
        checkpoint.norms[name] = np.array(load(file), dtype=np.float32)
    checkpoint.validate()
    return checkpoint
