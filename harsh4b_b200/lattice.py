"""The LATTICE checkpoint as the model's source: reading it, converting its
projections to the packed int4 cache on the GPU, and building the decode
model from it -- the B200 counterpart of ``cpu_lightspark.build_litespark_cpu``
(cpu_lightspark.py:559-676).

* :func:`read_lattice` maps the checkpoint (a ``torch.save`` archive of a
  dict: per projection ``<name>.weight`` -> the packed LATTICE fields,
  ``<name>.L`` / ``<name>.R`` -> the absorbed rotation, plus the fp32/fp16
  embedding and norm vectors and ``__latmeta__``).
* :func:`convert_projection` / :func:`convert_rows` run the conversion
  kernels of ``csrc/lattice.cu`` (``h4b_lattice_to_int4``,
  ``h4b_rows_to_int4``), replacing ``_convert_projection`` and
  ``_convert_embedding`` (cpu_lightspark.py:149-229).
* :func:`build_b200_model` finds or writes the cache directory the reference
  uses (same identity digest, file names and manifest, so either side reuses
  the other's cache), takes the norms from the checkpoint as the reference
  does (cpu_lightspark.py:650-668), and returns a
  :class:`harsh4b_b200.model.CudaQwen`.
"""
from __future__ import annotations

import ctypes
import hashlib
import json
import os
from pathlib import Path

import numpy as np

from .cache import Checkpoint, projection_names, slug

CACHE_VERSION = 2  # the reference's cache layout version (cpu_lightspark.py:32)
FORMAT = "lattice-to-row-int4-litespark"


def cache_identity(model_path) -> tuple[str, dict]:
    """The cache key of a checkpoint file, computed as the reference computes
    it (cpu_lightspark.py:232-243), so both find the same directory."""
    model_path = Path(model_path)
    stat = model_path.stat()
    identity = {"version": CACHE_VERSION, "source": str(model_path.resolve()), "size": stat.st_size,
                "mtime_ns": stat.st_mtime_ns, "format": FORMAT, "embedding": "symmetric-int4-per-row"}
    digest = hashlib.sha256(json.dumps(identity, sort_keys=True).encode()).hexdigest()[:16]
    return digest, identity


def read_lattice(path) -> dict:
    """Memory-maps a LATTICE checkpoint; tensor payloads stay on disk until
    read. Rejects anything but plain tensors, dicts, tuples and numbers."""
    import torch

    state = torch.load(str(path), map_location="cpu", mmap=True, weights_only=True)
    if not isinstance(state, dict) or "__latmeta__" not in state:
        raise ValueError(f"{path} is not a LATTICE checkpoint (no __latmeta__)")
    return state


def _numpy(value) -> np.ndarray:
    return value.numpy() if hasattr(value, "numpy") else np.asarray(value)


def _device_tensor(value, dtype=None):
    import torch

    array = np.ascontiguousarray(_numpy(value))
    if dtype is not None:
        array = array.astype(dtype, copy=False)
    return torch.from_numpy(array).cuda()


def convert_projection(packed: dict, left, right):
    """``_convert_projection`` (cpu_lightspark.py:149-201) on the GPU: returns
    (uint8[rows, width/2], float32[rows]) device tensors."""
    import torch

    from ._lib import LatticeProjectionDesc, check, lib, stream_handle

    rows, width = (int(v) for v in packed["shape"])
    blocksize = int(packed["blocksize"])
    nblocks = (width + blocksize - 1) // blocksize
    if width % 2:
        raise ValueError("LiteSpark int4 projections require even width")
    row_bytes = (width + 3) // 4
    maskid = _device_tensor(packed["maskid"], np.uint8).reshape(-1)
    t0 = _device_tensor(packed["T0"], np.uint8).reshape(-1)
    if maskid.numel() != rows * row_bytes or t0.numel() != rows * row_bytes:
        raise ValueError("LATTICE code planes do not match the projection shape")
    t1c = _device_tensor(packed["T1c"], np.uint8).reshape(-1)
    params = [_numpy(packed[k]) for k in ("mu", "a0", "a1")]
    half = all(p.dtype == np.float16 for p in params)
    dtype = np.float16 if half else np.float32
    mu, a0, a1 = (_device_tensor(p, dtype) for p in params)
    if mu.shape != (4, rows, nblocks) or a0.shape != (4, rows, nblocks) or a1.shape[1:] != (rows, nblocks):
        raise ValueError("LATTICE scale planes do not match the projection shape")
    o2 = [int(x) for x in _numpy(packed["o2_idx"]).reshape(-1)]
    if len(o2) != a1.shape[0] or len(o2) > 4:
        raise ValueError("o2_idx does not match the a1 planes")
    left_d = _device_tensor(left, np.float32)
    right_d = _device_tensor(right, np.float32)
    dim_l, dim_r = left_d.shape[0], right_d.shape[0]
    if left_d.shape != (dim_l, dim_l) or right_d.shape != (dim_r, dim_r) or dim_l * dim_r != width:
        raise ValueError("KOTMS rotation dimensions do not match projection width")
    desc = LatticeProjectionDesc()
    desc.rows, desc.width, desc.blocksize, desc.nblocks = rows, width, blocksize, nblocks
    desc.maskid, desc.t0, desc.t1c = maskid.data_ptr(), t0.data_ptr(), t1c.data_ptr()
    desc.n_t1, desc.t1c_bytes = int(packed["n_T1"]), int(t1c.numel())
    desc.mu, desc.a0, desc.a1 = mu.data_ptr(), a0.data_ptr(), a1.data_ptr()
    desc.param_dtype, desc.n_o2 = (1 if half else 0), len(o2)
    for i, mode in enumerate(o2):
        desc.o2_idx[i] = mode
    desc.left, desc.right, desc.dim_l, desc.dim_r = left_d.data_ptr(), right_d.data_ptr(), dim_l, dim_r
    out = torch.empty((rows, width // 2), dtype=torch.uint8, device="cuda")
    scales = torch.empty(rows, dtype=torch.float32, device="cuda")
    scratch = torch.empty(int(lib().h4b_lattice_scratch_bytes(rows)), dtype=torch.uint8, device="cuda")
    error = ctypes.c_int(0)
    rc = lib().h4b_lattice_to_int4(ctypes.byref(desc), out.data_ptr(), scales.data_ptr(), scratch.data_ptr(),
                                   ctypes.byref(error), stream_handle())
    if error.value:
        raise ValueError("T1 count does not match mask IDs")
    check(rc, "h4b_lattice_to_int4")
    return out, scales


def convert_rows(source):
    """``_convert_embedding`` (cpu_lightspark.py:204-229) on the GPU: per-row
    symmetric int4 of a dense float32 / float16 matrix."""
    import torch

    from ._lib import check, lib, stream_handle

    array = _numpy(source)
    if array.ndim != 2 or array.shape[1] % 2:
        raise ValueError("int4 embedding width must be even")
    dtype = np.float16 if array.dtype == np.float16 else np.float32
    rows, width = array.shape
    out = torch.empty((rows, width // 2), dtype=torch.uint8, device="cuda")
    scales = torch.empty(rows, dtype=torch.float32, device="cuda")
    # In slices, so a 1.5 GB fp32 embedding never sits whole on the device twice.
    step = max(1, (256 << 20) // (width * array.itemsize))
    for start in range(0, rows, step):
        stop = min(rows, start + step)
        src = _device_tensor(array[start:stop], dtype)
        check(lib().h4b_rows_to_int4(src.data_ptr(), 1 if dtype == np.float16 else 0, stop - start, width,
                                     out[start:stop].data_ptr(), scales[start:stop].data_ptr(), stream_handle()),
              "h4b_rows_to_int4")
    return out, scales


def _atomic_npy(path: Path, array: np.ndarray) -> None:
    temporary = path.with_suffix(".npy.tmp")
    with open(temporary, "wb") as handle:
        np.save(handle, array, allow_pickle=False)
    os.replace(temporary, path)


def _atomic_json(path: Path, value: dict) -> None:
    temporary = path.with_suffix(".tmp")
    temporary.write_text(json.dumps(value, indent=2, sort_keys=True))
    os.replace(temporary, path)


def norms_from_state(state: dict, config: dict) -> dict:
    """The fp32 norm vectors the reference takes from the checkpoint
    (cpu_lightspark.py:653-668)."""
    names = []
    for index in range(int(config["num_hidden_layers"])):
        prefix = f"model.layers.{index}"
        names += [f"{prefix}.input_layernorm.weight", f"{prefix}.post_attention_layernorm.weight",
                  f"{prefix}.self_attn.q_norm.weight", f"{prefix}.self_attn.k_norm.weight"]
    names.append("model.norm.weight")
    return {name: np.array(_numpy(state[name]), dtype=np.float32, copy=True) for name in names}


def build_cache(model_path, config: dict, cache_dir=None, verbose: bool = False) -> Checkpoint:
    """Finds or writes the packed cache of a LATTICE checkpoint and returns it
    with the checkpoint's norms. Missing projection files are converted on
    the GPU; existing ones (written by this code or by the reference's
    ``build_litespark_cpu``) are used as they are."""
    model_path = Path(model_path)
    digest, identity = cache_identity(model_path)
    directory = Path(cache_dir) if cache_dir else model_path.parent / ".cache" / "litespark-lattice" / digest
    directory.mkdir(parents=True, exist_ok=True)
    manifest_path = directory / "manifest.json"
    manifest = json.loads(manifest_path.read_text()) if manifest_path.exists() else {
        "identity": identity, "complete": False, "projections": {}}
    if manifest["identity"] != identity:
        raise ValueError(f"LiteSpark cache does not match checkpoint: {directory}")
    _atomic_json(manifest_path, manifest)
    state = read_lattice(model_path)
    names = projection_names(config)
    checkpoint = Checkpoint(config=dict(config))
    for index, name in enumerate(names, 1):
        weights_path = directory / f"{slug(name)}.int4.npy"
        scales_path = directory / f"{slug(name)}.scales.npy"
        if not weights_path.exists() or not scales_path.exists():
            if verbose:
                print(f"  Converting projection {index}/{len(names)} on the GPU: {name}", flush=True)
            packed, scales = convert_projection(state[name + ".weight"], state[name + ".L"], state[name + ".R"])
            _atomic_npy(weights_path, packed.cpu().numpy())
            _atomic_npy(scales_path, scales.cpu().numpy())
        manifest["projections"][name] = {"weights": weights_path.name, "scales": scales_path.name}
        _atomic_json(manifest_path, manifest)
        checkpoint.projections[name] = (np.load(weights_path, mmap_mode="r", allow_pickle=False),
                                        np.load(scales_path, mmap_mode="r", allow_pickle=False))
    embed_path, embed_scale_path = directory / "embedding.int4.npy", directory / "embedding.scales.npy"
    if not embed_path.exists() or not embed_scale_path.exists():
        if verbose:
            print("  Converting tied embedding/lm_head to int4 on the GPU", flush=True)
        packed, scales = convert_rows(state["model.embed_tokens.weight"])
        _atomic_npy(embed_path, packed.cpu().numpy())
        _atomic_npy(embed_scale_path, scales.cpu().numpy())
    checkpoint.embedding = np.load(embed_path, mmap_mode="r", allow_pickle=False)
    checkpoint.embedding_scales = np.load(embed_scale_path, mmap_mode="r", allow_pickle=False)
    checkpoint.norms = norms_from_state(state, config)
    checkpoint.validate()
    manifest["complete"] = True
    _atomic_json(manifest_path, manifest)
    return checkpoint


def build_b200_model(model_path, config: dict | None = None, cache_dir=None, verbose: bool = False, **model_kwargs):
    """``build_litespark_cpu`` (cpu_lightspark.py:559-676) for the B200: a
    :class:`CudaQwen` from a LATTICE checkpoint, through the shared cache.
    ``config`` defaults to Qwen3-4B (the reference's configs/qwen3-4b.json)."""
    from .model import CudaQwen
    from .synthetic import qwen3_4b_config

    checkpoint = build_cache(model_path, config or qwen3_4b_config(), cache_dir=cache_dir, verbose=verbose)
    return CudaQwen.from_checkpoint(checkpoint, **model_kwargs)
