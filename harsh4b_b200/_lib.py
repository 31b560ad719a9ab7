"""ctypes binding of ``libharsh4b_b200.so`` (declared in include/harsh4b_b200.h).

There is no fallback: if the library is missing or no CUDA device is
visible, every entry point raises.
"""
from __future__ import annotations

import ctypes
from functools import lru_cache
from pathlib import Path

LIBRARY = Path(__file__).resolve().parent / "libharsh4b_b200.so"

H4B_EINVAL = -1
H4B_EUNSUPPORTED = -2
H4B_ETOOBIG = -3

STATUS_WAIT_TIMEOUT = 1
STATUS_BAD_TOKEN = 2
STATUS_BAD_POSITION = 4

_vp, _i32, _f32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_float


class ModelDesc(ctypes.Structure):
    """Mirror of ``h4b_model``."""

    _fields_ = [(n, _i32) for n in ("layers", "hidden", "intermediate", "heads", "kv_heads", "head_dim",
                                    "vocab", "max_pos")] + [("eps", _f32)] + [
        (n, _vp) for n in ("w_qkv", "s_qkv", "w_o", "s_o", "w_gate_up", "s_gate_up", "w_down", "s_down",
                           "w_embed", "s_embed", "norm_in", "norm_post", "norm_q", "norm_k", "norm_final",
                           "rope_cos", "rope_sin")]


class StateDesc(ctypes.Structure):
    """Mirror of ``h4b_state``."""

    _fields_ = [("capacity", _i32), ("kv_dtype", _i32), ("attn_splits", _i32)] + [
        (n, _vp) for n in ("k_cache", "v_cache", "position", "token", "next_token", "x", "qkv", "attended",
                           "act", "logits", "absmax", "argmax_key", "attn_partials", "attn_counters", "exchange")]


class BatchStateDesc(ctypes.Structure):
    """Mirror of ``h4b_batch_state``."""

    _fields_ = [("batch", _i32), ("capacity", _i32), ("kv_dtype", _i32), ("attn_splits", _i32)] + [
        (n, _vp) for n in ("k_cache", "v_cache", "positions", "tokens", "next_tokens", "x", "x8", "act_scale",
                           "act_sum", "qkv", "attended", "proj", "gate_up", "act", "logits", "attn_partials",
                           "attn_counters", "gemm_acc")] + [("attn_kernel", _i32), ("gemm_acc_width", _i32)]


class PrefillScratchDesc(ctypes.Structure):
    """Mirror of ``h4b_prefill_scratch``."""

    _fields_ = [("max_tokens", _i32), ("attn_queries", _i32), ("attn_splits", _i32)] + [
        (n, _vp) for n in ("x", "x8", "act_scale", "act_sum", "qkv", "attended", "gate_up", "act", "proj", "tokens",
                           "positions", "attn_partials", "attn_counters")] + [("attn_kernel", _i32)]


class LatticeProjectionDesc(ctypes.Structure):
    """Mirror of ``h4b_lattice_projection``."""

    _fields_ = [("rows", _i32), ("width", _i32), ("blocksize", _i32), ("nblocks", _i32),
                ("maskid", _vp), ("t0", _vp), ("t1c", _vp), ("n_t1", ctypes.c_longlong),
                ("t1c_bytes", ctypes.c_longlong), ("mu", _vp), ("a0", _vp), ("a1", _vp),
                ("param_dtype", _i32), ("n_o2", _i32), ("o2_idx", _i32 * 4), ("left", _vp), ("right", _vp),
                ("dim_l", _i32), ("dim_r", _i32)]


class TpGroupDesc(ctypes.Structure):
    """Mirror of ``h4b_tp_group``."""

    _fields_ = [("world", _i32), ("rank", _i32), ("capacity", _i32), ("buffers", _vp * 8), ("generation", _vp)]


_SIGNATURES = {
    "h4b_prepare": [],
    "h4b_get_status": [_vp],
    "h4b_device_info": [_vp, _vp, _vp],
    "h4b_int4_i8_gemv": [_vp, _vp, _vp, _f32, _vp, _vp, _i32, _i32, _vp],
    "h4b_int4_gemv_fused_quant": [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _vp],
    "h4b_int4_gemv_fused_quant_ex": [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp],
    "h4b_quantize_activation": [_vp, _vp, _vp, _i32, _vp],
    "h4b_rmsnorm": [_vp, _vp, _vp, _i32, _f32, _vp],
    "h4b_add_inplace": [_vp, _vp, _i32, _vp],
    "h4b_gqa_decode": [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _vp],
    "h4b_gqa_decode_noalloc": [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _vp],
    "h4b_embedding": [_vp, _vp, _vp, _vp, _i32, _i32, _vp],
    "h4b_argmax": [_vp, _i32, _vp, _vp],
    "h4b_validate": [ctypes.POINTER(ModelDesc), ctypes.POINTER(StateDesc)],
    "h4b_decode_stage": [ctypes.POINTER(ModelDesc), ctypes.POINTER(StateDesc), _i32, _i32, _vp],
    "h4b_decode_step": [ctypes.POINTER(ModelDesc), ctypes.POINTER(StateDesc), _vp],
    "h4b_graph_create": [ctypes.POINTER(ModelDesc), ctypes.POINTER(StateDesc), _vp, ctypes.POINTER(_vp)],
    "h4b_decode_persistent": [ctypes.POINTER(ModelDesc), ctypes.POINTER(StateDesc), _vp],
    "h4b_graph_create_persistent": [ctypes.POINTER(ModelDesc), ctypes.POINTER(StateDesc), _vp,
                                    ctypes.POINTER(_vp)],
    "h4b_graph_launch": [_vp, _vp],
    "h4b_graph_destroy": [_vp],
    "h4b_persistent_exchange_words": [ctypes.POINTER(ModelDesc)],
    "h4b_sample": [_vp, _i32, _vp, _i32, _f32, _i32, _f32, _f32, ctypes.c_double, _vp, _vp, _vp, _vp, _vp],
    "h4b_sample_scratch_bytes": [_i32, _i32],
    "h4b_quantize_rows": [_vp, _vp, _vp, _vp, _i32, _i32, _vp],
    "h4b_int4_gemm": [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp],
    "h4b_int4_gemm_ex": [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _vp],
    "h4b_graph_token": [_vp, _vp, _vp, _vp, _vp, _vp],
    "h4b_int4_gemm_acc": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _vp],
    "h4b_validate_batch": [ctypes.POINTER(ModelDesc), ctypes.POINTER(BatchStateDesc)],
    "h4b_int4_gemv_absmax": [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _vp],
    "h4b_residual_acc": [_vp, _vp, _vp, _vp, _i32, _vp],
    "h4b_decode_batch": [ctypes.POINTER(ModelDesc), ctypes.POINTER(BatchStateDesc), _vp],
    "h4b_batch_attention": [ctypes.POINTER(ModelDesc), ctypes.POINTER(BatchStateDesc), _i32, _vp],
    "h4b_prefill_attention": [ctypes.POINTER(ModelDesc), ctypes.POINTER(StateDesc), ctypes.POINTER(PrefillScratchDesc),
                              _i32, _i32, _vp],
    "h4b_tp_buffer_bytes": [_i32, _i32],
    "h4b_ipc_alloc": [ctypes.c_longlong, ctypes.POINTER(_vp), _vp],
    "h4b_ipc_open": [_vp, ctypes.POINTER(_vp)],
    "h4b_ipc_close": [_vp],
    "h4b_ipc_free": [_vp],
    "h4b_tp_allreduce_max": [ctypes.POINTER(TpGroupDesc), _vp, _vp],
    "h4b_tp_allreduce_sum_residual": [ctypes.POINTER(TpGroupDesc), _vp, _vp, _vp, _vp, _i32, _vp],
    "h4b_tp_gather_best": [ctypes.POINTER(TpGroupDesc), _vp, _vp, _i32, _vp, _vp],
    "h4b_prefill": [ctypes.POINTER(ModelDesc), ctypes.POINTER(StateDesc), ctypes.POINTER(PrefillScratchDesc), _i32,
                    _vp],
    "h4b_prefill_tp_stage": [ctypes.POINTER(ModelDesc), ctypes.POINTER(StateDesc), ctypes.POINTER(PrefillScratchDesc),
                             _i32, _i32, _i32, _vp, _vp, _i32, _vp, _vp, _vp],
    "h4b_lattice_scratch_bytes": [_i32],
    "h4b_lattice_to_int4": [ctypes.POINTER(LatticeProjectionDesc), _vp, _vp, _vp, ctypes.POINTER(_i32), _vp],
    "h4b_rows_to_int4": [_vp, _i32, _i32, _i32, _vp, _vp, _vp],
}
_RESTYPES = {"h4b_persistent_exchange_words": ctypes.c_longlong, "h4b_sample_scratch_bytes": ctypes.c_longlong,
             "h4b_tp_buffer_bytes": ctypes.c_longlong, "h4b_lattice_scratch_bytes": ctypes.c_longlong}


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


@lru_cache(None)
def load_library(path: str | None = None) -> ctypes.CDLL:
    """Load the library without touching the GPU (works on a CPU-only host)."""
    target = Path(path) if path else LIBRARY
    if not target.exists():
        raise RuntimeError(f"{target.name} is not built; run `python -m harsh4b_b200.build` "
                           "(harsh4b_b200 has no CPU fallback)")
    lib = ctypes.CDLL(str(target))
    for name, argtypes in _SIGNATURES.items():
        function = getattr(lib, name)
        function.argtypes = argtypes
        function.restype = _RESTYPES.get(name, _i32)
    return lib


@lru_cache(None)
def lib() -> ctypes.CDLL:
    """The library, after checking that a CUDA device is usable."""
    import torch

    if not torch.cuda.is_available():
        raise RuntimeError("harsh4b_b200 needs a CUDA device (B200, sm_100a); there is no CPU fallback")
    major, minor = torch.cuda.get_device_capability()
    if (major, minor) != (10, 0):
        raise RuntimeError(f"harsh4b_b200 is built for sm_100a; this device is sm_{major}{minor}")
    library = load_library()
    check(library.h4b_prepare(), "h4b_prepare")
    return library


_MESSAGES = {H4B_EINVAL: "invalid argument (size, alignment or null pointer)",
             H4B_EUNSUPPORTED: "shape not supported by the sm_100a kernels",
             H4B_ETOOBIG: "request exceeds the library's static scratch (kv_heads * groups * (head_dim + 4) "
                          "must be <= 262144 floats)"}


def check(rc: int, what: str) -> None:
    if rc == 0:
        return
    if rc in _MESSAGES:
        raise ValueError(f"{what}: {_MESSAGES[rc]}")
    raise RuntimeError(f"{what}: CUDA error {rc}")


def stream_handle(stream=None) -> int:
    import torch

    stream = stream or torch.cuda.current_stream()
    return stream.cuda_stream


def device_status() -> int:
    """Read and clear the device status word (synchronises the device)."""
    value = ctypes.c_int(0)
    check(lib().h4b_get_status(ctypes.byref(value)), "h4b_get_status")
    return value.value
