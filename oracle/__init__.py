"""CPU oracle -- TEST INFRASTRUCTURE ONLY.

A restatement of the reference's CPU int4 decode path: the C kernels in
``litespark_oracle.c`` plus the numpy model in ``oracle.model``. Only tests/,
``__graft_entry__.smoke()`` and bench.py's cpu_baseline / ``--impl reference``
leg import this package, and only as the checker or the timed CPU baseline;
``harsh4b_b200`` never imports it.

Parity status: the model orchestration is pinned against fixtures produced by
running the reference's own ``cpu_lightspark.LiteSparkQwen.forward_token``
(``tests/golden/make_golden.py``); the GEMV and GQA kernels are pinned by the
reference's known-answer tests (``tests/test_cpu_lightspark.py:59-122`` of the
reference). The third-party ``litespark_inference`` arithmetic (RMSNorm,
activation quantisation, residual add) is restated, not pinned.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from functools import lru_cache
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIBRARY = HERE / "liblitespark_oracle.so"


def build(force: bool = False) -> Path:
    """Compile the C oracle with its Makefile (gcc + OpenMP)."""
    source = HERE / "litespark_oracle.c"
    if force or not LIBRARY.exists() or LIBRARY.stat().st_mtime < source.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE), "-B" if force else "liblitespark_oracle.so"],
                       check=True)
    return LIBRARY


@lru_cache(None)
def library() -> ctypes.CDLL:
    if not LIBRARY.exists():
        build()
    lib = ctypes.CDLL(str(LIBRARY))
    vp, f32, i32 = ctypes.c_void_p, ctypes.c_float, ctypes.c_int
    lib.oracle_int4_i8_gemv.argtypes = [vp, vp, vp, f32, vp, i32, i32]
    lib.oracle_int4_i8_gemv.restype = None
    lib.oracle_int4_i8_gemv_acc.argtypes = [vp, vp, vp, f32, vp, vp, i32, i32, i32]
    lib.oracle_int4_i8_gemv_acc.restype = None
    lib.oracle_quantize_activation.argtypes = [vp, vp, i32]
    lib.oracle_quantize_activation.restype = f32
    lib.oracle_rmsnorm.argtypes = [vp, vp, vp, i32, f32]
    lib.oracle_rmsnorm.restype = None
    lib.oracle_add_inplace.argtypes = [vp, vp, i32]
    lib.oracle_add_inplace.restype = None
    lib.oracle_gqa_decode.argtypes = [vp] * 5 + [i32] * 5
    lib.oracle_gqa_decode.restype = None
    lib.oracle_expf.argtypes = [f32]
    lib.oracle_expf.restype = f32
    lib.oracle_exp_array.argtypes = [vp, vp, i32]
    lib.oracle_exp_array.restype = None
    lib.oracle_qk_norm.argtypes = [vp, vp, i32, f32]
    lib.oracle_qk_norm.restype = None
    lib.oracle_silu_mul.argtypes = [vp, vp, vp, i32]
    lib.oracle_silu_mul.restype = None
    lib.oracle_gqa_splitk.argtypes = [vp, vp, vp, vp, i32, i32, i32, ctypes.c_long, ctypes.c_long, i32]
    lib.oracle_gqa_splitk.restype = None
    lib.oracle_max_threads.argtypes = []
    lib.oracle_max_threads.restype = i32
    return lib


def _ptr(array: np.ndarray) -> int:
    if not array.flags.c_contiguous:
        raise ValueError("oracle kernels need C-contiguous arrays")
    return array.ctypes.data


def max_threads() -> int:
    return int(library().oracle_max_threads())


def int4_gemv_function():
    """The C function with litespark_int4_i8_gemv's ctypes signature
    (cpu_lightspark.py:71-79), usable as LiteSparkQwen.int4_kernel."""
    return library().oracle_int4_i8_gemv


def int4_gemv(x8: np.ndarray, weights: np.ndarray, scales: np.ndarray, activation_scale: float,
              *, scalar: bool = False) -> tuple[np.ndarray, np.ndarray]:
    """Returns (fp32 outputs, int32 accumulators) for packed uint8[N, K/2]."""
    rows, packed = weights.shape
    out = np.empty(rows, dtype=np.float32)
    acc = np.empty(rows, dtype=np.int32)
    x8 = np.ascontiguousarray(x8, dtype=np.int8)
    if x8.size != 2 * packed:
        raise ValueError("activation width does not match the packed weights")
    library().oracle_int4_i8_gemv_acc(_ptr(x8), _ptr(weights), _ptr(scales), float(activation_scale),
                                      _ptr(out), _ptr(acc), rows, 2 * packed, 0 if scalar else 1)
    return out, acc


def quantize_activation(values: np.ndarray, quantized: np.ndarray) -> float:
    if quantized.size < values.size or quantized.dtype != np.int8:
        raise ValueError("int8 output buffer is smaller than the activation")
    return float(library().oracle_quantize_activation(_ptr(values), _ptr(quantized), values.size))


def exp(values: np.ndarray) -> np.ndarray:
    """The shared exp (oracle_expf) applied elementwise to float32 values."""
    values = np.ascontiguousarray(values, dtype=np.float32)
    out = np.empty_like(values)
    library().oracle_exp_array(_ptr(values), _ptr(out), values.size)
    return out


def gqa_splitk(query, keys, values, output, context, kv_heads, groups, splits):
    """GQA in the device's split-K order; keys/values [time, kv_heads, 128]."""
    if query.shape[-1] != 128 or not 1 <= splits <= 64:
        raise ValueError("device-order attention needs head_dim 128 and 1..64 splits")
    library().oracle_gqa_splitk(_ptr(query), _ptr(keys), _ptr(values), _ptr(output), context, kv_heads,
                                groups, kv_heads * 128, 128, splits)


def gqa_decode(query, keys, values, scores, output, context, kv_heads, groups, head_dim, score_stride):
    library().oracle_gqa_decode(_ptr(query), _ptr(keys), _ptr(values), _ptr(scores), _ptr(output),
                                context, kv_heads, groups, head_dim, score_stride)


class OracleKernel:
    """Restates the third-party ``litespark_inference.torchless.kernel`` object
    that ``LiteSparkQwen`` calls (cpu_lightspark.py:362-365, 431-463)."""

    def rmsnorm_into(self, x, weight, out, eps):
        library().oracle_rmsnorm(_ptr(x), _ptr(weight), _ptr(out), x.size, float(eps))

    def quantize_activation(self, values, quantized):
        return quantize_activation(values, quantized)

    def add_inplace(self, x, y):
        library().oracle_add_inplace(_ptr(x), _ptr(y), x.size)

    def lm_head_int4(self, weights, scales, values, out, width):
        # The non-ARM fallback of cpu_lightspark.py:361-366: quantise, then GEMV.
        quantized = np.empty(width, dtype=np.int8)
        scale = self.quantize_activation(np.ascontiguousarray(values, dtype=np.float32), quantized)
        library().oracle_int4_i8_gemv(_ptr(quantized), _ptr(weights), _ptr(scales), scale, _ptr(out),
                                      weights.shape[0], width)

    def max_threads(self):
        return max_threads()


def configure_threads(threads: int | None = None) -> int:
    """OMP settings as cpu_lightspark.configure_threads (cpu_lightspark.py:38-42);
    must run before the library is first loaded to take effect."""
    threads = threads or os.cpu_count() or 1
    os.environ["OMP_NUM_THREADS"] = str(threads)
    os.environ.setdefault("OMP_WAIT_POLICY", "ACTIVE")
    return threads


from .model import OracleLayer, OracleProjection, OracleQwen, OracleState, sample_logits  # noqa: E402

__all__ = [
    "OracleKernel", "OracleLayer", "OracleProjection", "OracleQwen", "OracleState", "build",
    "configure_threads", "exp", "gqa_decode", "gqa_splitk", "int4_gemv", "int4_gemv_function", "library", "max_threads",
    "quantize_activation", "sample_logits",
]
