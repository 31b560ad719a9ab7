"""Operator-level wrappers over the C ABI, on torch CUDA tensors.

Each function mirrors one call the reference's CPU path makes (the C ABI
declarations in include/harsh4b_b200.h cite the reference lines). Inputs
must already be CUDA tensors; nothing here copies to or from the host.
"""
from __future__ import annotations

import torch

from ._lib import check, lib, stream_handle


def _dev(tensor: torch.Tensor, dtype: torch.dtype, name: str) -> int:
    if not isinstance(tensor, torch.Tensor) or not tensor.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if tensor.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {tensor.dtype}")
    if not tensor.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return tensor.data_ptr()


def int4_i8_gemv(x8: torch.Tensor, weights: torch.Tensor, scales: torch.Tensor, activation_scale: float,
                 *, out: torch.Tensor | None = None, acc: torch.Tensor | None = None):
    """litespark_int4_i8_gemv on the GPU: returns (fp32 out[rows], int32 acc[rows] or None)."""
    rows, packed = weights.shape
    out = torch.empty(rows, dtype=torch.float32, device=weights.device) if out is None else out
    check(lib().h4b_int4_i8_gemv(_dev(x8, torch.int8, "x8"), _dev(weights, torch.uint8, "weights"),
                                 _dev(scales, torch.float32, "scales"), float(activation_scale),
                                 _dev(out, torch.float32, "out"),
                                 _dev(acc, torch.int32, "acc") if acc is not None else None,
                                 rows, 2 * packed, stream_handle()), "h4b_int4_i8_gemv")
    return out, acc


def int4_gemv_fused_quant(values: torch.Tensor, weights: torch.Tensor, scales: torch.Tensor,
                          *, out: torch.Tensor | None = None, acc: torch.Tensor | None = None,
                          scale: torch.Tensor | None = None, pdl: bool = False):
    """quantize_activation + int4 GEMV in one kernel: returns (out, acc, act_scale tensor[1]).
    pdl=True launches with programmatic dependent launch (H4B_LAUNCH_PDL)."""
    rows, packed = weights.shape
    out = torch.empty(rows, dtype=torch.float32, device=weights.device) if out is None else out
    scale = torch.empty(1, dtype=torch.float32, device=weights.device) if scale is None else scale
    check(lib().h4b_int4_gemv_fused_quant_ex(_dev(values, torch.float32, "values"),
                                             _dev(weights, torch.uint8, "weights"),
                                             _dev(scales, torch.float32, "scales"), _dev(out, torch.float32, "out"),
                                             _dev(acc, torch.int32, "acc") if acc is not None else None,
                                             _dev(scale, torch.float32, "scale"), rows, 2 * packed,
                                             1 if pdl else 0, stream_handle()),
          "h4b_int4_gemv_fused_quant_ex")
    return out, acc, scale


def quantize_activation(values: torch.Tensor, quantized: torch.Tensor | None = None):
    """Returns (int8 tensor, dequant scale tensor[1])."""
    quantized = torch.empty(values.numel(), dtype=torch.int8, device=values.device) if quantized is None else quantized
    if quantized.numel() < values.numel():
        raise ValueError("int8 output buffer is smaller than the activation")
    scale = torch.empty(1, dtype=torch.float32, device=values.device)
    check(lib().h4b_quantize_activation(_dev(values, torch.float32, "values"),
                                        _dev(quantized, torch.int8, "quantized"), scale.data_ptr(),
                                        values.numel(), stream_handle()), "h4b_quantize_activation")
    return quantized, scale


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    out = torch.empty_like(x) if out is None else out
    check(lib().h4b_rmsnorm(_dev(x, torch.float32, "x"), _dev(weight, torch.float32, "weight"),
                            _dev(out, torch.float32, "out"), x.numel(), float(eps), stream_handle()), "h4b_rmsnorm")
    return out


def add_inplace(x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    check(lib().h4b_add_inplace(_dev(x, torch.float32, "x"), _dev(y, torch.float32, "y"), x.numel(),
                                stream_handle()), "h4b_add_inplace")
    return x


def gqa_decode(query: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, context: int,
               kv_heads: int, groups: int, *, scores: torch.Tensor | None = None,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """litespark_gqa_decode on the GPU; keys/values fp32 [capacity, kv_heads, head_dim]."""
    capacity, _, head_dim = keys.shape
    q_heads = kv_heads * groups
    scores = torch.empty(q_heads * capacity, dtype=torch.float32, device=query.device) if scores is None else scores
    out = torch.empty(q_heads, head_dim, dtype=torch.float32, device=query.device) if out is None else out
    check(lib().h4b_gqa_decode(_dev(query, torch.float32, "query"), _dev(keys, torch.float32, "keys"),
                               _dev(values, torch.float32, "values"), _dev(scores, torch.float32, "scores"),
                               _dev(out, torch.float32, "out"), context, kv_heads, groups, head_dim, capacity,
                               stream_handle()), "h4b_gqa_decode")
    return out


def gqa_decode_noalloc(query: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, context: int,
                       kv_heads: int, groups: int, *, out: torch.Tensor | None = None) -> torch.Tensor:
    """gqa_decode without a scratch buffer, for callers that cannot allocate
    device memory when attention runs (see h4b_gqa_decode_noalloc in
    include/harsh4b_b200.h): the split partials live in a fixed 1 MiB array
    inside the library, so concurrent calls on different streams race."""
    head_dim = keys.shape[-1]
    if out is None:
        raise ValueError("gqa_decode_noalloc allocates nothing: pass `out` (q_heads x head_dim fp32)")
    check(lib().h4b_gqa_decode_noalloc(_dev(query, torch.float32, "query"), _dev(keys, torch.float32, "keys"),
                                       _dev(values, torch.float32, "values"), _dev(out, torch.float32, "out"),
                                       context, kv_heads, groups, head_dim, stream_handle()),
          "h4b_gqa_decode_noalloc")
    return out


def embedding(token: torch.Tensor, table: torch.Tensor, scales: torch.Tensor,
              out: torch.Tensor | None = None) -> torch.Tensor:
    vocab, packed = table.shape
    out = torch.empty(2 * packed, dtype=torch.float32, device=table.device) if out is None else out
    check(lib().h4b_embedding(_dev(token, torch.int32, "token"), _dev(table, torch.uint8, "table"),
                              _dev(scales, torch.float32, "scales"), _dev(out, torch.float32, "out"), vocab,
                              2 * packed, stream_handle()), "h4b_embedding")
    return out


def argmax(logits: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    out = torch.empty(1, dtype=torch.int32, device=logits.device) if out is None else out
    check(lib().h4b_argmax(_dev(logits, torch.float32, "logits"), logits.numel(), _dev(out, torch.int32, "out"),
                           stream_handle()), "h4b_argmax")
    return out


def sample(logits: torch.Tensor, generated: torch.Tensor | None, uniform: float, *, temperature: float = 0.7,
           top_k: int = 50, top_p: float = 0.9, repetition_penalty: float = 1.15, out: torch.Tensor | None = None,
           scratch: torch.Tensor | None = None, return_candidates: bool = False):
    """h4b_sample: one token from fp32 logits (penalised IN PLACE) on the GPU.
    `generated` holds distinct int32 ids (or None); `uniform` is a draw in
    [0, 1) from the caller's generator. Returns the int32 token tensor[1]
    (and the candidate ids / probabilities when asked)."""
    vocab = logits.numel()
    out = torch.empty(1, dtype=torch.int32, device=logits.device) if out is None else out
    k = min(top_k if top_k > 0 else 50, vocab)
    if scratch is None:
        nbytes = int(lib().h4b_sample_scratch_bytes(vocab, top_k))
        if nbytes < 0:
            check(nbytes, "h4b_sample_scratch_bytes")
        scratch = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=logits.device)
    ids = torch.empty(k, dtype=torch.int32, device=logits.device) if return_candidates else None
    probs = torch.empty(k, dtype=torch.float32, device=logits.device) if return_candidates else None
    n_gen = 0 if generated is None else generated.numel()
    check(lib().h4b_sample(_dev(logits, torch.float32, "logits"), vocab,
                           _dev(generated, torch.int32, "generated") if n_gen else None, n_gen, float(temperature),
                           int(top_k), float(top_p), float(repetition_penalty), float(uniform),
                           _dev(out, torch.int32, "out"), ids.data_ptr() if ids is not None else None,
                           probs.data_ptr() if probs is not None else None, scratch.data_ptr(), stream_handle()),
          "h4b_sample")
    return (out, ids, probs) if return_candidates else out


def quantize_rows(values: torch.Tensor):
    """Per-token int8 quantisation of fp32 [M, K]: returns (x8, scales[M], sums[M])."""
    rows, width = values.shape
    x8 = torch.empty(rows, width, dtype=torch.int8, device=values.device)
    scales = torch.empty(rows, dtype=torch.float32, device=values.device)
    sums = torch.empty(rows, dtype=torch.int32, device=values.device)
    check(lib().h4b_quantize_rows(_dev(values, torch.float32, "values"), x8.data_ptr(), scales.data_ptr(),
                                  sums.data_ptr(), rows, width, stream_handle()), "h4b_quantize_rows")
    return x8, scales, sums


GEMM_KERNELS = {"auto": 0, "tcgen05": 1, "mma_sync": 2}


def int4_gemm(x8: torch.Tensor, act_scales: torch.Tensor, act_sums: torch.Tensor, weights: torch.Tensor,
              scales: torch.Tensor, out: torch.Tensor | None = None, kernel: str = "auto") -> torch.Tensor:
    """h4b_int4_gemm_ex: fp32 [M, N] from int8 activations [M, K] and int4
    weights [N, K/2]; `kernel` picks tcgen05, mma.sync or the automatic choice."""
    tokens, width = x8.shape
    rows = weights.shape[0]
    out = torch.empty(tokens, rows, dtype=torch.float32, device=x8.device) if out is None else out
    check(lib().h4b_int4_gemm_ex(_dev(x8, torch.int8, "x8"), _dev(act_scales, torch.float32, "act_scales"),
                                 _dev(act_sums, torch.int32, "act_sums"), _dev(weights, torch.uint8, "weights"),
                                 _dev(scales, torch.float32, "scales"), _dev(out, torch.float32, "out"), tokens,
                                 rows, width, GEMM_KERNELS[kernel], stream_handle()), "h4b_int4_gemm_ex")
    return out


def int4_gemm_acc(x8: torch.Tensor, act_scales: torch.Tensor, act_sums: torch.Tensor, weights: torch.Tensor,
                  scales: torch.Tensor, acc: torch.Tensor, out: torch.Tensor | None = None,
                  residual: bool = False) -> torch.Tensor:
    """h4b_int4_gemm_acc: int4_gemm with the K sum split over CTAs through the
    zeroed int32 buffer `acc` [M, N] (left zero); `residual` adds into `out`."""
    tokens, width = x8.shape
    rows = weights.shape[0]
    if residual and out is None:
        raise ValueError("residual needs out")
    if acc.numel() < tokens * rows:
        raise ValueError(f"acc holds {acc.numel()} int32, needs {tokens * rows}")
    out = torch.empty(tokens, rows, dtype=torch.float32, device=x8.device) if out is None else out
    check(lib().h4b_int4_gemm_acc(_dev(x8, torch.int8, "x8"), _dev(act_scales, torch.float32, "act_scales"),
                                  _dev(act_sums, torch.int32, "act_sums"), _dev(weights, torch.uint8, "weights"),
                                  _dev(scales, torch.float32, "scales"), _dev(out, torch.float32, "out"),
                                  _dev(acc, torch.int32, "acc"), tokens, rows, width, 1 if residual else 0,
                                  stream_handle()), "h4b_int4_gemm_acc")
    return out


def int4_gemm_rows(values: torch.Tensor, weights: torch.Tensor, scales: torch.Tensor,
                   kernel: str = "auto") -> torch.Tensor:
    """fp32 [M, K] -> fp32 [M, N]: per-token quantisation, then the batched GEMM."""
    x8, act_scales, sums = quantize_rows(values)
    return int4_gemm(x8, act_scales, sums, weights, scales, kernel=kernel)


def int4_gemv_absmax(values: torch.Tensor, absmax: torch.Tensor, weights: torch.Tensor, scales: torch.Tensor,
                     acc: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Quantise with a given device absmax, GEMV, int32 row sums into `acc`."""
    rows, packed = weights.shape
    check(lib().h4b_int4_gemv_absmax(_dev(values, torch.float32, "values"), _dev(absmax, torch.float32, "absmax"),
                                     _dev(weights, torch.uint8, "weights"), _dev(scales, torch.float32, "scales"),
                                     _dev(out, torch.float32, "out") if out is not None else None,
                                     _dev(acc, torch.int32, "acc"), rows, 2 * packed, stream_handle()),
          "h4b_int4_gemv_absmax")
    return acc


def residual_acc(x: torch.Tensor, acc: torch.Tensor, absmax: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """x += float(acc) * dequant(absmax) * scales (in place)."""
    check(lib().h4b_residual_acc(_dev(x, torch.float32, "x"), _dev(acc, torch.int32, "acc"),
                                 _dev(absmax, torch.float32, "absmax"), _dev(scales, torch.float32, "scales"),
                                 x.numel(), stream_handle()), "h4b_residual_acc")
    return x
