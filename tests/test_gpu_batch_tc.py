"""Tensor-core batched-decode attention (decode_tc.cu, attention="tensor" on
a CudaBatchState): keys-as-M tcgen05 MMAs with split fp16 operands, held to
the tolerance contract:

* kernel level: every sequence's attention output for one batched step,
  each sequence at its own context (1 to 400 keys: one tile, tile edges,
  several tiles, splits with no keys), against an fp64 restatement over the
  same normalised q rows and fp16 caches, within 1e-3 relative (measured
  ~1e-6), also with NaN / inf cache entries past the contexts;
* model level (Qwen3-4B shapes, 2 layers): identical greedy tokens against
  the exact batched decode, logits as close as a change of the exact
  kernel's split count puts them."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from harsh4b_b200.model import CudaQwen  # noqa: E402
from harsh4b_b200.synthetic import qwen3_4b_config, synthetic_checkpoint, synthetic_prompt, tiny_config  # noqa: E402

REL_TOL = 1e-3
LOGIT_TOL = 1e-2
POSITIONS = [0, 63, 127, 128, 200, 399]


def _one_layer_model(seed):
    checkpoint = synthetic_checkpoint(tiny_config(num_hidden_layers=1), seed=seed)
    return CudaQwen.from_checkpoint(checkpoint, kv_dtype="float16", mode="chain")


def _step(model, attention, splits, fill_tail=None):
    """One batched step with every sequence at its own position over caches
    of N(0, 1) values; returns the attention rows, the q rows and the caches."""
    B, cap = len(POSITIONS), 400
    state = model.new_batch_state(B, cap, attn_splits=splits, attention=attention)
    gen = torch.Generator(device="cpu").manual_seed(5)
    for cache in (state.k_cache, state.v_cache):
        cache.copy_(torch.randn(cache.shape, generator=gen).to(cache.dtype))
    if fill_tail is not None:
        for b, p in enumerate(POSITIONS):
            state.k_cache[b, :, :, p + 1:] = float("nan")
            state.v_cache[b, :, :, p + 1:] = fill_tail
    state.positions.copy_(torch.tensor(POSITIONS, dtype=torch.int32))
    state.position[:] = POSITIONS
    model.forward_batch([(7 * b + 3) % model.vocab for b in range(B)], state)
    torch.cuda.synchronize()
    out = (state.attended.double().cpu().numpy(), state.qkv[:, :model.q_size].double().cpu().numpy(),
           state.k_cache[:, 0].double().cpu().numpy(), state.v_cache[:, 0].double().cpu().numpy())
    assert model.status() == 0
    return out


def _attention_fp64(model, q, k, v):
    d, G, KV = model.head_dim, model.groups, model.kv_heads
    out = np.zeros((len(POSITIONS), KV * G * d))
    for b, p in enumerate(POSITIONS):
        qb = q[b].reshape(KV * G, d)
        for head in range(KV * G):
            kk, vv = k[b, head // G, :p + 1], v[b, head // G, :p + 1]
            s = kk @ qb[head] / np.sqrt(d)
            w = np.exp(s - s.max())
            out[b, head * d:(head + 1) * d] = (w / w.sum()) @ vv
    return out


def _rel_err(got, want):
    scale = np.abs(want).reshape(len(POSITIONS), -1, 128).max(axis=2, keepdims=True)
    return float((np.abs(got - want).reshape(len(POSITIONS), -1, 128) / scale).max())


@pytest.mark.parametrize("splits", [1, 2, 3, 16])
def test_tensor_batch_attention_matches_fp64(splits):
    model = _one_layer_model(61)
    got, q, k, v = _step(model, "tensor", splits)
    err = _rel_err(got, _attention_fp64(model, q, k, v))
    print(f"splits {splits}: max relative error vs fp64 {err:.2e}")
    assert np.isfinite(got).all()
    assert err <= REL_TOL
    assert err < 1e-4
    exact, *_ = _step(model, "exact", splits)
    assert _rel_err(got, exact) <= REL_TOL


def test_tensor_batch_attention_ignores_non_finite_cache_past_the_context():
    model = _one_layer_model(62)
    for tail in (float("nan"), float("inf")):
        got, q, k, v = _step(model, "tensor", 3, fill_tail=tail)
        k = np.nan_to_num(k, nan=0.0, posinf=0.0)
        v = np.nan_to_num(v, nan=0.0, posinf=0.0)
        assert np.isfinite(got).all()
        assert _rel_err(got, _attention_fp64(model, q, k, v)) <= REL_TOL


def test_qwen_shaped_tensor_batch_decode_greedy_tokens():
    config = qwen3_4b_config(num_hidden_layers=2)
    checkpoint = synthetic_checkpoint(config, seed=12)
    model = CudaQwen.from_checkpoint(checkpoint, kv_dtype="float16")
    prompts = [synthetic_prompt(config, 150, seed=s) for s in range(4)]
    runs = {}
    for name, attention, splits in (("exact", "exact", 16), ("reordered", "exact", 3), ("tensor", "tensor", 2)):
        state = model.new_batch_state(4, 180, attn_splits=splits, attention=attention)
        for i in range(len(prompts[0])):
            logits = model.forward_batch([p[i] for p in prompts], state)
        rows, tokens = [logits.cpu().numpy().copy()], []
        for _ in range(12):
            tokens.append(rows[-1].argmax(axis=1).tolist())
            rows.append(model.forward_batch(tokens[-1], state).cpu().numpy().copy())
        runs[name] = (np.stack(rows), tokens)
    drift = np.abs(runs["tensor"][0] - runs["exact"][0]).max()
    reorder = np.abs(runs["reordered"][0] - runs["exact"][0]).max()
    print(f"batched logits max-abs vs exact: tensor {drift:.3e}, exact with 3 splits {reorder:.3e}")
    assert runs["tensor"][1] == runs["exact"][1]
    assert drift <= max(LOGIT_TOL, 2 * reorder)
    assert model.status() == 0


def test_unknown_batch_attention_rejected():
    model = _one_layer_model(63)
    with pytest.raises(ValueError):
        model.new_batch_state(2, 16, attention="fast")
