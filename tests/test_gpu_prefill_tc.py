"""Tensor-core prefill attention (prefill_tc.cu, attention="tensor"): the
tcgen05 kernel with split fp16 operands, held to the tolerance contract
instead of bit equality:

* kernel level: every prompt row's attention output against an fp64
  restatement of causal GQA softmax attention over the same q rows and the
  same fp16 cache, within 1e-3 relative (measured ~1e-6), for ragged prompt
  lengths, a prompt that continues an earlier context, a prompt that ends at
  the state's capacity, and non-finite cache entries past the context;
* model level (Qwen3-4B shapes, 2 layers): logits within 1e-2 max-abs of the
  exact (decode-order) prefill and identical greedy tokens over the decode
  that follows."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from harsh4b_b200.model import CudaQwen  # noqa: E402
from harsh4b_b200.synthetic import qwen3_4b_config, synthetic_checkpoint, synthetic_prompt, tiny_config  # noqa: E402

REL_TOL = 1e-3   # fp32 attention outputs, relative to the row's largest magnitude
LOGIT_TOL = 1e-2  # final logits, max-abs


def _attention_fp64(model, scratch, state, count, p0):
    """Causal GQA attention of layer 0 in fp64 from the q rows the prefill
    normalised and rotated in place (scratch.qkv) and the fp16 cache."""
    d, G, KV = model.head_dim, model.groups, model.kv_heads
    q = scratch.qkv[:count, :model.q_size].double().cpu().numpy().reshape(count, KV * G, d)
    k = state.k_cache[0].double().cpu().numpy()  # [kv_heads][capacity][d]
    v = state.v_cache[0].double().cpu().numpy()
    out = np.zeros((count, KV * G, d))
    for i in range(count):
        ctx = p0 + i + 1
        for head in range(KV * G):
            s = k[head // G, :ctx] @ q[i, head] / np.sqrt(d)
            w = np.exp(s - s.max())
            out[i, head] = (w / w.sum()) @ v[head // G, :ctx]
    return out.reshape(count, -1)


def _one_layer_model(seed):
    checkpoint = synthetic_checkpoint(tiny_config(num_hidden_layers=1), seed=seed)
    return CudaQwen.from_checkpoint(checkpoint, kv_dtype="float16", mode="chain")


def _check_rows(got, want):
    scale = np.abs(want).max(axis=1, keepdims=True)
    rel = np.abs(got - want) / scale
    assert np.isfinite(got).all()
    assert rel.max() <= REL_TOL, rel.max()
    return float(rel.max())


@pytest.mark.parametrize("count", [1, 31, 32, 33, 64, 65, 127, 200])
def test_tensor_attention_matches_fp64(count):
    model = _one_layer_model(51)
    prompt = synthetic_prompt(model.config, count, seed=count)
    state = model.new_state(256)
    model.prefill(prompt, state, attention="tensor")
    scratch = model._prefill_scratch
    got = scratch.attended[:count].double().cpu().numpy()
    err = _check_rows(got, _attention_fp64(model, scratch, state, count, 0))
    print(f"count {count}: max relative error vs fp64 {err:.2e}")
    # the exact kernel (fp32, decode order) sits as close to fp64
    exact_state = model.new_state(256)
    model.prefill(prompt, exact_state, attention="exact")
    exact = model._prefill_scratch.attended[:count].double().cpu().numpy()
    assert np.abs(got - exact).max() <= REL_TOL * np.abs(exact).max()
    assert err < 1e-4
    assert model.status() == 0
    state.close()
    exact_state.close()


def test_tensor_attention_continues_an_earlier_context():
    """A second prompt at position 70: its rows attend to the first one's keys."""
    model = _one_layer_model(52)
    first = synthetic_prompt(model.config, 70, seed=1)
    second = synthetic_prompt(model.config, 45, seed=2)
    state = model.new_state(200)
    model.prefill(first, state, attention="tensor")
    model.prefill(second, state, attention="tensor")
    assert state.position == 115
    scratch = model._prefill_scratch
    _check_rows(scratch.attended[:45].double().cpu().numpy(), _attention_fp64(model, scratch, state, 45, 70))
    assert model.status() == 0
    state.close()


def test_tensor_attention_at_capacity_and_non_finite_cache_tail():
    """The prompt ends exactly at a capacity that is not a multiple of the
    64-key tile (the TMA reads past it as zeros), and the cache entries past
    the context hold NaN / inf (never read into a sum)."""
    model = _one_layer_model(53)
    for capacity, count in ((100, 100), (300, 77)):
        state = model.new_state(capacity)
        state.k_cache.fill_(float("nan"))
        state.v_cache[:, :, ::2].fill_(float("nan"))
        state.v_cache[:, :, 1::2].fill_(float("inf"))
        prompt = synthetic_prompt(model.config, count, seed=capacity)
        model.prefill(prompt, state, attention="tensor")
        scratch = model._prefill_scratch
        _check_rows(scratch.attended[:count].double().cpu().numpy(),
                    _attention_fp64(model, scratch, state, count, 0))
        assert model.status() == 0
        state.close()


def test_tensor_prefill_chunks_match_one_pass_within_tolerance():
    model = _one_layer_model(54)
    prompt = synthetic_prompt(model.config, 150, seed=3)
    one = model.new_state(160)
    a = model.prefill(prompt, one, attention="tensor").cpu().numpy().copy()
    model._prefill_scratch = None
    chunked = model.new_state(160)
    b = model.prefill(prompt, chunked, max_tokens=40, attention="tensor").cpu().numpy().copy()
    assert np.abs(a - b).max() <= LOGIT_TOL
    one.close()
    chunked.close()


def test_qwen_shaped_tensor_prefill_logits_and_greedy_tokens():
    """Identical greedy tokens after the prefill, and logits as close to the
    exact prefill as a mere change of the exact kernel's summation order
    (one attention split against three) puts them: every int8 requantisation
    downstream turns 1e-6 differences into whole-code flips."""
    config = qwen3_4b_config(num_hidden_layers=2)
    checkpoint = synthetic_checkpoint(config, seed=8)
    model = CudaQwen.from_checkpoint(checkpoint, kv_dtype="float16", mode="persistent")
    prompt = synthetic_prompt(config, 300, seed=9)
    runs = {}
    for name, attention, splits in (("exact", "exact", 1), ("reordered", "exact", 3), ("tensor", "tensor", 1)):
        state = model.new_state(len(prompt) + 16)
        last = model.prefill(prompt, state, attention=attention, attn_splits=splits).cpu().numpy().copy()
        tokens = [int(np.argmax(last))]
        for _ in range(12):
            tokens.append(int(np.argmax(model.forward_token(tokens[-1], state).cpu().numpy())))
        runs[name] = (last, tokens)
        state.close()
    drift = np.abs(runs["tensor"][0] - runs["exact"][0]).max()
    reorder = np.abs(runs["reordered"][0] - runs["exact"][0]).max()
    print(f"prefill logits max-abs vs exact: tensor {drift:.3e}, exact with 3 splits {reorder:.3e}")
    assert runs["tensor"][1] == runs["exact"][1]
    assert drift <= max(LOGIT_TOL, 2 * reorder)
    assert model.status() == 0


def test_unsupported_shapes_fall_back_to_the_exact_kernel():
    """An fp32 cache takes the exact kernel: attention="tensor" then leaves
    the same bits as attention="exact"."""
    checkpoint = synthetic_checkpoint(tiny_config(num_hidden_layers=1), seed=55)
    model = CudaQwen.from_checkpoint(checkpoint, kv_dtype="float32", mode="chain")
    prompt = synthetic_prompt(model.config, 40, seed=4)
    out = {}
    for attention in ("exact", "tensor"):
        state = model.new_state(64)
        out[attention] = model.prefill(prompt, state, attention=attention).cpu().numpy().copy()
        state.close()
    np.testing.assert_array_equal(out["tensor"], out["exact"])
    with pytest.raises(ValueError):
        model.prefill(prompt, model.new_state(64), attention="fast")


@pytest.mark.parametrize("attention", ["tensor", "exact"])
def test_prefill_attention_entry_repeats_the_layer(attention):
    """h4b_prefill_attention (the timing entry) recomputes the last layer's
    prompt attention from what the prefill left: the same bits."""
    import ctypes

    from harsh4b_b200._lib import check, lib

    model = _one_layer_model(56)
    prompt = synthetic_prompt(model.config, 97, seed=7)
    state = model.new_state(128)
    model.prefill(prompt, state, attention=attention)
    scratch = model._prefill_scratch
    first = scratch.attended[:97].clone()
    scratch.attended.zero_()
    check(lib().h4b_prefill_attention(ctypes.byref(model.desc), ctypes.byref(state.desc), ctypes.byref(scratch.desc),
                                      97, 0, state.stream.cuda_stream), "h4b_prefill_attention")
    torch.cuda.synchronize()
    assert torch.equal(scratch.attended[:97], first)
    assert lib().h4b_prefill_attention(ctypes.byref(model.desc), ctypes.byref(state.desc), ctypes.byref(scratch.desc),
                                       97, 1, state.stream.cuda_stream) != 0  # no layer 1
    assert model.status() == 0
    state.close()
