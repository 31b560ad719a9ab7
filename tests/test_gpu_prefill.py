"""Prefill (h4b_prefill / CudaQwen.prefill): a prompt fed in one pass through
the batched GEMMs must leave the session exactly where feeding it token by
token leaves it -- the last prompt row's logits and every later decode
token equal the oracle's bit for bit, with the oracle told the attention
split count each token used."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from _models import oracle_model  # noqa: E402
from harsh4b_b200.model import CudaQwen  # noqa: E402
from harsh4b_b200.synthetic import qwen3_4b_config, synthetic_checkpoint, synthetic_prompt, tiny_config  # noqa: E402


def _oracle_run(reference, prompt, steps):
    state = reference.new_state(len(prompt) + steps)
    out = [reference.forward_token(int(t), state).copy() for t in prompt]
    last, greedy, after = out[-1], [], []
    for _ in range(steps):
        greedy.append(int(np.argmax(out[-1])))
        out.append(reference.forward_token(greedy[-1], state).copy())
        after.append(out[-1])
    return last, greedy, np.stack(after) if after else None


def _cuda_run(model, prompt, steps, splits, max_tokens=2048, prefill_splits=None):
    state = model.new_state(len(prompt) + steps, attn_splits=splits)
    last = model.prefill(prompt, state, max_tokens=max_tokens, attention="exact",
                         attn_splits=splits if prefill_splits is None else prefill_splits).cpu().numpy().copy()
    assert state.position == len(prompt)
    greedy, after = [], []
    logits = last
    for _ in range(steps):
        greedy.append(int(np.argmax(logits)))
        logits = model.forward_token(greedy[-1], state).cpu().numpy().copy()
        after.append(logits)
    state.close()
    return last, greedy, np.stack(after) if after else None


@pytest.mark.parametrize("kv_dtype", ["float32", "float16"])
@pytest.mark.parametrize("splits", [1, 3, 16])
def test_tiny_prefill_then_chain_decode_bit_exact(kv_dtype, splits):
    checkpoint = synthetic_checkpoint(tiny_config(), seed=33)
    prompt = synthetic_prompt(checkpoint.config, 21, seed=5)
    model = CudaQwen.from_checkpoint(checkpoint, kv_dtype=kv_dtype, mode="chain", attn_splits=splits)
    reference = oracle_model(checkpoint, kv_dtype=np.float32 if kv_dtype == "float32" else np.float16,
                             attn_splits=splits)
    want_last, want_greedy, want_after = _oracle_run(reference, prompt, 6)
    got_last, got_greedy, got_after = _cuda_run(model, prompt, 6, splits)
    np.testing.assert_array_equal(got_last, want_last)
    assert got_greedy == want_greedy
    np.testing.assert_array_equal(got_after, want_after)
    assert model.status() == 0


def test_prefill_in_chunks_equals_one_pass():
    checkpoint = synthetic_checkpoint(tiny_config(), seed=34)
    prompt = synthetic_prompt(checkpoint.config, 23, seed=6)
    model = CudaQwen.from_checkpoint(checkpoint, kv_dtype="float16", mode="chain")
    one = _cuda_run(model, prompt, 3, 16)
    model._prefill_scratch = None
    chunked = _cuda_run(model, prompt, 3, 16, max_tokens=5)
    np.testing.assert_array_equal(one[0], chunked[0])
    assert one[1] == chunked[1]
    np.testing.assert_array_equal(one[2], chunked[2])


def test_prefill_then_persistent_decode():
    """The persistent step picks its split count per token; the prefill uses
    the state's fixed count. The oracle gets the same rule per context."""
    checkpoint = synthetic_checkpoint(tiny_config(), seed=35)
    prompt = synthetic_prompt(checkpoint.config, 40, seed=7)
    model = CudaQwen.from_checkpoint(checkpoint, kv_dtype="float16", mode="persistent")
    persistent = model.attention_split_rule()
    n = len(prompt)
    reference = oracle_model(checkpoint, kv_dtype=np.float16, attn_splits=lambda ctx: 1 if ctx <= n else persistent(ctx))
    want_last, want_greedy, want_after = _oracle_run(reference, prompt, 8)
    got_last, got_greedy, got_after = _cuda_run(model, prompt, 8, 16, prefill_splits=1)
    np.testing.assert_array_equal(got_last, want_last)
    assert got_greedy == want_greedy
    np.testing.assert_array_equal(got_after, want_after)
    assert model.status() == 0


@pytest.mark.parametrize("prefill_splits", [1, 2])
def test_prefill_split_count_independent_of_the_session(prefill_splits):
    """The prompt's queries use the prefill's split count, later tokens the
    session's: the oracle is told each."""
    checkpoint = synthetic_checkpoint(tiny_config(), seed=37)
    prompt = synthetic_prompt(checkpoint.config, 90, seed=8)
    model = CudaQwen.from_checkpoint(checkpoint, kv_dtype="float16", mode="chain")
    n = len(prompt)
    reference = oracle_model(checkpoint, kv_dtype=np.float16, attn_splits=lambda ctx: prefill_splits if ctx <= n else 5)
    want_last, want_greedy, want_after = _oracle_run(reference, prompt, 4)
    got_last, got_greedy, got_after = _cuda_run(model, prompt, 4, 5, prefill_splits=prefill_splits)
    np.testing.assert_array_equal(got_last, want_last)
    assert got_greedy == want_greedy
    np.testing.assert_array_equal(got_after, want_after)


def test_qwen_shaped_prefill_matches_oracle():
    config = qwen3_4b_config(num_hidden_layers=2)
    checkpoint = synthetic_checkpoint(config, seed=8)
    prompt = synthetic_prompt(config, 70, seed=9)
    model = CudaQwen.from_checkpoint(checkpoint, kv_dtype="float16", mode="chain")
    reference = oracle_model(checkpoint, kv_dtype=np.float16, attn_splits=16)
    want_last, want_greedy, want_after = _oracle_run(reference, prompt, 2)
    got_last, got_greedy, got_after = _cuda_run(model, prompt, 2, 16)
    np.testing.assert_array_equal(got_last, want_last)
    assert got_greedy == want_greedy
    np.testing.assert_array_equal(got_after, want_after)


def test_prefill_rejects_bad_input():
    checkpoint = synthetic_checkpoint(tiny_config(), seed=36)
    model = CudaQwen.from_checkpoint(checkpoint, mode="chain")
    state = model.new_state(8)
    with pytest.raises(ValueError):
        model.prefill([], state)
    with pytest.raises(ValueError):
        model.prefill([1] * 9, state)
    with pytest.raises(ValueError):
        model.prefill([model.vocab], state)
    model.prefill([1, 2, 3], state)
    with pytest.raises(ValueError):
        model.prefill([1] * 6, state)
    assert state.position == 3
    assert model.status() == 0
