"""Batched decode (h4b_decode_batch): each sequence of the batch must get
the logits the oracle's single-token decode gives it, bit for bit, with the
same attention splits; the device greedy loop must feed its own tokens."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from _models import oracle_model  # noqa: E402
from harsh4b_b200.model import CudaQwen  # noqa: E402
from harsh4b_b200.synthetic import qwen3_4b_config, synthetic_checkpoint, synthetic_prompt, tiny_config  # noqa: E402


def _batch_decode(model, prompts, steps, splits):
    B, n = len(prompts), len(prompts[0])
    state = model.new_batch_state(B, n + steps, attn_splits=splits, attention="exact")
    rows = []
    for i in range(n):
        rows.append(model.forward_batch([p[i] for p in prompts], state).cpu().numpy().copy())
    greedy = []
    for _ in range(steps):
        tokens = rows[-1].argmax(axis=1)
        greedy.append(tokens)
        rows.append(model.forward_batch(tokens, state).cpu().numpy().copy())
    return np.stack(rows, axis=1), np.stack(greedy, axis=1), state


def _oracle_seq(reference, prompt, steps):
    state = reference.new_state(len(prompt) + steps)
    out = [reference.forward_token(int(t), state).copy() for t in prompt]
    greedy = []
    for _ in range(steps):
        greedy.append(int(np.argmax(out[-1])))
        out.append(reference.forward_token(greedy[-1], state).copy())
    return np.stack(out), greedy


@pytest.mark.parametrize("kv_dtype", ["float32", "float16"])
@pytest.mark.parametrize("splits", [1, 3, 16])
def test_tiny_batch_bit_exact_per_sequence(kv_dtype, splits):
    checkpoint = synthetic_checkpoint(tiny_config(), seed=21)
    prompts = [synthetic_prompt(checkpoint.config, 12, seed=s) for s in range(3)]
    model = CudaQwen.from_checkpoint(checkpoint, kv_dtype=kv_dtype)
    reference = oracle_model(checkpoint, kv_dtype=np.float32 if kv_dtype == "float32" else np.float16,
                             attn_splits=splits)
    logits, greedy, _ = _batch_decode(model, prompts, 8, splits)
    for b, prompt in enumerate(prompts):
        want, want_greedy = _oracle_seq(reference, prompt, 8)
        np.testing.assert_array_equal(logits[b], want)
        assert list(greedy[b]) == want_greedy
    assert model.status() == 0


def test_qwen_shaped_batch_matches_oracle_and_device_loop():
    config = qwen3_4b_config(num_hidden_layers=2)
    checkpoint = synthetic_checkpoint(config, seed=4)
    prompts = [synthetic_prompt(config, 6, seed=10 + s) for s in range(4)]
    model = CudaQwen.from_checkpoint(checkpoint, kv_dtype="float16")
    reference = oracle_model(checkpoint, kv_dtype=np.float16, attn_splits=16)
    logits, greedy, state = _batch_decode(model, prompts, 3, 16)
    for b, prompt in enumerate(prompts):
        want, want_greedy = _oracle_seq(reference, prompt, 3)
        np.testing.assert_array_equal(logits[b], want)
        assert list(greedy[b]) == want_greedy
    # device-side greedy loop from the same point: 2 more tokens
    fresh = model.new_batch_state(4, 16, attn_splits=16, attention="exact")
    for i in range(6):
        model.forward_batch([p[i] for p in prompts], fresh)
    model.generate_batch(fresh, 3)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(fresh.positions.cpu().numpy(), np.full(4, 9))
    with pytest.raises(ValueError):
        model.forward_batch([0, 1], fresh)


@pytest.mark.parametrize("attention", ["exact", "tensor"])
def test_graph_replayed_steps_equal_eager_launches(attention):
    """CudaBatchState.step replays a CUDA graph from the second step on: the
    same kernels as launching h4b_decode_batch eagerly, so the same bits."""
    import ctypes

    from harsh4b_b200._lib import check, lib

    config = tiny_config(num_hidden_layers=2)
    model = CudaQwen.from_checkpoint(synthetic_checkpoint(config, seed=71), kv_dtype="float16")
    prompts = [synthetic_prompt(config, 9, seed=s) for s in range(3)]
    graphed = model.new_batch_state(3, 32, attn_splits=2, attention=attention)
    eager = model.new_batch_state(3, 32, attn_splits=2, attention=attention)
    stream = torch.cuda.current_stream().cuda_stream
    for i in range(len(prompts[0])):
        ids = [p[i] for p in prompts]
        a = model.forward_batch(ids, graphed).cpu().numpy().copy()
        eager.tokens.copy_(torch.tensor(ids, dtype=torch.int32))
        check(lib().h4b_decode_batch(ctypes.byref(model.desc), ctypes.byref(eager.desc), stream), "h4b_decode_batch")
        np.testing.assert_array_equal(a, eager.logits.cpu().numpy())
    assert graphed._graph is not None
    model.generate_batch(graphed, 4)
    for _ in range(4):
        check(lib().h4b_decode_batch(ctypes.byref(model.desc), ctypes.byref(eager.desc), stream), "h4b_decode_batch")
    torch.cuda.synchronize()
    np.testing.assert_array_equal(graphed.logits.cpu().numpy(), eager.logits.cpu().numpy())
    np.testing.assert_array_equal(graphed.next_tokens.cpu().numpy(), eager.next_tokens.cpu().numpy())
    assert model.status() == 0
