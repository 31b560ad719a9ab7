"""Runtime contract (inference_runtime.py:71-122): the backend-independent
stream() logic on CPU with a scripted backend, and CudaRuntime on the GPU."""
import numpy as np
import pytest

tokenizers = pytest.importorskip("tokenizers")

from harsh4b_b200.runtime import Runtime  # noqa: E402


class _Tokenizer:
    """ChatTokenizer stand-in: a word-level vocabulary t0..t{n-1}."""

    def __init__(self, vocab: int, stop_ids=(3,)):
        from tokenizers import Tokenizer, models, pre_tokenizers

        words = {f"t{i}": i for i in range(vocab)}
        self.backend = Tokenizer(models.WordLevel(words, unk_token="t0"))
        self.backend.pre_tokenizer = pre_tokenizers.Whitespace()
        self.stop_ids = set(stop_ids)


class _Scripted(Runtime):
    device, hardware, description = "cpu", "test", "scripted"

    def __init__(self, script):
        self.script, self.tokenizer, self.calls = list(script), _Tokenizer(16), []

    def prefill(self, ids, max_tokens):
        self.calls.append(("prefill", list(ids), max_tokens))
        return None, {"pos": len(ids)}

    def decode(self, token, session):
        self.calls.append(("decode", token))
        session["pos"] += 1
        return None

    def sample(self, logits, generated, temperature):
        return self.script.pop(0)


def test_stream_stops_at_stop_token_and_counts_steps():
    rt = _Scripted([5, 6, 3])
    events = list(rt.stream([1, 2], max_tokens=10, temperature=0.7))
    assert events[-1]["done"] and events[-1]["stats"]["tokens"] == 2
    assert events[-1]["stats"]["decode_steps"] == 2
    assert [c[0] for c in rt.calls] == ["prefill", "decode", "decode"]


def test_stream_no_forward_after_last_token():
    rt = _Scripted([5, 6, 7, 8])
    events = list(rt.stream([1], max_tokens=2, temperature=0.7))
    assert events[-1]["stats"]["tokens"] == 2
    assert [c[0] for c in rt.calls] == ["prefill", "decode"]


def test_stream_rejects_oversized_requests():
    rt = _Scripted([])
    with pytest.raises(ValueError):
        list(rt.stream([1] * 2000, max_tokens=100, temperature=0.7))
    with pytest.raises(ValueError):
        list(rt.stream([], max_tokens=1, temperature=0.7))


@pytest.mark.gpu
def test_cuda_runtime_matches_oracle_greedy_and_sampled():
    import torch

    from harsh4b_b200.model import CudaQwen
    from harsh4b_b200.runtime import CudaRuntime
    from harsh4b_b200.synthetic import synthetic_checkpoint, synthetic_prompt, tiny_config
    from oracle.model import sample_runtime
    from _models import oracle_model

    checkpoint = synthetic_checkpoint(tiny_config(), seed=3)
    prompt = synthetic_prompt(checkpoint.config, 10, seed=3)
    model = CudaQwen.from_checkpoint(checkpoint, kv_dtype="float32")
    # the prompt goes through one prefill pass (one split per query), later
    # tokens through the persistent step (its per-context rule)
    decode_rule, n = model.attention_split_rule(), len(prompt)
    reference = oracle_model(checkpoint, kv_dtype=np.float32,
                             attn_splits=lambda ctx: 1 if ctx <= n else decode_rule(ctx))
    for temperature in (0.0, 0.7):
        rt = CudaRuntime(model=model, tokenizer=_Tokenizer(model.vocab), seed=11)
        draws = np.random.default_rng(11)
        logits, session = rt.prefill(prompt, 12)
        state = reference.new_state(len(prompt) + 12)
        for token in prompt:
            want_logits = reference.forward_token(int(token), state)
        np.testing.assert_array_equal(logits.cpu().numpy(), want_logits)
        generated = []
        for _ in range(10):
            token = rt.sample(logits, generated, temperature)
            uniform = float(draws.random()) if temperature > 0.01 else 0.0
            want, _, probs = sample_runtime(want_logits, generated, uniform, temperature=temperature,
                                            return_candidates=True)
            if token != want:  # only a last-ulp exp difference at a CDF boundary may flip a draw
                cdf = probs.astype(np.float64).cumsum() / probs.astype(np.float64).sum()
                assert np.min(np.abs(cdf - uniform)) < 1e-6
                break
            generated.append(token)
            logits = rt.decode(token, session)
            want_logits = reference.forward_token(token, state)
        assert rt.status()["ready"] and rt.memory_gib() > 0
    events = list(CudaRuntime(model=model, tokenizer=_Tokenizer(model.vocab), seed=1).stream(prompt, 8, 0.7))
    assert events[-1]["done"] and events[-1]["stats"]["tokens"] <= 8
    torch.cuda.synchronize()
