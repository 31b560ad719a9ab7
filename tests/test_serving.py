"""Continuous batching (harsh4b_b200.serving): requests that arrive while
others decode join free slots between steps, and every request's greedy
tokens equal a single-session decode of its own prompt (oracle with the same
attention splits: one per prompt query in the prefill, the batch's 16 in
decode). Stop ids, token limits and cancellation end a request and free its
slot."""
import threading

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _oracle_greedy(checkpoint, prompt, max_tokens, stop_ids):
    from _models import oracle_model

    n = len(prompt)
    model = oracle_model(checkpoint, kv_dtype=np.float16, attn_splits=lambda ctx: 1 if ctx <= n else 16)
    state = model.new_state(n + max_tokens + 1)
    for token in prompt:
        logits = model.forward_token(int(token), state)
    out = []
    while True:
        token = int(np.argmax(logits))
        if token in stop_ids:
            return out
        out.append(token)
        if len(out) >= max_tokens:
            return out
        logits = model.forward_token(token, state)


def _drain(request):
    tokens = []
    while True:
        kind, value = request.events.get(timeout=120)
        if kind == "token":
            tokens.append(value)
        elif kind == "error":
            raise RuntimeError(value)
        else:
            return tokens, value


def test_continuous_batching_matches_single_sessions():
    from harsh4b_b200.model import CudaQwen
    from harsh4b_b200.serving import ContinuousBatcher
    from harsh4b_b200.synthetic import synthetic_checkpoint, tiny_config

    checkpoint = synthetic_checkpoint(tiny_config(), seed=9)
    model = CudaQwen.from_checkpoint(checkpoint, kv_dtype="float16")
    rng = np.random.default_rng(9)
    jobs = [([int(t) for t in rng.integers(0, 2048, n)], m) for n, m in
            [(5, 12), (17, 3), (9, 20), (30, 7), (3, 15), (12, 9), (21, 11)]]
    # a stop id that the greedy decode of job 2 emits part-way
    probe = _oracle_greedy(checkpoint, *jobs[2], stop_ids=set())
    stop_ids = {probe[6]}
    engine = ContinuousBatcher(model, slots=3, capacity=64, stop_ids=stop_ids, attention="exact").start()
    try:
        requests = [engine.submit(prompt, limit, 0.0) for prompt, limit in jobs]
        results = [_drain(r) for r in requests]
    finally:
        engine.close()
    for (prompt, limit), (tokens, stats) in zip(jobs, results):
        assert tokens == _oracle_greedy(checkpoint, prompt, limit, stop_ids)
        assert stats["tokens"] == len(tokens)
    assert len(results[2][0]) < jobs[2][1]  # the stop id ended it early
    assert {r.slot for r in requests} == {0, 1, 2}  # later requests reused freed slots
    assert engine.steps < sum(len(t) for t, _ in results)  # tokens of several requests per step
    assert model.status() == 0


def test_batched_backend_streams_concurrent_requests_and_cancels():
    from harsh4b_b200.model import CudaQwen
    from harsh4b_b200.serving import BatchedCudaBackend
    from harsh4b_b200.synthetic import synthetic_checkpoint, tiny_config
    from test_runtime import _Tokenizer

    checkpoint = synthetic_checkpoint(tiny_config(), seed=9)
    model = CudaQwen.from_checkpoint(checkpoint, kv_dtype="float16")
    backend = BatchedCudaBackend(model=model, tokenizer=_Tokenizer(model.vocab, stop_ids=()), slots=4, capacity=128)
    outputs, errors = {}, []
    cancel = threading.Event()

    def client(name, prompt, limit, stopped=lambda: False):
        try:
            outputs[name] = list(backend.stream(prompt, limit, 0.0, stopped))
        except Exception as exc:  # pragma: no cover - reported below
            errors.append(exc)

    threads = [threading.Thread(target=client, args=(f"r{i}", list(range(i + 2, i + 12)), 16)) for i in range(6)]
    threads.append(threading.Thread(target=client, args=("cancelled", list(range(40)), 60, cancel.is_set)))
    for t in threads:
        t.start()
    cancel.set()
    for t in threads:
        t.join(timeout=300)
    backend.close()
    assert not errors
    for i in range(6):
        events = outputs[f"r{i}"]
        stats = events[-1]["stats"]
        assert events[-1]["done"] and stats["tokens"] == 16 and stats["runtime"] == "cuda"
        want = _oracle_greedy(checkpoint, list(range(i + 2, i + 12)), 16, set())
        text = "".join(e["token"] for e in events[:-1])
        assert text.split() == [f"t{t}" for t in want]
    assert outputs["cancelled"][-1]["stats"]["tokens"] < 60
