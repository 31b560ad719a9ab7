"""The runtime boundary.

CPU (needs a checkout of the reference): the backend half composed with the
reference's own ``inference_runtime.Runtime`` drives its ``stream()``; the
documented edits to ``inference_runtime.py`` and ``test.py`` (tests/
reference_patches.py, applied to temporary copies) route ``"cuda"`` here.
The model there is the CPU oracle handed in through ``model=`` -- the
boundary is what is checked, not the kernels.

GPU: :class:`CudaBackend` with the CUDA model against the oracle, greedy and
sampled, and ``run_test_py`` (``test.py --runtime cuda``) end to end.
"""
import argparse
import importlib.util
import sys
from pathlib import Path

import numpy as np
import pytest

from conftest import REFERENCE_ROOT, reference_available

tokenizers = pytest.importorskip("tokenizers")
needs_reference = pytest.mark.skipif(not reference_available(), reason="needs the reference checkout")


class _Tokenizer:
    """ChatTokenizer stand-in: a word-level vocabulary t0..t{n-1}."""

    def __init__(self, vocab: int, stop_ids=(3,)):
        from tokenizers import Tokenizer, models, pre_tokenizers

        words = {f"t{i}": i for i in range(vocab)}
        self.backend = Tokenizer(models.WordLevel(words, unk_token="t0"))
        self.backend.pre_tokenizer = pre_tokenizers.Whitespace()
        self.stop_ids = set(stop_ids)


class _OracleModel:
    """The oracle behind the model surface CudaBackend calls (new_state,
    prefill, forward_token)."""

    device, mode, kv_dtype = "cpu", "oracle", "float32"

    def __init__(self, checkpoint):
        from _models import oracle_model

        self.inner = oracle_model(checkpoint)
        self.vocab = int(checkpoint.config["vocab_size"])

    def new_state(self, capacity):
        return self.inner.new_state(capacity)

    def prefill(self, ids, state):
        for token in ids:
            logits = self.inner.forward_token(int(token), state)
        return logits.copy()

    def forward_token(self, token, state):
        return self.inner.forward_token(int(token), state).copy()


def _import_file(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    module = importlib.util.module_from_spec(spec)
    sys.modules[name] = module
    spec.loader.exec_module(module)
    return module


@pytest.fixture
def reference_path():
    sys.path.insert(0, str(REFERENCE_ROOT))
    yield REFERENCE_ROOT
    sys.path.remove(str(REFERENCE_ROOT))


def _tiny():
    from harsh4b_b200.synthetic import synthetic_checkpoint, synthetic_prompt, tiny_config

    checkpoint = synthetic_checkpoint(tiny_config(), seed=3)
    return checkpoint, synthetic_prompt(checkpoint.config, 6, seed=3)


def _reference_sampler(reference_runtime, seed):
    """The reference's sample_numpy with its global numpy generator seeded."""
    np.random.seed(seed)
    drawn = []

    def sampler(logits, generated, temperature):
        token = reference_runtime.sample_numpy(np, np.asarray(logits), generated, temperature)
        drawn.append(token)
        return token

    return sampler, drawn


@needs_reference
def test_backend_composes_with_reference_runtime(reference_path):
    import inference_runtime

    from harsh4b_b200.runtime import CudaBackend

    class CudaRuntime(CudaBackend, inference_runtime.Runtime):
        pass

    # stream/status come from the reference, the backend methods from here
    assert CudaRuntime.stream is inference_runtime.Runtime.stream
    assert CudaRuntime.status is inference_runtime.Runtime.status
    for name in ("prefill", "decode", "sample", "memory_gib"):
        assert getattr(CudaRuntime, name) is getattr(CudaBackend, name)
    checkpoint, prompt = _tiny()
    model = _OracleModel(checkpoint)
    sampler, drawn = _reference_sampler(inference_runtime, 17)
    runtime = CudaRuntime(model=model, tokenizer=_Tokenizer(model.vocab), sampler=sampler)
    events = list(runtime.stream(prompt, 8, 0.7))
    stats = events[-1]["stats"]
    assert events[-1]["done"] and stats["runtime"] == "cuda" and stats["tokens"] <= 8
    assert runtime.status()["runtime"] == "cuda" and runtime.status()["ready"]
    # the same request through the reference's own CPU-runtime loop
    reference = _OracleModel(checkpoint)
    np.random.seed(17)
    state = reference.new_state(len(prompt) + 8)
    logits = reference.prefill(prompt, state)
    generated, want = [], []
    token = inference_runtime.sample_numpy(np, logits, generated, 0.7)
    while token not in runtime.tokenizer.stop_ids and len(generated) < 8:
        generated.append(token)
        if len(generated) >= 8:
            break
        logits = reference.forward_token(token, state)
        token = inference_runtime.sample_numpy(np, logits, generated, 0.7)
    assert drawn[:len(generated)] == generated
    assert stats["tokens"] == len(generated)


def _chat_tokenizer_file(path):
    """A tokenizer.json that the reference's ChatTokenizer accepts (Qwen3's
    special ids at their places, word-level otherwise)."""
    from tokenizers import Tokenizer, models, pre_tokenizers

    words = {f"t{i}": i for i in range(151936)}
    for word, index in (("<|endoftext|>", 151643), ("<|im_end|>", 151645)):
        del words[f"t{index}"]
        words[word] = index
    tokenizer = Tokenizer(models.WordLevel(words, unk_token="t0"))
    tokenizer.pre_tokenizer = pre_tokenizers.Whitespace()
    tokenizer.save(str(path))
    return path


@needs_reference
def test_create_runtime_routes_cuda_to_the_backend(reference_path, tmp_path):
    from reference_patches import INFERENCE_RUNTIME, apply

    patched = tmp_path / "inference_runtime_cuda.py"
    patched.write_text(apply((reference_path / "inference_runtime.py").read_text(), INFERENCE_RUNTIME))
    module = _import_file("inference_runtime_cuda", patched)
    checkpoint_file = tmp_path / "model.lat.pt"
    checkpoint_file.write_bytes(b"")
    tokenizer_file = _chat_tokenizer_file(tmp_path / "tokenizer.json")
    checkpoint, prompt = _tiny()
    sampler, _ = _reference_sampler(module, 5)
    runtime = module.create_runtime("cuda", model_path=checkpoint_file, tokenizer_path=tokenizer_file,
                                    model=_OracleModel(checkpoint), sampler=sampler)
    assert isinstance(runtime, module.CudaRuntime) and runtime.device == "cuda"
    assert runtime.tokenizer.stop_ids == {151643, 151645}
    events = list(runtime.stream(prompt, 5, 0.0))
    assert events[-1]["done"] and events[-1]["stats"]["tokens"] == 5


@needs_reference
def test_test_py_accepts_runtime_cuda(reference_path, tmp_path, monkeypatch):
    from reference_patches import TEST_PY, apply

    from harsh4b_b200 import cli

    patched = tmp_path / "test_py_cuda.py"
    patched.write_text(apply((reference_path / "test.py").read_text(), TEST_PY))
    module = _import_file("test_py_cuda", patched)
    model_file = tmp_path / "model.lat.pt"
    model_file.write_bytes(b"")
    monkeypatch.setattr(module, "MODEL_PATH", model_file)
    calls = []
    monkeypatch.setattr(cli, "run_test_py", lambda *a, **k: calls.append(a))
    monkeypatch.setattr(sys, "argv", ["test.py", "--runtime", "cuda", "--token-ids", "1,2,3",
                                      "--max-new-tokens", "4", "--temperature", "0"])
    module.main()
    (args, tokens, tokenizer, path), = calls
    assert args.runtime == "cuda" and tokens == [1, 2, 3] and tokenizer is None and path == model_file
    monkeypatch.setattr(sys, "argv", ["test.py", "--runtime", "tpu", "--token-ids", "1"])
    with pytest.raises(SystemExit):
        module.parse_args()


@pytest.mark.gpu
def test_cuda_backend_matches_oracle_greedy_and_sampled():
    import torch

    from _models import oracle_model
    from harsh4b_b200.model import CudaQwen
    from harsh4b_b200.runtime import CudaBackend
    from harsh4b_b200.synthetic import synthetic_checkpoint, synthetic_prompt, tiny_config
    from oracle.model import sample_runtime

    checkpoint = synthetic_checkpoint(tiny_config(), seed=3)
    prompt = synthetic_prompt(checkpoint.config, 10, seed=3)
    model = CudaQwen.from_checkpoint(checkpoint, kv_dtype="float32")
    # the prompt goes through one prefill pass (one split per query), later
    # tokens through the persistent step (its per-context rule)
    decode_rule, n = model.attention_split_rule(), len(prompt)
    reference = oracle_model(checkpoint, kv_dtype=np.float32,
                             attn_splits=lambda ctx: 1 if ctx <= n else decode_rule(ctx))
    for temperature in (0.0, 0.7):
        rt = CudaBackend(model=model, tokenizer=_Tokenizer(model.vocab), seed=11)
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
        assert rt.memory_gib() > 0 and rt.device == "cuda" and "B200" in rt.description
    torch.cuda.synchronize()


@pytest.mark.gpu
def test_run_test_py_greedy_matches_oracle(tmp_path):
    """test.py --runtime cuda's loop on a packed cache directory."""
    from _models import oracle_decode, oracle_model

    from harsh4b_b200.cache import write_cache
    from harsh4b_b200.cli import run_test_py
    from harsh4b_b200.runtime import load_model

    checkpoint, prompt = _tiny()
    write_cache(tmp_path / "cache", checkpoint)
    model = load_model(tmp_path / "cache", kv_dtype="float32")
    rule, n = model.attention_split_rule(), len(prompt)
    _, greedy = oracle_decode(oracle_model(checkpoint, attn_splits=lambda ctx: 1 if ctx <= n else rule(ctx)),
                              prompt, 7)
    args = argparse.Namespace(max_new_tokens=6, warmup_tokens=2, temperature=0.0, top_p=0.9, top_k=50,
                              repetition_penalty=1.0, seed=0)
    lines = []
    result = run_test_py(args, prompt, None, tmp_path / "cache", model=model,
                         out=lambda *a, **k: lines.append(" ".join(str(x) for x in a)))
    stops = {151643, 151645}
    want = []
    for token in greedy:
        if token in stops or len(want) >= 6:
            break
        want.append(token)
    assert result["generated"] == want
    assert any(line.startswith("prefill:") for line in lines) and any(line.startswith("decode:") for line in lines)
