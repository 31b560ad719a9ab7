"""Device sampling (h4b_sample) against the oracle restatement of the
reference's CPU-runtime sampler and its golden tokens."""
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from harsh4b_b200 import ops  # noqa: E402
from oracle.model import sample_runtime  # noqa: E402

GOLDEN = Path(__file__).resolve().parent / "golden" / "sample_cases.npz"
PROB_RTOL = 2e-6  # exp of the device vs numpy may differ in the last ulp


def _device(logits, generated, uniform, **kw):
    x = torch.from_numpy(np.ascontiguousarray(logits, dtype=np.float32)).cuda()
    gen = sorted(set(generated))
    g = torch.tensor(gen, dtype=torch.int32, device="cuda") if gen else None
    token, ids, probs = ops.sample(x, g, uniform, return_candidates=True, **kw)
    torch.cuda.synchronize()
    return int(token.item()), ids.cpu().numpy(), probs.cpu().numpy()


def _near_boundary(probs, uniform, eps=1e-6):
    cdf = probs.astype(np.float64).cumsum()
    cdf /= cdf[-1]
    return bool(np.any(np.abs(cdf - uniform) < eps))


def test_golden_tokens_on_device():
    data = np.load(GOLDEN)
    for i in range(len(data["tokens"])):
        temperature, top_p, top_k, penalty = data["params"][i]
        generated = [int(t) for t in data["generated"][i] if t >= 0]
        token, ids, probs = _device(data["logits"][i], generated, float(data["uniform"][i]), temperature=temperature,
                                    top_p=top_p, top_k=int(top_k), repetition_penalty=penalty)
        assert token == int(data["tokens"][i]) or (temperature > 0.01 and _near_boundary(probs, data["uniform"][i]))


@pytest.mark.parametrize("top_k,top_p,temperature", [(50, 0.9, 0.7), (40, 1.0, 1.3), (64, 0.5, 0.4), (1, 0.9, 0.7)])
def test_full_vocab_matches_oracle(top_k, top_p, temperature):
    rng = np.random.default_rng(top_k)
    for trial in range(12):
        logits = rng.normal(0, 4, 151936).astype(np.float32)
        generated = list(rng.integers(0, 151936, 24))
        uniform = float(rng.random())
        want, w_ids, w_probs = sample_runtime(logits, generated, uniform, temperature=temperature, top_p=top_p,
                                              top_k=top_k, repetition_penalty=1.15, return_candidates=True)
        got, ids, probs = _device(logits, generated, uniform, temperature=temperature, top_p=top_p, top_k=top_k,
                                  repetition_penalty=1.15)
        np.testing.assert_array_equal(ids, w_ids)
        np.testing.assert_allclose(probs, w_probs, rtol=PROB_RTOL, atol=1e-9)
        assert got == want or _near_boundary(w_probs, uniform)


def test_greedy_is_argmax_of_penalised_logits():
    rng = np.random.default_rng(5)
    logits = rng.normal(0, 1, 151936).astype(np.float32)
    top = int(np.argmax(logits))
    want = sample_runtime(logits, [top], 0.0, temperature=0.0, repetition_penalty=1.5)
    got, _, _ = _device(logits, [top], 0.0, temperature=0.0, repetition_penalty=1.5)
    assert got == want


def test_rejects_large_top_k_and_bad_uniform():
    x = torch.zeros(1000, device="cuda")
    with pytest.raises(ValueError):
        ops.sample(x, None, 0.5, top_k=65)
    with pytest.raises(ValueError):
        ops.sample(x, None, 1.0)
