"""The CPU oracle against the reference's own known answers and fixtures.

KATs follow the reference's tests/test_cpu_lightspark.py (int4 packing
:59-64, SDOT GEMV vs integer reference :71-99, GQA vs einsum :101-122,
argmax :36-39); ``tests/golden/tiny_decode.npz`` holds logits produced by the
reference's ``LiteSparkQwen.forward_token`` (see ``tests/golden/make_golden.py``).
"""
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

import oracle
from harsh4b_b200.cache import pack_int4, unpack_int4
from harsh4b_b200.synthetic import synthetic_checkpoint

GOLDEN = Path(__file__).resolve().parent / "golden" / "tiny_decode.npz"


def test_int4_packing_known_answer():
    weights = np.array([[-7, -1, 0, 7], [6, -6, 3, -3]], dtype=np.int8)
    expected = np.array([[0xF9, 0x70], [0xA6, 0xD3]], dtype=np.uint8)
    np.testing.assert_array_equal(pack_int4(weights), expected)
    np.testing.assert_array_equal(unpack_int4(expected), weights)
    with pytest.raises(ValueError, match=r"\[-7,\+7\]"):
        pack_int4(np.array([[8, 0]], dtype=np.int8))


def _seed41_gemv_case():
    rng = np.random.default_rng(41)
    weights = rng.integers(-7, 8, size=(67, 128), dtype=np.int8)
    activation = rng.integers(-127, 128, size=128, dtype=np.int8)
    scales = rng.random(67, dtype=np.float32)
    return rng, weights, activation, scales


@pytest.mark.parametrize("scalar", [True, False])
def test_gemv_matches_integer_reference(scalar):
    _, weights, activation, scales = _seed41_gemv_case()
    integer = weights.astype(np.int32) @ activation.astype(np.int32)
    expected = integer.astype(np.float32) * scales * np.float32(0.007)
    out, acc = oracle.int4_gemv(activation, pack_int4(weights), scales, 0.007, scalar=scalar)
    np.testing.assert_array_equal(acc, integer)
    np.testing.assert_allclose(out, expected, rtol=2e-6, atol=2e-5)
    # The epilogue order of litespark_int4.cpp:73-74 makes the result exact.
    np.testing.assert_array_equal(out, integer.astype(np.float32) * np.float32(0.007) * scales)


@pytest.mark.parametrize("rows,width", [(1, 2), (5, 34), (67, 136), (130, 1000)])
def test_gemv_tails_and_odd_shapes(rows, width):
    rng = np.random.default_rng(rows * 1000 + width)
    weights = rng.integers(-7, 8, size=(rows, width), dtype=np.int8)
    x = rng.integers(-127, 128, size=width, dtype=np.int8)
    scales = rng.random(rows, dtype=np.float32)
    packed = pack_int4(weights)
    integer = weights.astype(np.int32) @ x.astype(np.int32)
    for scalar in (True, False):
        _, acc = oracle.int4_gemv(x, packed, scales, 1.0, scalar=scalar)
        np.testing.assert_array_equal(acc, integer)


def test_gqa_matches_einsum_reference():
    rng, *_ = _seed41_gemv_case()
    kv_heads, groups, context, capacity, head_dim = 2, 3, 7, 11, 16
    query = rng.standard_normal((kv_heads * groups, head_dim), dtype=np.float32)
    keys = rng.standard_normal((capacity, kv_heads, head_dim), dtype=np.float32)
    values = rng.standard_normal((capacity, kv_heads, head_dim), dtype=np.float32)
    scores = np.empty((kv_heads, groups, capacity), dtype=np.float32)
    attended = np.empty_like(query)
    oracle.gqa_decode(query, keys, values, scores, attended, context, kv_heads, groups, head_dim, capacity)
    s = np.einsum("hgd,thd->hgt", query.reshape(kv_heads, groups, head_dim), keys[:context],
                  dtype=np.float32) / np.sqrt(np.float32(head_dim))
    p = np.exp(s - s.max(axis=-1, keepdims=True))
    p /= p.sum(axis=-1, keepdims=True)
    reference = np.einsum("hgt,thd->hgd", p, values[:context], dtype=np.float32)
    np.testing.assert_allclose(attended, reference.reshape(kv_heads * groups, head_dim), rtol=2e-5, atol=2e-5)


def test_argmax_known_answer():
    logits = np.array([-1.0, 3.0, 2.0], dtype=np.float32)
    assert oracle.sample_logits(logits, [], argmax=True) == 1


def test_quantize_activation_contract():
    x = np.array([0.5, -2.0, 1.0, 0.0, 1.99], dtype=np.float32)
    q = np.empty(5, dtype=np.int8)
    scale = oracle.quantize_activation(x, q)
    assert scale == np.float32(2.0) / np.float32(127.0)
    qs = np.float32(127.0) / np.float32(2.0)
    np.testing.assert_array_equal(q, np.clip(np.rint(x * qs), -127, 127).astype(np.int8))
    assert q[1] == -127
    zeros = np.zeros(8, dtype=np.float32)
    assert oracle.quantize_activation(zeros, np.empty(8, np.int8)) == np.float32(1e-5) / np.float32(127)
    with pytest.raises(ValueError):
        oracle.quantize_activation(x, np.empty(3, dtype=np.int8))


def _digest(checkpoint):
    digest = hashlib.sha256()
    for name in sorted(checkpoint.projections):
        for array in checkpoint.projections[name]:
            digest.update(np.ascontiguousarray(array).tobytes())
    digest.update(checkpoint.embedding.tobytes())
    digest.update(checkpoint.embedding_scales.tobytes())
    for name in sorted(checkpoint.norms):
        digest.update(checkpoint.norms[name].tobytes())
    return digest.hexdigest()


def oracle_model(checkpoint, kv_dtype=np.float32):
    config = checkpoint.config
    layers = []
    for index in range(int(config["num_hidden_layers"])):
        parts = checkpoint.layer(index)
        layers.append(oracle.OracleLayer(*[oracle.OracleProjection(*p) for p in parts[:4]], *parts[4:]))
    return oracle.OracleQwen(config, layers, checkpoint.embedding, checkpoint.embedding_scales,
                             checkpoint.norms["model.norm.weight"], kv_dtype=kv_dtype)


# The oracle sums RMSNorm / qk-norm / attention in the device's order with the
# shared exp; the reference sums in numpy's order. On this int8-quantised
# model that difference alone moves logits by a few 1e-3 (see
# test_reduction_order_sensitivity), well inside the 1e-2 contract.
REFERENCE_ORDER_TOL = 5e-3


def test_oracle_reproduces_reference_decode():
    golden = np.load(GOLDEN)
    config = json.loads(str(golden["config"]))
    checkpoint = synthetic_checkpoint(config, seed=int(golden["seed"]))
    assert _digest(checkpoint) == str(golden["digest"]), "synthetic generator drifted"
    model = oracle_model(checkpoint)
    prompt, tokens = list(golden["prompt"]), list(golden["tokens"])
    state = model.new_state(len(prompt) + len(tokens))
    logits = [model.forward_token(int(t), state).copy() for t in prompt]
    generated = []
    for step in range(len(tokens)):
        generated.append(oracle.sample_logits(logits[-1], generated, argmax=True))
        logits.append(model.forward_token(generated[-1], state).copy())
    assert generated == tokens
    np.testing.assert_allclose(np.stack(logits), golden["logits"], rtol=0, atol=REFERENCE_ORDER_TOL)


def test_shared_exp_accuracy():
    x = np.linspace(-87.0, 88.0, 1_000_001, dtype=np.float32)
    y = oracle.exp(x).astype(np.float64)
    exact = np.exp(x.astype(np.float64))
    ulp = np.spacing(exact.astype(np.float32)).astype(np.float64)
    assert (np.abs(y - exact) / ulp).max() < 2.0
    assert oracle.exp(np.array([0.0, -np.inf, -90.0], dtype=np.float32)).tolist() == [1.0, 0.0, 0.0]


def test_kv_precision_sensitivity():
    """Why device parity is checked bit-exactly per KV precision rather than
    with one tolerance: on this synthetic int8-quantised model, rounding the
    KV cache to fp16 (the device's production setting) moves full-vocabulary
    logits by more than the 1e-2 contract even in a 2-layer model on the CPU
    oracle alone, because the per-token int8 quantiser turns small
    differences into code flips."""
    from harsh4b_b200.synthetic import qwen3_4b_config, synthetic_prompt

    config = qwen3_4b_config(num_hidden_layers=2)
    checkpoint = synthetic_checkpoint(config, seed=0)
    prompt = synthetic_prompt(config, 16, seed=0)
    a, b = oracle_model(checkpoint), oracle_model(checkpoint, kv_dtype=np.float16)
    sa, sb = a.new_state(16), b.new_state(16)
    drift = max(float(np.abs(a.forward_token(t, sa) - b.forward_token(t, sb)).max()) for t in prompt)
    assert drift > 1e-2


def test_choice_uniform_is_numpy_choice():
    """Generator.choice(ids, p) == the float64 CDF search at generator.random()."""
    from oracle.model import choice_uniform

    for seed in range(200):
        rng = np.random.default_rng(seed)
        n = int(rng.integers(1, 65))
        p = rng.random(n).astype(np.float32)
        p /= p.sum(dtype=np.float32)
        ids = rng.permutation(5000)[:n]
        a, b = np.random.default_rng(seed + 1), np.random.default_rng(seed + 1)
        assert int(a.choice(ids, p=p)) == choice_uniform(ids, p, b.random())


def test_sample_runtime_matches_reference_golden():
    """Tokens the reference's sample_numpy drew (tests/golden/sample_cases.npz)."""
    from oracle.model import sample_runtime

    data = np.load(Path(__file__).resolve().parent / "golden" / "sample_cases.npz")
    for i in range(len(data["tokens"])):
        temperature, top_p, top_k, penalty = data["params"][i]
        generated = [int(t) for t in data["generated"][i] if t >= 0]
        token = sample_runtime(data["logits"][i], generated, float(data["uniform"][i]), temperature=temperature,
                               top_p=top_p, top_k=int(top_k), repetition_penalty=penalty)
        assert token == int(data["tokens"][i]), i


def test_oracle_matches_reference_at_qwen_shapes():
    """The oracle (device-ordered reductions, its own exp) against the
    reference's numpy forward_token at Qwen3-4B's shapes
    (tests/golden/qwen_shape_decode.npz), fp32 KV as the reference keeps it:
    the same greedy token at every step, and logits no further from the
    numpy path than the reference's own native-kernel attention path is
    (one int8 code flipped by a last-ulp attention difference moves every
    later logit by a few 1e-2)."""
    import json

    from _models import oracle_model
    from harsh4b_b200.synthetic import synthetic_checkpoint

    golden = np.load(Path(__file__).resolve().parent / "golden" / "qwen_shape_decode.npz")
    checkpoint = synthetic_checkpoint(json.loads(str(golden["config"])), seed=int(golden["seed"]))
    model = oracle_model(checkpoint, kv_dtype=np.float32)
    prompt, tokens = golden["prompt"], golden["tokens"]
    state = model.new_state(len(prompt) + len(tokens))
    for token in prompt[:-1]:
        model.forward_token(int(token), state)
    worst = 0.0
    for step, token in enumerate([int(prompt[-1])] + [int(t) for t in tokens]):
        row = model.forward_token(token, state)
        got = np.concatenate([row[golden["sample_ids"]], row[golden["top_ids"][step]]])
        want = np.concatenate([golden["sample_logits"][step], golden["top_logits"][step]])
        worst = max(worst, float(np.abs(got - want).max()))
        if step < len(tokens):
            assert int(np.argmax(row)) == int(tokens[step])
    assert worst <= max(1e-2, float(golden["reference_path_drift"])), worst
