"""Operator-level parity of the sm_100a kernels against the CPU oracle.

Integer work (int32 GEMV accumulators, int8 quantisation, argmax, nibble
unpacking) must be bit-exact; the GEMV fp32 outputs are bit-exact too
because the epilogue order float(acc) * act_scale * w_scale is the
reference's (litespark_int4.cpp:73-74). Shapes follow the reference's KAT
(67 x 128, seed 41) and the seven body projections of Qwen3-4B.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import oracle  # noqa: E402
from harsh4b_b200 import ops  # noqa: E402
from harsh4b_b200.cache import pack_int4  # noqa: E402
from harsh4b_b200.synthetic import int4_matrix, outlier_activation, row_scales  # noqa: E402

SHAPES = {"q": (4096, 2560), "k": (1024, 2560), "v": (1024, 2560), "o": (2560, 4096),
          "gate": (9728, 2560), "up": (9728, 2560), "down": (2560, 9728)}


def cuda(array):
    return torch.from_numpy(np.ascontiguousarray(array)).cuda()


def test_reference_kat_gemv_seed41():
    rng = np.random.default_rng(41)
    weights = rng.integers(-7, 8, size=(67, 128), dtype=np.int8)
    x = rng.integers(-127, 128, size=128, dtype=np.int8)
    scales = rng.random(67, dtype=np.float32)
    integer = weights.astype(np.int32) @ x.astype(np.int32)
    acc = torch.empty(67, dtype=torch.int32, device="cuda")
    out, _ = ops.int4_i8_gemv(cuda(x), cuda(pack_int4(weights)), cuda(scales), 0.007, acc=acc)
    np.testing.assert_array_equal(acc.cpu().numpy(), integer)
    expected = integer.astype(np.float32) * np.float32(0.007) * scales
    np.testing.assert_array_equal(out.cpu().numpy(), expected)
    np.testing.assert_allclose(out.cpu().numpy(), integer.astype(np.float32) * scales * np.float32(0.007),
                               rtol=2e-6, atol=2e-5)


@pytest.mark.parametrize("name", list(SHAPES))
def test_body_gemv_int8_bit_exact(name):
    rows, width = SHAPES[name]
    rng = np.random.default_rng([3, rows, width])
    packed, scales = int4_matrix(rng, rows, width), row_scales(rng, rows)
    x = rng.integers(-127, 128, size=width, dtype=np.int8)
    want_out, want_acc = oracle.int4_gemv(x, packed, scales, 0.0123)
    acc = torch.empty(rows, dtype=torch.int32, device="cuda")
    out, _ = ops.int4_i8_gemv(cuda(x), cuda(packed), cuda(scales), 0.0123, acc=acc)
    np.testing.assert_array_equal(acc.cpu().numpy(), want_acc)
    np.testing.assert_array_equal(out.cpu().numpy(), want_out)


@pytest.mark.parametrize("name", list(SHAPES))
def test_body_gemv_fused_quant_bit_exact(name):
    """Config 1: fp32 N(0,1) activations with 0.5% x20 outliers, quantised in-kernel."""
    rows, width = SHAPES[name]
    rng = np.random.default_rng([4, rows, width])
    packed, scales = int4_matrix(rng, rows, width), row_scales(rng, rows)
    x = outlier_activation(width, seed=rows)
    q = np.empty(width, dtype=np.int8)
    act_scale = oracle.quantize_activation(x, q)
    want_out, want_acc = oracle.int4_gemv(q, packed, scales, act_scale)
    acc = torch.empty(rows, dtype=torch.int32, device="cuda")
    out, _, scale = ops.int4_gemv_fused_quant(cuda(x), cuda(packed), cuda(scales), acc=acc)
    assert scale.item() == np.float32(act_scale)
    np.testing.assert_array_equal(acc.cpu().numpy(), want_acc)
    np.testing.assert_array_equal(out.cpu().numpy(), want_out)
    rel = np.abs(out.cpu().numpy() - want_out) / np.maximum(np.abs(want_out), 1e-30)
    assert rel.max() <= 1e-3


@pytest.mark.parametrize("rows,width", [(1, 32), (7, 64), (300, 96), (1000, 6144), (64, 16384)])
def test_gemv_odd_shapes(rows, width):
    rng = np.random.default_rng([5, rows, width])
    packed, scales = int4_matrix(rng, rows, width), row_scales(rng, rows)
    x = rng.integers(-127, 128, size=width, dtype=np.int8)
    _, want_acc = oracle.int4_gemv(x, packed, scales, 1.0)
    acc = torch.empty(rows, dtype=torch.int32, device="cuda")
    ops.int4_i8_gemv(cuda(x), cuda(packed), cuda(scales), 1.0, acc=acc)
    np.testing.assert_array_equal(acc.cpu().numpy(), want_acc)


def test_gemv_rejects_bad_shapes():
    w = torch.zeros((4, 8), dtype=torch.uint8, device="cuda")
    s = torch.ones(4, dtype=torch.float32, device="cuda")
    x = torch.zeros(16, dtype=torch.int8, device="cuda")
    with pytest.raises(ValueError):
        ops.int4_i8_gemv(x, w, s, 1.0)  # width 16 is not a multiple of 32


@pytest.mark.parametrize("n", [8, 2560, 4096, 9728])
def test_quantize_activation_bit_exact(n):
    x = outlier_activation(n, seed=n)
    q = np.empty(n, dtype=np.int8)
    scale = oracle.quantize_activation(x, q)
    got_q, got_scale = ops.quantize_activation(cuda(x))
    np.testing.assert_array_equal(got_q.cpu().numpy(), q)
    assert got_scale.item() == np.float32(scale)


def test_rmsnorm_matches_oracle():
    rng = np.random.default_rng(8)
    x = rng.standard_normal(2560, dtype=np.float32)
    w = (1 + 0.02 * rng.standard_normal(2560)).astype(np.float32)
    want = np.empty_like(x)
    oracle.OracleKernel().rmsnorm_into(x, w, want, 1e-6)
    got = ops.rmsnorm(cuda(x), cuda(w), 1e-6).cpu().numpy()
    np.testing.assert_allclose(got, want, rtol=2e-6, atol=1e-7)


def test_add_inplace():
    rng = np.random.default_rng(9)
    x, y = rng.standard_normal(2560, dtype=np.float32), rng.standard_normal(2560, dtype=np.float32)
    got = ops.add_inplace(cuda(x), cuda(y)).cpu().numpy()
    np.testing.assert_array_equal(got, x + y)


@pytest.mark.parametrize("kv_heads,groups,context,capacity", [(2, 3, 7, 11), (8, 4, 1, 1), (8, 4, 1000, 1024),
                                                              (1, 8, 300, 5000)])
def test_gqa_decode_matches_oracle(kv_heads, groups, context, capacity):
    rng = np.random.default_rng([41, context])
    d = 128
    q = rng.standard_normal((kv_heads * groups, d), dtype=np.float32)
    keys = rng.standard_normal((capacity, kv_heads, d), dtype=np.float32)
    values = rng.standard_normal((capacity, kv_heads, d), dtype=np.float32)
    scores = np.empty((kv_heads * groups, capacity), dtype=np.float32)
    want = np.empty_like(q)
    oracle.gqa_decode(q, keys, values, scores, want, context, kv_heads, groups, d, capacity)
    got = ops.gqa_decode(cuda(q), cuda(keys), cuda(values), context, kv_heads, groups).cpu().numpy()
    np.testing.assert_allclose(got, want, rtol=2e-5, atol=2e-5)


def test_embedding_and_argmax_exact():
    rng = np.random.default_rng(10)
    table, scales = int4_matrix(rng, 1000, 256), row_scales(rng, 1000)
    for token in (0, 17, 999):
        t = torch.tensor([token], dtype=torch.int32, device="cuda")
        got = ops.embedding(t, cuda(table), cuda(scales)).cpu().numpy()
        signed = table[token].view(np.int8)
        want = np.empty(256, dtype=np.float32)
        want[0::2], want[1::2] = (signed << 4) >> 4, signed >> 4
        want *= scales[token]
        np.testing.assert_array_equal(got, want)
    logits = rng.standard_normal(151936).astype(np.float32)
    logits[[5, 70000]] = logits.max() + 1  # a tie: the first index wins
    assert ops.argmax(cuda(logits)).item() == 5
    assert ops.argmax(cuda(np.array([-1.0, 3.0, 2.0], dtype=np.float32))).item() == 1


def test_long_gemv_repeated_launches_exact():
    """A long GEMV wraps the shared-memory ring ~16 times per CTA; repeated
    launches catch ordering races between the ring's producer and its
    consumer warps (each launch must stay bit-exact)."""
    rows, width = 151936, 2560
    rng = np.random.default_rng([6, rows, width])
    packed, scales = int4_matrix(rng, rows, width), row_scales(rng, rows)
    w, s = cuda(packed), cuda(scales)
    for trial in range(12):
        x = outlier_activation(width, seed=100 + trial)
        q = np.empty(width, dtype=np.int8)
        _, want = oracle.int4_gemv(q, packed, scales, oracle.quantize_activation(x, q))
        acc = torch.empty(rows, dtype=torch.int32, device="cuda")
        ops.int4_gemv_fused_quant(cuda(x), w, s, acc=acc)
        np.testing.assert_array_equal(acc.cpu().numpy(), want)
