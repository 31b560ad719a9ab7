"""Batched int4 x int8 GEMM (h4b_int4_gemm), per-token quantisation of rows
and PackedInt4Linear: every row must equal the oracle's single-token
quantise + GEMV bit for bit."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import oracle  # noqa: E402
from harsh4b_b200 import ops, packed  # noqa: E402
from harsh4b_b200.synthetic import int4_matrix, outlier_activation, row_scales  # noqa: E402


def _problem(rng, tokens, rows, width):
    weights = int4_matrix(rng, rows, width)
    scales = row_scales(rng, rows)
    seed = int(rng.integers(1 << 30))
    values = np.stack([outlier_activation(width, seed=seed + t) for t in range(tokens)]).astype(np.float32)
    return weights, scales, values


def _oracle_rows(weights, scales, values):
    outs, x8s, act, sums = [], [], [], []
    for row in values:
        q = np.empty(row.size, dtype=np.int8)
        s = oracle.quantize_activation(np.ascontiguousarray(row), q)
        out, _ = oracle.int4_gemv(q, weights, scales, s)
        outs.append(out), x8s.append(q), act.append(s), sums.append(int(q.astype(np.int64).sum()))
    return np.stack(outs), np.stack(x8s), np.array(act, dtype=np.float32), np.array(sums)


@pytest.mark.parametrize("tokens,rows,width", [(2, 256, 2560), (17, 6144, 2560), (64, 2560, 9728),
                                               (130, 2560, 4096), (5, 128, 64)])
def test_gemm_rows_bit_exact(tokens, rows, width):
    rng = np.random.default_rng(tokens * 7 + rows)
    weights, scales, values = _problem(rng, tokens, rows, width)
    want, want_x8, want_scale, want_sum = _oracle_rows(weights, scales, values)
    v = torch.from_numpy(values).cuda()
    x8, act, sums = ops.quantize_rows(v)
    np.testing.assert_array_equal(x8.cpu().numpy(), want_x8)
    np.testing.assert_array_equal(act.cpu().numpy(), want_scale)
    np.testing.assert_array_equal(sums.cpu().numpy(), want_sum)
    out = ops.int4_gemm(x8, act, sums, torch.from_numpy(weights).cuda(), torch.from_numpy(scales).cuda())
    np.testing.assert_array_equal(out.cpu().numpy(), want)


def test_gemm_rejects_unsupported_shapes():
    x = torch.zeros(4, 64, device="cuda")
    w = torch.zeros(100, 32, dtype=torch.uint8, device="cuda")
    s = torch.ones(100, device="cuda")
    with pytest.raises(ValueError):
        ops.int4_gemm_rows(x, w, s)


def test_packed_linear_one_and_many_tokens():
    rng = np.random.default_rng(9)
    weights, scales, values = _problem(rng, 6, 1024, 2560)
    want, _, _, _ = _oracle_rows(weights, scales, values)
    bias = rng.normal(0, 1, 1024).astype(np.float32)
    layer = packed.PackedInt4Linear(torch.from_numpy(weights).cuda(), torch.from_numpy(scales).cuda(),
                                    torch.from_numpy(bias).cuda())
    x = torch.from_numpy(values).cuda().reshape(2, 3, 2560)
    got = layer(x)
    assert got.shape == (2, 3, 1024) and got.dtype == torch.float32
    np.testing.assert_array_equal(got.reshape(6, 1024).cpu().numpy(), want + bias)
    one = layer(x[0, 0])
    np.testing.assert_array_equal(one.cpu().numpy(), want[0] + bias)
    half = layer(x.to(torch.bfloat16))
    assert half.dtype == torch.bfloat16 and half.shape == (2, 3, 1024)
    dense = (layer.dequant() @ x.reshape(6, 2560).T).T + layer.bias
    assert torch.allclose(got.reshape(6, 1024), dense, rtol=0.05, atol=0.05 * dense.abs().max().item())
    assert "b200_int4" in packed.KERNELS
    packed.set_kernel("b200_int4")
