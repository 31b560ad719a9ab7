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


SHAPES = [(2, 256, 2560), (17, 6144, 2560), (64, 2560, 9728), (100, 1024, 2560), (130, 2560, 4096),
          (300, 384, 2560), (5, 128, 64)]


@pytest.mark.parametrize("kernel", ["tcgen05", "mma_sync", "auto"])
@pytest.mark.parametrize("tokens,rows,width", SHAPES)
def test_gemm_rows_bit_exact(tokens, rows, width, kernel):
    if kernel == "tcgen05" and width % 128:
        pytest.skip("the tcgen05 kernel needs width % 128 == 0")
    rng = np.random.default_rng(tokens * 7 + rows)
    weights, scales, values = _problem(rng, tokens, rows, width)
    want, want_x8, want_scale, want_sum = _oracle_rows(weights, scales, values)
    v = torch.from_numpy(values).cuda()
    x8, act, sums = ops.quantize_rows(v)
    np.testing.assert_array_equal(x8.cpu().numpy(), want_x8)
    np.testing.assert_array_equal(act.cpu().numpy(), want_scale)
    np.testing.assert_array_equal(sums.cpu().numpy(), want_sum)
    out = ops.int4_gemm(x8, act, sums, torch.from_numpy(weights).cuda(), torch.from_numpy(scales).cuda(),
                        kernel=kernel)
    np.testing.assert_array_equal(out.cpu().numpy(), want)


@pytest.mark.parametrize("rows,width", [(2560, 2560), (9728, 2560), (2560, 9728)])
def test_tcgen05_equals_mma_sync_at_prefill_size(rows, width):
    """2048 tokens (a prefill): the two tensor-core kernels give the same bits
    (each is pinned to the oracle above at smaller sizes)."""
    g = torch.Generator(device="cuda").manual_seed(rows + width)
    x8 = torch.randint(-127, 128, (2048, width), dtype=torch.int8, device="cuda", generator=g)
    act = torch.rand(2048, device="cuda", generator=g) * 1e-2
    sums = x8.to(torch.int32).sum(dim=1, dtype=torch.int32)
    codes = torch.randint(-7, 8, (rows, width), dtype=torch.int16, device="cuda", generator=g)
    w = ((codes[:, 0::2] & 0xF) | ((codes[:, 1::2] & 0xF) << 4)).to(torch.uint8)
    scales = torch.rand(rows, device="cuda", generator=g) * 1e-2
    a = ops.int4_gemm(x8, act, sums, w, scales, kernel="tcgen05")
    b = ops.int4_gemm(x8, act, sums, w, scales, kernel="mma_sync")
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    dense = (codes.to(torch.float64) @ x8[:64].to(torch.float64).T).T  # exact integers in float64
    want = (dense.to(torch.float32) * act[:64, None]) * scales[None, :]
    assert torch.equal(a[:64], want[:64])


# (tokens, rows, width): stream-K at M <= 64 (gate_up's 152 row tiles, qkv,
# o, down, tiny), the LM head (too many tiles: no split, acc untouched),
# split-K slices at M = 100, a prefill-sized M with no split
ACC_SHAPES = [(64, 19456, 2560), (64, 6144, 2560), (64, 2560, 4096), (64, 2560, 9728), (33, 19456, 2560),
              (1, 128, 128), (17, 384, 256), (64, 151936, 2560), (100, 2560, 2560), (2048, 2560, 2560)]


@pytest.mark.parametrize("tokens,rows,width", ACC_SHAPES)
def test_gemm_through_acc_buffer_same_bits(tokens, rows, width):
    """h4b_int4_gemm_acc (K split over CTAs, exact int32 partial sums added in
    a zeroed buffer): the same bits as h4b_int4_gemm and as exact integer
    sums, the residual form equal to x + proj, the buffer left zero."""
    g = torch.Generator(device="cuda").manual_seed(tokens * 131 + rows + width)
    x8 = torch.randint(-127, 128, (tokens, width), dtype=torch.int8, device="cuda", generator=g)
    act = torch.rand(tokens, device="cuda", generator=g) * 1e-2
    sums = x8.to(torch.int32).sum(dim=1, dtype=torch.int32)
    codes = torch.randint(-7, 8, (rows, width), dtype=torch.int16, device="cuda", generator=g)
    w = ((codes[:, 0::2] & 0xF) | ((codes[:, 1::2] & 0xF) << 4)).to(torch.uint8)
    scales = torch.rand(rows, device="cuda", generator=g) * 1e-2
    acc = torch.zeros(tokens * rows, dtype=torch.int32, device="cuda")
    plain = ops.int4_gemm(x8, act, sums, w, scales)
    split = ops.int4_gemm_acc(x8, act, sums, w, scales, acc)
    prev = torch.randn(tokens, rows, device="cuda", generator=g)
    res = ops.int4_gemm_acc(x8, act, sums, w, scales, acc, out=prev.clone(), residual=True)
    torch.cuda.synchronize()
    assert torch.equal(split, plain)
    assert torch.equal(res, prev + plain)
    assert int(acc.abs().max()) == 0
    m = min(tokens, 64)
    dense = (codes.to(torch.float64) @ x8[:m].to(torch.float64).T).T  # exact integers in float64
    assert torch.equal(split[:m], (dense.to(torch.float32) * act[:m, None]) * scales[None, :])


def test_gemm_acc_unaligned_output_same_bits():
    """An output that is not 16-byte aligned takes the scalar finalize: the
    same bits as the vectorised one."""
    g = torch.Generator(device="cuda").manual_seed(7)
    tokens, rows, width = 64, 2560, 4096
    x8 = torch.randint(-127, 128, (tokens, width), dtype=torch.int8, device="cuda", generator=g)
    act = torch.rand(tokens, device="cuda", generator=g) * 1e-2
    sums = x8.to(torch.int32).sum(dim=1, dtype=torch.int32)
    w = torch.randint(0, 256, (rows, width // 2), dtype=torch.uint8, device="cuda", generator=g)
    scales = torch.rand(rows, device="cuda", generator=g) * 1e-2
    acc = torch.zeros(tokens * rows, dtype=torch.int32, device="cuda")
    base = torch.randn(tokens * rows + 1, device="cuda", generator=g)
    shifted = base[1:].view(tokens, rows)  # 4 bytes past a 16-byte boundary
    want = shifted + ops.int4_gemm(x8, act, sums, w, scales)
    ops.int4_gemm_acc(x8, act, sums, w, scales, acc, out=shifted, residual=True)
    torch.cuda.synchronize()
    assert torch.equal(shifted, want)
    assert int(acc.abs().max()) == 0


def test_gemm_acc_rejects_short_buffer():
    x8 = torch.zeros(4, 256, dtype=torch.int8, device="cuda")
    w = torch.zeros(128, 128, dtype=torch.uint8, device="cuda")
    one = torch.ones(4, device="cuda")
    with pytest.raises(ValueError):
        ops.int4_gemm_acc(x8, one, torch.zeros(4, dtype=torch.int32, device="cuda"), w, torch.ones(128, device="cuda"),
                          torch.zeros(10, dtype=torch.int32, device="cuda"))


def test_tcgen05_rejects_width_not_multiple_of_128():
    x8 = torch.zeros(4, 64, dtype=torch.int8, device="cuda")
    act = torch.ones(4, device="cuda")
    sums = torch.zeros(4, dtype=torch.int32, device="cuda")
    w = torch.zeros(128, 32, dtype=torch.uint8, device="cuda")
    s = torch.ones(128, device="cuda")
    with pytest.raises(ValueError):
        ops.int4_gemm(x8, act, sums, w, s, kernel="tcgen05")


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
