"""The allocation-free attention entry point (h4b_gqa_decode_noalloc).

It serves callers that cannot allocate device memory at the point they run
attention (a serving process whose own pool already holds nearly all HBM, or
a plugin whose host owns the device allocator). Called through the C ABI,
it must agree with h4b_gqa_decode -- the entry point that takes caller
scratch -- within the attention tolerance of the other tests, on two calls in
a row that share the library's static scratch array. Both are also checked
against the CPU oracle's restatement of litespark_gqa_decode, so a fault the
two device entry points share does not pass unseen.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import oracle  # noqa: E402
from harsh4b_b200 import _lib  # noqa: E402

TOL = 2e-5  # the attention tolerance of tests/test_gpu_ops.py


def _case(seed, kv_heads, groups, context, capacity):
    rng = np.random.default_rng([seed, context])
    q = torch.from_numpy(rng.standard_normal((kv_heads * groups, 128), dtype=np.float32)).cuda()
    keys = torch.from_numpy(rng.standard_normal((capacity, kv_heads, 128), dtype=np.float32)).cuda()
    values = torch.from_numpy(rng.standard_normal((capacity, kv_heads, 128), dtype=np.float32)).cuda()
    return q, keys, values


def _with_scratch(lib, q, keys, values, context, kv_heads, groups):
    capacity = keys.shape[0]
    scores = torch.empty(kv_heads * groups * capacity, dtype=torch.float32, device="cuda")
    out = torch.empty(kv_heads * groups, 128, dtype=torch.float32, device="cuda")
    rc = lib.h4b_gqa_decode(q.data_ptr(), keys.data_ptr(), values.data_ptr(), scores.data_ptr(), out.data_ptr(),
                            context, kv_heads, groups, 128, capacity, torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    return out


def _no_alloc(lib, q, keys, values, context, kv_heads, groups):
    out = torch.full((kv_heads * groups, 128), float("nan"), dtype=torch.float32, device="cuda")
    rc = lib.h4b_gqa_decode_noalloc(q.data_ptr(), keys.data_ptr(), values.data_ptr(), out.data_ptr(), context,
                                    kv_heads, groups, 128, torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    return out


def test_no_alloc_attention_matches_scratch_entry_point_twice():
    lib = _lib.lib()
    # Two calls in a row: the second reuses the static array the first filled.
    for seed, (kv_heads, groups, context, capacity) in enumerate([(8, 4, 3000, 4096), (2, 3, 700, 900)]):
        q, keys, values = _case(seed, kv_heads, groups, context, capacity)
        want = _with_scratch(lib, q, keys, values, context, kv_heads, groups).cpu().numpy()
        got = _no_alloc(lib, q, keys, values, context, kv_heads, groups).cpu().numpy()
        np.testing.assert_allclose(got, want, rtol=TOL, atol=TOL)
        capacity = keys.shape[0]
        cpu = np.empty((kv_heads * groups, 128), dtype=np.float32)
        scores = np.empty(kv_heads * groups * capacity, dtype=np.float32)
        oracle.gqa_decode(q.cpu().numpy(), keys.cpu().numpy(), values.cpu().numpy(), scores, cpu, context,
                          kv_heads, groups, 128, capacity)
        np.testing.assert_allclose(got, cpu, rtol=TOL, atol=TOL)
        np.testing.assert_allclose(want, cpu, rtol=TOL, atol=TOL)
    assert _lib.device_status() == 0


def test_no_alloc_rejects_requests_beyond_its_static_scratch():
    lib = _lib.lib()
    dummy = torch.zeros(4, dtype=torch.float32, device="cuda")
    # 256 kv heads x 8 groups x 132 floats per split is above the 262144-float array.
    rc = lib.h4b_gqa_decode_noalloc(dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), 16,
                                    256, 8, 128, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.H4B_ETOOBIG
    with pytest.raises(ValueError, match="static scratch"):
        _lib.check(rc, "h4b_gqa_decode_noalloc")
