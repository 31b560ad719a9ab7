"""The GPU LATTICE -> int4 converter (csrc/lattice.cu through the C ABI)
against the reference's conversion (golden fixtures) and the CPU
restatement, and the model built from a LATTICE checkpoint file.

Tolerance: the rotation is accumulated in fp64 on the device, so against
the restatement's fp64 rotation the scales agree to 2.5e-7 (they are
bit-equal in practice); the reference rotates in fp32 through its BLAS,
whose rounding moves a row maximum by up to ~1e-6 relative (measured: 4-7
ulp), so against it the scales agree to 2e-6 and a code may differ by one
where w / scale lies within 1e-4 of a rounding boundary. The dense-row
(embedding) conversion has no product and must be bit-exact.
"""
import json
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle import lattice as L  # noqa: E402

GOLDEN = Path(__file__).resolve().parent / "golden" / "lattice_cases.npz"
TIE = 1e-4


def _unpack(packed):
    signed = packed.view(np.int8)
    out = np.empty((packed.shape[0], packed.shape[1] * 2), dtype=np.int8)
    out[:, 0::2] = (signed << 4) >> 4
    out[:, 1::2] = signed >> 4
    return out


def assert_codes_close(got_packed, got_scales, want_packed, want_scales, weight, rtol=2.5e-7):
    """Scales within rtol; codes equal except near-ties, where they may differ by one."""
    np.testing.assert_allclose(got_scales, want_scales, rtol=rtol, atol=0)
    got, want = _unpack(np.asarray(got_packed)), _unpack(np.asarray(want_packed))
    diff = got.astype(np.int16) - want.astype(np.int16)
    assert np.abs(diff).max(initial=0) <= 1
    rows, cols = np.nonzero(diff)
    ratio = weight[rows, cols] / want_scales[rows]
    assert np.all(np.abs(np.abs(ratio - np.floor(ratio)) - 0.5) < TIE), "a code differs away from a rounding tie"
    return len(rows)


def _projection(golden, i):
    prefix = f"p{i}_"
    p = {k[len(prefix):]: golden[k] for k in golden.files if k.startswith(prefix)}
    p["shape"] = tuple(int(v) for v in p["shape"])
    return p


def test_projection_matches_reference_golden():
    from harsh4b_b200.lattice import convert_projection

    golden = np.load(GOLDEN)
    for i in range(int(golden["n_projections"])):
        p = _projection(golden, i)
        packed, scales = convert_projection(p, p["left"], p["right"])
        _, _, weight = L.convert_projection(p, p["left"], p["right"])
        assert_codes_close(packed.cpu().numpy(), scales.cpu().numpy(), p["packed"], p["scales"], weight, rtol=2e-6)


def test_embedding_rows_bit_exact_with_reference_golden():
    from harsh4b_b200.lattice import convert_rows

    golden = np.load(GOLDEN)
    for i in range(int(golden["n_embeddings"])):
        packed, scales = convert_rows(golden[f"e{i}_source"])
        np.testing.assert_array_equal(packed.cpu().numpy(), golden[f"e{i}_packed"])
        np.testing.assert_array_equal(scales.cpu().numpy(), golden[f"e{i}_scales"])


@pytest.mark.parametrize("rows,width,dims,blocksize", [(96, 2560, (40, 64), 128), (64, 4096, (64, 64), 128),
                                                       (40, 9728, (76, 128), 128), (33, 2560, (64, 40), 64)])
def test_projection_qwen_widths_against_restatement(rows, width, dims, blocksize):
    from harsh4b_b200.lattice import convert_projection

    rng = np.random.default_rng([rows, width])
    p = L.synthetic_projection(rng, rows, width, blocksize)
    left, right = L.orthogonal(rng, dims[0]), L.orthogonal(rng, dims[1])
    packed, scales = convert_projection(p, left, right)
    packed, scales = packed.cpu().numpy(), scales.cpu().numpy()
    # fp64 on both sides: equal but for fp32 rounding of the last step
    want, want_scales, weight = L.convert_projection(p, left, right, exact=True)
    assert_codes_close(packed, scales, want, want_scales, weight)
    # the reference's fp32 order: a handful of tie flips at most
    want32, scales32, weight32 = L.convert_projection(p, left, right)
    flips = assert_codes_close(packed, scales, want32, scales32, weight32, rtol=2e-6)
    assert flips <= max(2, rows * width // 10000)


def test_t1_count_mismatch_is_rejected():
    from harsh4b_b200.lattice import convert_projection

    golden = np.load(GOLDEN)
    p = _projection(golden, 0)
    p["n_T1"] = int(p["n_T1"]) + 1
    with pytest.raises(ValueError, match="T1 count"):
        convert_projection(p, p["left"], p["right"])


def test_model_from_lattice_checkpoint(tmp_path):
    """build_b200_model: convert a LATTICE file into the shared cache on the
    GPU, take the norms from the checkpoint, and decode; the cache must equal
    the restatement's conversion (ties aside) and the decode must equal the
    oracle's decode of that same cache bit for bit. A second build reuses the
    cache files untouched."""
    from _models import cuda_decode, oracle_decode, oracle_for, write_lattice_checkpoint

    from harsh4b_b200.cache import read_cache, slug
    from harsh4b_b200.lattice import build_b200_model, build_cache
    from harsh4b_b200.synthetic import synthetic_prompt, tiny_config

    config = tiny_config()
    path = tmp_path / "model.lat.pt"
    plain, embedding, norms = write_lattice_checkpoint(path, config, seed=5)
    cache_dir = tmp_path / "cache"
    model = build_b200_model(path, config=config, cache_dir=cache_dir, kv_dtype="float32")
    manifest = json.loads((cache_dir / "manifest.json").read_text())
    assert manifest["complete"] and len(manifest["projections"]) == 7 * config["num_hidden_layers"]
    for name, (packed, left, right) in plain.items():
        want, want_scales, weight = L.convert_projection(packed, left, right, exact=True)
        got = np.load(cache_dir / f"{slug(name)}.int4.npy")
        got_scales = np.load(cache_dir / f"{slug(name)}.scales.npy")
        assert_codes_close(got, got_scales, want, want_scales, weight)
    want_embed, want_embed_scales = L.convert_rows(embedding)
    np.testing.assert_array_equal(np.load(cache_dir / "embedding.int4.npy"), want_embed)
    np.testing.assert_array_equal(np.load(cache_dir / "embedding.scales.npy"), want_embed_scales)

    checkpoint = read_cache(cache_dir, config)
    checkpoint.norms = norms
    prompt = synthetic_prompt(config, 5, seed=5)
    want_logits, greedy = oracle_decode(oracle_for(checkpoint, model), prompt, 6)
    got_logits, got_greedy = cuda_decode(model, prompt, 6, teacher=greedy)
    assert got_greedy == greedy
    np.testing.assert_array_equal(got_logits, want_logits)

    stamps = {p.name: p.stat().st_mtime_ns for p in cache_dir.glob("*.npy")}
    again = build_cache(path, config, cache_dir=cache_dir)
    assert {p.name: p.stat().st_mtime_ns for p in cache_dir.glob("*.npy")} == stamps
    np.testing.assert_array_equal(again.norms["model.norm.weight"], norms["model.norm.weight"])
