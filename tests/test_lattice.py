"""The LATTICE -> int4 conversion restatement (oracle/lattice.py) against the
reference's own functions (tests/golden/lattice_cases.npz), and the host side
of harsh4b_b200.lattice that needs no GPU: the checkpoint reader and the
cache identity."""
import sys
from pathlib import Path

import numpy as np
import pytest

from conftest import REFERENCE_ROOT, reference_available
from oracle import lattice as L

GOLDEN = Path(__file__).resolve().parent / "golden" / "lattice_cases.npz"


def _projection(golden, i):
    prefix = f"p{i}_"
    p = {k[len(prefix):]: golden[k] for k in golden.files if k.startswith(prefix)}
    p["shape"] = tuple(int(v) for v in p["shape"])
    return p


def test_oracle_matches_reference_conversion_golden():
    golden = np.load(GOLDEN)
    for i in range(int(golden["n_projections"])):
        p = _projection(golden, i)
        np.testing.assert_array_equal(L.expand_t1(p["shape"], p["maskid"], p["T1c"], p["n_T1"]), p["t1_dense"])
        codes, scales, _ = L.convert_projection(p, p["left"], p["right"])
        np.testing.assert_array_equal(codes, p["packed"])
        np.testing.assert_array_equal(scales, p["scales"])
    for i in range(int(golden["n_embeddings"])):
        codes, scales = L.convert_rows(golden[f"e{i}_source"])
        np.testing.assert_array_equal(codes, golden[f"e{i}_packed"])
        np.testing.assert_array_equal(scales, golden[f"e{i}_scales"])


@pytest.mark.parametrize("rows,width", [(7, 73), (131, 1024), (25, 9728)])
@pytest.mark.parametrize("mode", [None, 0, 3])
def test_expand_t1_edges(rows, width, mode):
    # The reference's own boundary cases (MLX/tests/test_runner.py:18-37).
    rng = np.random.default_rng(71)
    modes = rng.integers(0, 4, (rows, width), dtype=np.uint8)
    if mode is not None:
        modes.fill(mode)
    codes = rng.integers(0, 4, (rows, width), dtype=np.uint8)
    selected = codes[modes < 2]
    t1c = L.pack_codes(selected.reshape(1, -1)).reshape(-1)
    expected = L.pack_codes(np.where(modes < 2, codes, 0))
    np.testing.assert_array_equal(L.expand_t1((rows, width), L.pack_codes(modes), t1c, selected.size), expected)
    with pytest.raises(ValueError, match="T1 count"):
        L.expand_t1((rows, width), L.pack_codes(modes), t1c, selected.size + 1)


def test_read_lattice_round_trip_and_rejects_plain_state(tmp_path):
    torch = pytest.importorskip("torch")
    from _models import write_lattice_checkpoint

    from harsh4b_b200.lattice import norms_from_state, read_lattice
    from harsh4b_b200.synthetic import tiny_config

    config = tiny_config(num_hidden_layers=1, vocab_size=64)
    path = tmp_path / "model.lat.pt"
    plain, embedding, norms = write_lattice_checkpoint(path, config)
    state = read_lattice(path)
    name = "model.layers.0.mlp.down_proj"
    packed, left, right = plain[name]
    got = state[name + ".weight"]
    assert tuple(got["shape"]) == packed["shape"] and int(got["n_T1"]) == packed["n_T1"]
    np.testing.assert_array_equal(got["maskid"].numpy(), packed["maskid"])
    np.testing.assert_array_equal(got["mu"].numpy(), packed["mu"])
    np.testing.assert_array_equal(state[name + ".R"].numpy(), right)
    np.testing.assert_array_equal(state["model.embed_tokens.weight"].numpy(), embedding)
    for key, value in norms_from_state(state, config).items():
        np.testing.assert_array_equal(value, norms[key])
    other = tmp_path / "plain.pt"
    torch.save({"weight": torch.zeros(2)}, str(other))
    with pytest.raises(ValueError, match="LATTICE"):
        read_lattice(other)


@pytest.mark.skipif(not reference_available(), reason="needs the reference checkout")
def test_cache_identity_matches_reference(tmp_path):
    from harsh4b_b200.lattice import cache_identity

    sys.path.insert(0, str(REFERENCE_ROOT))
    try:
        import cpu_lightspark
    finally:
        sys.path.remove(str(REFERENCE_ROOT))
    path = tmp_path / "model.lat.pt"
    path.write_bytes(b"checkpoint bytes")
    assert cache_identity(path) == cpu_lightspark._cache_identity(path)


def test_reference_style_cache_without_norms_is_rejected_clearly(tmp_path):
    """A cache written the way the reference writes it (no norm vectors)
    cannot build a model on its own; the error names the way that works."""
    from harsh4b_b200.cache import read_cache, write_cache
    from harsh4b_b200.synthetic import synthetic_checkpoint, tiny_config

    checkpoint = synthetic_checkpoint(tiny_config(num_hidden_layers=1), seed=1)
    checkpoint.norms = {}
    write_cache(tmp_path, checkpoint)
    loaded = read_cache(tmp_path)
    assert loaded.norms == {}
    from harsh4b_b200.model import CudaQwen

    with pytest.raises(ValueError, match="build_b200_model"):
        CudaQwen.from_checkpoint(loaded)
