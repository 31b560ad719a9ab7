"""CPU restatement of the LATTICE -> row-int4 conversion -- TEST
INFRASTRUCTURE ONLY (only tests/ import it, as the checker of
``harsh4b_b200.lattice`` / ``csrc/lattice.cu``).

Follows the reference step by step:

* :func:`expand_t1` -- ``MLX/lattice_model.py:160-185`` (compact T1 codes of
  the mode-0/1 columns back to a dense per-row 2-bit plane);
* :func:`reconstruct` -- the fp32 weight of ``_convert_projection``
  (``cpu_lightspark.py:172-188``): mu + a0 * trit(T0) + [mode == o2] * a1 *
  trit(T1), added in that order;
* :func:`convert_projection` -- the rotation ``L^T W R^T`` per row in fp32 (as
  numpy evaluates it) and the row int4 quantisation (``:189-195``);
* :func:`convert_rows` -- ``_convert_embedding`` (``:204-229``).

Pinned by ``tests/golden/lattice_cases.npz``, written by
``tests/golden/make_lattice_golden.py`` from the reference's own functions.
"""
from __future__ import annotations

import numpy as np

TRIT = np.array([0.0, 1.0, -1.0, 0.0], dtype=np.float32)


def unpack_codes(codes: np.ndarray, width: int) -> np.ndarray:
    """Four 2-bit codes per byte, code j in bits 2(j % 4) of byte j // 4."""
    codes = np.asarray(codes, dtype=np.uint8)
    out = np.empty((codes.shape[0], codes.shape[1] * 4), dtype=np.uint8)
    for s in range(4):
        out[:, s::4] = (codes >> np.uint8(2 * s)) & np.uint8(3)
    return out[:, :width]


def pack_codes(codes: np.ndarray) -> np.ndarray:
    codes = np.asarray(codes, dtype=np.uint8)
    pad = (-codes.shape[1]) % 4
    if pad:
        codes = np.concatenate([codes, np.zeros((codes.shape[0], pad), dtype=np.uint8)], axis=1)
    out = np.zeros((codes.shape[0], codes.shape[1] // 4), dtype=np.uint8)
    for s in range(4):
        out |= codes[:, s::4] << np.uint8(2 * s)
    return out


def expand_t1(shape, maskid, t1c, n_t1) -> np.ndarray:
    """Dense per-row T1 codes (0 where the mode id is 2 or 3)."""
    rows, width = shape
    modes = unpack_codes(maskid, width)
    selected = modes < 2
    count = int(selected.sum())
    t1c = np.asarray(t1c, dtype=np.uint8).reshape(-1)
    if count != int(n_t1) or (count + 3) // 4 > t1c.size:
        raise ValueError("T1 count does not match mask IDs")
    index = np.arange(count, dtype=np.int64)
    flat = (t1c[index >> 2] >> ((index & 3) * 2).astype(np.uint8)) & np.uint8(3)
    dense = np.zeros((rows, width), dtype=np.uint8)
    dense[selected] = flat  # boolean assignment walks the rows in row-major order
    return pack_codes(dense)


def reconstruct(packed: dict) -> np.ndarray:
    """The fp32 LATTICE weight before rotation."""
    rows, width = (int(v) for v in packed["shape"])
    blocksize = int(packed["blocksize"])
    modes = unpack_codes(packed["maskid"], width).astype(np.int64)
    code0 = unpack_codes(packed["T0"], width)
    code1 = unpack_codes(expand_t1((rows, width), packed["maskid"], packed["T1c"], packed["n_T1"]), width)
    blocks = np.arange(width, dtype=np.int64)[None, :] // blocksize
    r = np.arange(rows, dtype=np.int64)[:, None]
    mu, a0, a1 = (np.asarray(packed[k]) for k in ("mu", "a0", "a1"))
    weight = mu[modes, r, blocks].astype(np.float32)
    weight = weight + a0[modes, r, blocks].astype(np.float32) * TRIT[code0]
    for index, mode in enumerate(int(x) for x in np.asarray(packed["o2_idx"]).reshape(-1)):
        term = np.where(modes == mode, a1[index, r, blocks].astype(np.float32), np.float32(0.0)) * TRIT[code1]
        weight = weight + term
    return weight.astype(np.float32)


def quantize_rows(weight: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Row scale max(max|w|, 1e-8) / 7 and codes clip(rint(w / scale), -7, 7),
    packed two per byte (low nibble = even column)."""
    weight = np.asarray(weight, dtype=np.float32)
    scale = np.maximum(np.max(np.abs(weight), axis=1), np.float32(1e-8)) / np.float32(7.0)
    codes = np.rint(weight / scale[:, None]).clip(-7, 7).astype(np.int8)
    packed = (codes[:, 0::2].view(np.uint8) & np.uint8(15)) | ((codes[:, 1::2].view(np.uint8) & np.uint8(15)) << 4)
    return packed.astype(np.uint8), scale.astype(np.float32)


def rotate(weight: np.ndarray, left, right, exact: bool = False) -> np.ndarray:
    """left^T W_r right^T per row (W_r = the row as dim_l x dim_r), in fp32 as
    the reference evaluates it, or in fp64 rounded once (``exact``)."""
    left = np.asarray(left, dtype=np.float32)
    right = np.asarray(right, dtype=np.float32)
    rows, width = weight.shape
    dl, dr = left.shape[0], right.shape[0]
    w = weight.reshape(rows, dl, dr)
    if exact:
        out = left.T.astype(np.float64) @ w.astype(np.float64) @ right.T.astype(np.float64)
    else:
        out = left.T @ w @ right.T
    return out.reshape(rows, width).astype(np.float32)


def convert_projection(packed: dict, left, right, exact: bool = False) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """(packed uint8[rows, width/2], scales float32[rows], rotated fp32 weight)."""
    weight = rotate(reconstruct(packed), left, right, exact=exact)
    codes, scales = quantize_rows(weight)
    return codes, scales, weight


def convert_rows(source) -> tuple[np.ndarray, np.ndarray]:
    """``_convert_embedding``: per-row symmetric int4 of a dense matrix."""
    return quantize_rows(np.asarray(source).astype(np.float32))


def synthetic_projection(rng: np.random.Generator, rows: int, width: int, blocksize: int = 64,
                         o2=(0, 1), half: bool = True) -> dict:
    """A random LATTICE projection in the checkpoint's field layout (compact T1)."""
    nblocks = (width + blocksize - 1) // blocksize
    modes = rng.integers(0, 4, (rows, width), dtype=np.uint8)
    c0 = rng.integers(0, 4, (rows, width), dtype=np.uint8)
    c1 = rng.integers(0, 4, (rows, width), dtype=np.uint8)
    selected = c1[modes < 2]
    dtype = np.float16 if half else np.float32
    return {
        "shape": (rows, width), "blocksize": blocksize, "nblocks": nblocks,
        "maskid": pack_codes(modes), "T0": pack_codes(c0), "T1c": pack_codes(selected.reshape(1, -1)).reshape(-1),
        "n_T1": int(selected.size), "o2_idx": np.array(o2, dtype=np.int64),
        "mu": (rng.standard_normal((4, rows, nblocks)) * 0.02).astype(dtype),
        "a0": (rng.standard_normal((4, rows, nblocks)) * 0.02).astype(dtype),
        "a1": (rng.standard_normal((len(o2), rows, nblocks)) * 0.01).astype(dtype),
    }


def orthogonal(rng: np.random.Generator, n: int) -> np.ndarray:
    q, r = np.linalg.qr(rng.standard_normal((n, n)))
    return (q * np.sign(np.diag(r))).astype(np.float32)
