"""The bfp16ebs8 oracle against fixtures made by the reference's own code.

``tests/golden/bfp16.npz`` holds, for seeded matrices, the reference codec's
encoding (``quant/bfp16.py`` ``bfp16ebs8_encode``), its GEMV packing and
parse (``pack_bfp16_gemv`` / ``parse_bfp16_gemv_raw``) and its bit-level GEMV
model (``kernels/gemv_bfp16/reference.py`` ``bfp16_gemv_bit_reference``).
The oracle must reproduce each byte for byte; it is what a GPU path for the
format is checked against.
"""

from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np
import pytest

from oracle import bfp16 as b
from tests.golden.cases import BFP16_CASES, bfp16_input

GOLD = np.load(Path(__file__).parent / "golden" / "bfp16.npz")


def _sha(x) -> str:
    return hashlib.sha256(x if isinstance(x, bytes) else np.ascontiguousarray(x).tobytes()).hexdigest()


@pytest.mark.parametrize("name", list(BFP16_CASES))
def test_codec_and_layout_match_reference(name):
    n, k, seed, kind, t = BFP16_CASES[name]
    w, _ = bfp16_input(n, k, seed, kind, t)
    e, m = b.encode(w)
    # the codec's 9-byte records: exponent byte, then 8 mantissa bytes
    rec = np.concatenate([e[..., None], m.view(np.uint8)], axis=-1)
    assert _sha(rec) == str(GOLD[f"{name}/encode_sha"])
    packed = b.pack_gemv(w)
    assert len(packed) == n * k * 9 // 8
    assert _sha(packed) == str(GOLD[f"{name}/packed_sha"])
    pe, pm = b.parse_gemv(packed, K=k, M=n)
    np.testing.assert_array_equal(pe, GOLD[f"{name}/exponents"])
    assert _sha(pm) == str(GOLD[f"{name}/mantissas_sha"])
    fe, fm = b.flush_tiny(e, m)
    np.testing.assert_array_equal(pe, fe)
    np.testing.assert_array_equal(pm, fm.reshape(n, k))
    assert int(np.count_nonzero((e < b.E_MIN) & (m != 0).any(-1))) == int(GOLD[f"{name}/flushed"])


@pytest.mark.parametrize("name", list(BFP16_CASES))
def test_gemv_matches_reference_bits(name):
    n, k, seed, kind, t = BFP16_CASES[name]
    w, x = bfp16_input(n, k, seed, kind, t)
    e, m = b.parse_gemv(b.pack_gemv(w), K=k, M=n)
    y = np.stack([b.gemv(e, m, x[i]) for i in range(t)])
    np.testing.assert_array_equal(y, GOLD[f"{name}/y"])


def test_decode_is_mantissa_times_power_of_two():
    e = np.array([[7, 133, 140]], np.uint8)
    m = np.tile(np.array([-128, -1, 0, 1, 2, 64, 127, 5], np.int8), (1, 3, 1))
    d = b.decode(e, m)
    assert d[0, 1, 0] == -128.0 and d[0, 1, 3] == 1.0 and d[0, 2, 6] == 127.0 * 128
    assert d[0, 0, 3] == np.float32(2.0 ** -126)


def test_encode_carry_and_negative_limit():
    w = np.array([[1.9999] * 8 + [-1.9999] * 8], np.float32)
    e, m = b.encode(w)
    assert e[0, 0] == 128 and m[0, 0, 0] == 64       # +128 would not fit: exponent + 1
    assert e[0, 1] == 127 and m[0, 1, 0] == -128     # -128 fits
