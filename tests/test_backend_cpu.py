"""Host-side logic of the ``cuda`` backend that needs no GPU: the reference's
route validation and the f32 -> bf16 token conversion."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import q4nx as q
from raon_npu_b200.backend import _bf16_input, check_moe_routes


def test_route_validation_accepts_reference_shapes():
    ids = np.array([[3, 1, 7], [0, 5, 2]], np.int64)
    w = np.ones((2, 3), np.float32)
    i32, w32 = check_moe_routes(ids, w, 8, 3, tokens=2)
    assert i32.dtype == np.int32 and np.array_equal(i32, ids) and w32 is w


@pytest.mark.parametrize("ids,w,msg", [
    (np.array([[3, 3, 7]]), np.ones((1, 3), np.float32), "distinct"),
    (np.array([[3, 8, 7]]), np.ones((1, 3), np.float32), "0..7"),
    (np.array([[-1, 2, 7]]), np.ones((1, 3), np.float32), "0..7"),
    (np.array([[3.0, 2.0, 7.0]]), np.ones((1, 3), np.float32), "integer"),
    (np.array([[3, 2, 7]]), np.ones((1, 3), np.float64), "float32"),
    (np.array([[3, 2, 7]]), np.ones((1, 2), np.float32), "float32"),
])
def test_route_validation_rejects(ids, w, msg):
    with pytest.raises(ValueError, match=msg):
        check_moe_routes(ids, w, 8, 3)


def test_route_validation_token_count_and_k():
    with pytest.raises(ValueError):
        check_moe_routes(np.zeros((2, 3), np.int64) + [[0, 1, 2]], np.ones((2, 3), np.float32), 8, 3, tokens=3)
    with pytest.raises(ValueError):
        check_moe_routes(np.arange(17)[None], np.ones((1, 17), np.float32), 32, 17)


def test_bf16_input_rounds_f32_like_the_reference():
    rng = np.random.default_rng(0)
    xf = rng.standard_normal(256).astype(np.float32)
    xf[5] = np.nan
    got = _bf16_input(xf, 256, "x")
    np.testing.assert_array_equal(got, q.f32_to_bf16(xf))
    assert got[5] == 0x7FC0
    u = q.f32_to_bf16(xf)
    assert _bf16_input(u, 256, "x") is u
    with pytest.raises(ValueError):
        _bf16_input(xf[:10], 256, "x")
    with pytest.raises(ValueError):
        _bf16_input(xf.astype(np.float64), 256, "x")
