"""Fixed-point rows, the decode FFN's operand format, on the CPU: the
oracle's encoder against the properties the CUDA kernels rely on.

* every group's integers fit the byte planes and the largest one lands in the
  top binade pair, so each value is held to half a step of 2^e;
* the byte layout decodes back to the integers;
* the int32 trick that turns a group's integer dot product into a float
  (M + v read as a float, minus M) is exact over the whole range the
  encoding allows, including the worst case of all nibbles 0 (weight -8)
  against all integers at the limit.
"""
import numpy as np
import pytest

from oracle import moe_oracle as O


def _rows(seed, rows, K, scales):
    rng = np.random.default_rng(seed)
    v = rng.standard_normal((rows, K)).astype(np.float32)
    return (v * np.asarray(scales, dtype=np.float32)[:, None]).astype(np.float32)


@pytest.mark.parametrize("G", [32, 64])
def test_fx_encoding_bounds_and_round_trip(G):
    amax, _, _ = O.fx_limits(G)
    scales = [1.0, 1e-3, 1e5, 3e-20, 7e25, 0.0, 1.0, 2.5]
    v = _rows(1, len(scales), 512, scales)
    v[6, 5] = 1e6  # one outlier: its group takes a large exponent, the others keep theirs
    A, e, q, consts, bad = O.fx_encode_rows(v, G)
    assert not bad.any()
    assert np.array_equal(O.fx_decode_q(q), A)
    assert np.abs(A).max() <= amax
    Ag = np.abs(A.reshape(len(scales), -1, G)).max(-1)
    nz = Ag > 0
    assert np.all(Ag[nz] >= (amax + 1) // 2), "the group maximum uses the top two binades"
    # each value held to half a step of its group's 2^e
    step = np.exp2(e.astype(np.float64))
    err = np.abs(A.reshape(len(scales), -1, G) * step[..., None] - v.reshape(len(scales), -1, G).astype(np.float64))
    assert np.all(err <= 0.5 * step[..., None] * (1 + 1e-12))
    # constants: M is the float 1.5 * 2^(23 + e), C0 = M - 8 sum(A)
    M = consts[..., 1].astype(np.uint32).view(np.float32).astype(np.float64)
    assert np.array_equal(M, 1.5 * np.exp2(23.0 + e))
    assert np.array_equal(consts[..., 0], consts[..., 1] - 8 * A.reshape(len(scales), -1, G).sum(-1))


@pytest.mark.parametrize("G", [32, 64])
def test_fx_group_dot_is_exact(G):
    amax, _, _ = O.fx_limits(G)
    rng = np.random.default_rng(2)
    for trial in range(200):
        scale = float(np.exp2(rng.integers(-60, 60)))
        v = (rng.standard_normal((1, G)) * scale).astype(np.float32)
        n = rng.integers(0, 16, G)
        A, e, _, consts, _ = O.fx_encode_rows(v, G)
        got = O.fx_group_dot(n, A[0], consts[0, 0])
        want = float(((n - 8) * A[0].astype(np.int64)).sum()) * 2.0 ** float(e[0, 0])
        assert float(got) == want, (trial, got, want)
    # the extremes of the range: every weight -8 (nibble 0) against every
    # integer at +-amax, at the smallest and largest exponents
    for sign in (1, -1):
        for e0 in (O.FX_MIN_EXP, 0, O.FX_MAX_EXP):
            A = np.full(G, sign * amax, dtype=np.int64)
            M = O.FX_MAGIC + e0 * (1 << 23)
            consts = np.array([M - 8 * A.sum(), M], dtype=np.int64)
            got = O.fx_group_dot(np.zeros(G, dtype=np.int64), A, consts)
            assert float(got) == -8.0 * sign * amax * G * 2.0 ** e0


def test_fx_flags_values_it_cannot_hold():
    v = np.ones((4, 64), dtype=np.float32)
    v[0, 3] = np.inf
    v[1, 7] = np.nan
    v[2, 9] = 1e36  # beyond 8191 * 2^100
    A, e, _, _, bad = O.fx_encode_rows(v, 64)
    assert bad[:3, 0].all() and not bad[3, 0]
    assert e[0, 0] == O.FX_MAX_EXP and A[0, 3] == 8191   # infinity clamps to the largest integer
    assert A[1, 7] == 0 and e[1, 0] == e[3, 0]           # NaN encodes as 0; the max ignores it
    assert e[2, 0] == O.FX_MAX_EXP and A[2, 9] == 8191
