"""CPU tests: the oracle against the reference's golden vectors and known answers."""

import numpy as np
import pytest

import mxfp4_ref as o
from _util import golden


@pytest.fixture(scope="module")
def g():
    return golden()


def _cases(g):
    return sorted({k[:-2] for k in g.files if k.startswith("q_") and k.endswith("_x")})


def test_quantize_matches_reference_vectors(g):
    cases = _cases(g)
    assert len(cases) >= 10
    for tag in cases:
        ax = 0 if tag.endswith("ax0") else -1
        p, s = o.quantize_mxfp4(g[tag + "_x"], axis=ax)
        np.testing.assert_array_equal(p, g[tag + "_p"], err_msg=tag)
        np.testing.assert_array_equal(s, g[tag + "_s"], err_msg=tag)


def test_dequantize_matches_reference_vectors(g):
    d = o.dequantize_mxfp4(g["dq_p"], g["dq_s"], axis=0)
    r = g["dq_out"]
    nan = np.isnan(r)
    np.testing.assert_array_equal(np.isnan(d), nan)
    np.testing.assert_array_equal(d.view(np.uint32)[~nan], r.view(np.uint32)[~nan])


def test_ref_gemm_matches_reference_vectors(g):
    C = o.ref_gemm(g["gemm_A"], g["gemm_Bp"], g["gemm_Bs"])
    np.testing.assert_array_equal(C, g["gemm_C"])


def test_strategy_g_prepack_matches_reference_vectors(g):
    a, b = o.prepack_b_mxfp4(g["g_Bp"], g["g_Bs"])
    np.testing.assert_array_equal(a, g["g_prep"])
    np.testing.assert_array_equal(b, g["g_sprep"])


# the reference's own unit tests (tests/test_smoke.py), restated against the oracle
def test_roundtrip_zero():
    x = np.zeros((4, 32), dtype=np.float32)
    p, s = o.quantize_mxfp4(x, axis=-1)
    assert np.allclose(o.dequantize_mxfp4(p, s, axis=-1), x)


def test_roundtrip_small_values():
    x = np.random.default_rng(0).standard_normal((8, 64), dtype=np.float32)
    p, s = o.quantize_mxfp4(x, axis=-1)
    y = o.dequantize_mxfp4(p, s, axis=-1)
    assert p.shape == (8, 32) and s.shape == (8, 2)
    assert (np.abs(y - x) / (np.abs(x) + 1e-6)).mean() < 0.30


def test_packing_bit_layout_known_answer():
    p, s = o.quantize_mxfp4(np.array([[4.0, -4.0] * 16], dtype=np.float32), axis=-1)
    assert s[0, 0] == 127
    assert (p[0] == 0xE6).all()


def test_ref_gemm_shape_finite():
    rng = np.random.default_rng(1)
    A = rng.standard_normal((16, 32), dtype=np.float32)
    p, s = o.quantize_mxfp4(rng.standard_normal((32, 16), dtype=np.float32) * 0.1, axis=0)
    C = o.ref_gemm(A, p, s)
    assert C.shape == (16, 16) and np.isfinite(C).all()


# OCP MX quantiser: known answers written from the OCP MX v1.0 definition
def test_ocp_rne_ties_and_saturation():
    # block amax 4 -> exponent floor(log2 4) - 2 = 0, so values are quantised unscaled
    vals = np.array([4.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, -0.75, 0.3, 0.0], np.float32)
    x = np.zeros((1, 32), np.float32)
    x[0, : len(vals)] = vals
    p, s = o.quantize_mxfp4_ocp(x, axis=-1)
    assert s[0, 0] == 127
    d = o.dequantize_mxfp4(p, s, axis=-1)[0, : len(vals)]
    np.testing.assert_array_equal(d, [4.0, 0.0, 1.0, 1.0, 2.0, 2.0, 4.0, 4.0, -1.0, 0.5, 0.0])
    # amax 7 -> exponent 0 as well (floor(log2 7) = 2); 7 saturates to 6
    x2 = np.zeros((1, 32), np.float32)
    x2[0, 0], x2[0, 1] = 7.0, -6.5
    p2, s2 = o.quantize_mxfp4_ocp(x2, axis=-1)
    assert s2[0, 0] == 127
    np.testing.assert_array_equal(o.dequantize_mxfp4(p2, s2, axis=-1)[0, :2], [6.0, -6.0])


def test_ocp_exponent_exact_near_powers_of_two():
    below = np.nextafter(np.float32(8.0), np.float32(0.0))  # one ulp below 8
    x = np.zeros((1, 32), np.float32)
    x[0, 0] = below
    _, s = o.quantize_mxfp4_ocp(x, axis=-1)
    assert int(s[0, 0]) - 127 == 2 - 2  # floor(log2(8 - ulp)) = 2
    x[0, 0] = 8.0
    _, s = o.quantize_mxfp4_ocp(x, axis=-1)
    assert int(s[0, 0]) - 127 == 3 - 2


def test_ocp_zero_block():
    p, s = o.quantize_mxfp4_ocp(np.zeros((2, 64), np.float32), axis=-1)
    assert (s == 0).all() and (p == 0).all()


def test_b200_prepack_layout_roundtrip():
    rng = np.random.default_rng(3)
    K, N = 160, 200  # both ragged w.r.t. the 64 x 128 chunk
    Bp = rng.integers(0, 256, size=(K // 2, N), dtype=np.uint8)
    Bs = rng.integers(100, 150, size=(K // 32, N), dtype=np.uint8)
    P = o.b200_prepack(Bp, Bs)
    nb, kb = -(-N // 128), -(-K // 64)
    assert P.shape == (nb, kb, o.CHUNK_BYTES)
    # the offsets are a bijection onto the chunk
    r, g, p = np.meshgrid(np.arange(128), np.arange(2), np.arange(16), indexing="ij")
    offs = np.concatenate([o.chunk_data_offset(r, g, p % 4, p // 4).ravel(),
                           o.chunk_scale_offset(r[:, :, 0], g[:, :, 0]).ravel()])
    assert sorted(offs.tolist()) == list(range(o.CHUNK_BYTES))
    for n in (0, 5, 8, 15, 16, 127, 128, 199):
        for kp in (0, 3, 17, 31, 32, 79):
            c = P[n // 128, kp // 32]
            g, p = (kp % 32) // 16, kp % 16
            assert c[o.chunk_data_offset(n % 128, g, p % 4, p // 4)] == Bp[kp, n]
        for kg in range(K // 32):
            assert P[n // 128, kg // 2, o.chunk_scale_offset(n % 128, kg % 2)] == Bs[kg, n]
    # padding: rows beyond N and groups beyond K are zero nibbles with scale 127
    for r_ in range(200 - 128, 128):
        for g_ in range(2):
            assert (P[1, :, o.chunk_scale_offset(r_, g_)] == 127).all()
            assert (P[1, :, [o.chunk_data_offset(r_, g_, t, b) for t in range(4) for b in range(4)]] == 0).all()
    for r_ in range(128):
        assert (P[:, 2, o.chunk_scale_offset(r_, 1)] == 127).all()  # k group 5 (k >= 160) of chunk kb=2
