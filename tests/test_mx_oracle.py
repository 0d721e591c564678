"""CPU tests of the block-scaled (MXFP8 x MXFP4) path's oracle: the E4M3 codec pinned against
torch.float8_e4m3fn, the OCP scale rule on known answers, and the two layout restatements."""

import numpy as np
import torch

import mxfp4_ref as o


def test_e4m3_decode_matches_torch():
    v = o.e4m3_values()
    t = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(np.isnan(v), np.isnan(t))
    assert np.array_equal(v[~np.isnan(v)], t[~np.isnan(t)])


def test_e4m3_encode_matches_torch_including_ties():
    v = o.e4m3_values()[:127]
    mids = (v[:-1] + v[1:]) / 2  # exact midpoints: the round-to-nearest-even ties
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(100000).astype(np.float32) * 40, mids, -mids, v, -v,
                        np.float32([0.0, -0.0, 1e-9, -1e-9, 2.0**-10, 3 * 2.0**-11])]).astype(np.float32)
    x = x[np.abs(x) <= 448]  # torch maps out-of-range values to NaN; the cvt rule saturates
    ours = o.encode_e4m3(x)
    ref = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(ours, ref)


def test_e4m3_saturates():
    assert o.encode_e4m3(np.float32([449, 464, 500, 1e30])).tolist() == [0x7E] * 4
    assert o.encode_e4m3(np.float32([-449, -1e30])).tolist() == [0xFE] * 2


def test_act_quant_known_answers():
    c, s = o.quantize_act_mx8(np.ones((1, 32), np.float32))
    assert s.tolist() == [[127 - 8]] and (c == 0x78).all()  # 1 = 256 * 2**-8, 256 = code 0x78
    c, s = o.quantize_act_mx8(np.zeros((2, 64), np.float32))
    assert (s == 0).all() and (c == 0).all()
    x = np.zeros((1, 32), np.float32)
    x[0, 0], x[0, 1] = 448.0, -1.0  # floor(log2 448) = 8: scale 2**0, 448 -> 0x7E
    c, s = o.quantize_act_mx8(x)
    assert s[0, 0] == 127 and c[0, 0] == 0x7E and c[0, 1] == 0xB8
    x[0, 0] = 511.0  # floor(log2 511) = 8, 511 saturates to 448
    c, s = o.quantize_act_mx8(x)
    assert s[0, 0] == 127 and c[0, 0] == 0x7E


def test_act_quant_error_bound():
    rng = np.random.default_rng(1)
    A = rng.standard_normal((64, 256)).astype(np.float32)
    c, s = o.quantize_act_mx8(A)
    d = o.dequantize_act_mx8(c, s)
    g = np.abs(A).reshape(64, 8, 32).max(-1, keepdims=True)
    err = np.abs(d - A).reshape(64, 8, 32)
    e = s.astype(np.float64)[..., None] - 127
    sat = np.abs(A).reshape(64, 8, 32) * np.exp2(-e) > 448
    # 3 mantissa bits: half an ulp of the group max's binade bounds the error of every element
    # that does not saturate; a saturated one (scaled value in (448, 512)) is off by < 1/8
    assert (err[~sat] <= np.broadcast_to(g, err.shape)[~sat] * 2.0**-4).all()
    assert (err[sat] < np.broadcast_to(g, err.shape)[sat] / 8).all()


def test_mx_weight_layout_roundtrip():
    rng = np.random.default_rng(2)
    K, N = 224, 200  # K not a multiple of 128, N not a multiple of 128
    Bp = rng.integers(0, 256, size=(K // 2, N), dtype=np.uint8)
    Bs = rng.integers(100, 150, size=(K // 32, N), dtype=np.uint8)
    flat = o.mx_weight_layout(Bp, Bs)
    Np, Kp = 256, 256
    data = flat[: Np * Kp // 2].reshape(Np, Kp // 2)
    sf = flat[Np * Kp // 2:].reshape(Np // 128, Kp // 128, 512)
    assert flat.size == Np * Kp // 2 + Np * Kp // 32
    assert np.array_equal(data[:N, : K // 2], Bp.T) and (data[N:] == 0).all() and (data[:, K // 2:] == 0).all()
    r, j = np.meshgrid(np.arange(128), np.arange(4), indexing="ij")
    assert sorted(o.mx_sf_in_block(r, j).ravel().tolist()) == list(range(512))  # a bijection
    for n in (0, 31, 32, 100, 127, 128, 199, 200, 255):
        for g in range(Kp // 32):
            want = Bs[g, n] if (n < N and g < K // 32) else 127
            assert sf[n // 128, g // 4, o.mx_sf_in_block(n % 128, g % 4)] == want


def test_mx_act_layout():
    rng = np.random.default_rng(3)
    A = rng.standard_normal((300, 160)).astype(np.float32)
    c, s = o.quantize_act_mx8(A)
    codes, blocks = o.mx_act_layout(c, s)
    assert codes.shape == (300, 256) and blocks.shape == (2, 512 // 128, 512)
    assert np.array_equal(codes[:, :160], c) and (codes[:, 160:] == 0).all()
    for m in (0, 31, 32, 127, 128, 255, 299, 300, 511):
        for g in range(8):
            want = s[m, g] if (m < 300 and g < 5) else 0
            assert blocks[g // 4, m // 128, o.mx_sf_in_block(m % 128, g % 4)] == want


def test_ref_gemm_mx_close_to_exact():
    rng = np.random.default_rng(4)
    A = rng.standard_normal((16, 128)).astype(np.float32)
    Bp, Bs = o.quantize_mxfp4_ocp(rng.standard_normal((128, 64)).astype(np.float32) * 0.02, axis=0)
    exact = A @ o.dequantize_mxfp4(Bp, Bs, axis=0)
    mx = o.ref_gemm_mx(A, Bp, Bs)
    assert np.max(np.abs(mx - exact)) / np.max(np.abs(exact)) < 0.05
