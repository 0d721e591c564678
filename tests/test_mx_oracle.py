"""CPU tests of the block-scaled (MXFP8 x MXFP4) path's oracle: the E4M3 codec pinned against
torch.float8_e4m3fn, the OCP scale rule on known answers, and the two layout restatements."""

import numpy as np
import pytest
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
    [(c, s)] = o.quantize_act_mx8(np.ones((1, 32), np.float32))
    assert s.tolist() == [[127 - 8]] and (c == 0x78).all()  # 1 = 256 * 2**-8, 256 = code 0x78
    [(c, s)] = o.quantize_act_mx8(np.zeros((2, 64), np.float32))
    assert (s == 0).all() and (c == 0).all()
    x = np.zeros((1, 32), np.float32)
    x[0, 0], x[0, 1] = 448.0, -1.0  # floor(log2 448) = 8: scale 2**0, 448 -> 0x7E
    [(c, s)] = o.quantize_act_mx8(x)
    assert s[0, 0] == 127 and c[0, 0] == 0x7E and c[0, 1] == 0xB8
    x[0, 0] = 511.0  # floor(log2 511) = 8, 511 saturates to 448
    [(c, s)] = o.quantize_act_mx8(x)
    assert s[0, 0] == 127 and c[0, 0] == 0x7E


def test_act_quant_error_bound():
    rng = np.random.default_rng(1)
    A = rng.standard_normal((64, 256)).astype(np.float32)
    [(c, s)] = o.quantize_act_mx8(A)
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


def _row_of(m, p, G):
    return m if G == 0 else (m // G) * 2 * G + p * G + m % G


@pytest.mark.parametrize("M,mode", [(1, o.MX_Q8), (16, o.MX_SPLIT2), (300, o.MX_Q8), (300, o.MX_SPLIT2)])
def test_mx_act_layout(M, mode):
    rng = np.random.default_rng(3)
    A = rng.standard_normal((M, 160)).astype(np.float32)
    pieces = o.quantize_act_mx8(A, mode)
    codes, blocks = o.mx_act_layout(A, mode)
    G, rows = o.mx_act_rows(M, mode)
    assert codes.shape == (rows, 256) and blocks.shape == (2, -(-rows // 128), 512)
    assert (codes[:, 160:] == 0).all()
    used = set()
    for p in range(2):
        for m in range(M):
            b = _row_of(m, p, G)
            if p < len(pieces):
                c, s = pieces[p]
                assert np.array_equal(codes[b, :160], c[m])
                for g in range(8):
                    want = s[m, g] if g < 5 else 0
                    assert blocks[g // 4, b // 128, o.mx_sf_in_block(b % 128, g % 4)] == want
            used.add(b)
    for b in set(range(-(-rows // 128) * 128)) - used:  # padding rows: zero codes and scales
        if b < rows:
            assert (codes[b] == 0).all()
        assert (blocks[:, b // 128, [o.mx_sf_in_block(b % 128, j) for j in range(4)]] == 0).all()


def test_split2_pieces():
    rng = np.random.default_rng(5)
    A = (rng.standard_normal((64, 256)) * np.exp2(rng.integers(-6, 6, size=(64, 256)))).astype(np.float32)
    A = o.bf16_bits_to_f32(o.f32_to_bf16_bits(A))
    (ch, sh), (cl, sl) = o.quantize_act_mx8(A, o.MX_SPLIT2)
    g = np.abs(A).reshape(64, 8, 32).max(-1)
    _, E = np.frexp(g)
    assert np.array_equal(sh.astype(int) - 127, np.where(g > 0, E - 1 - 7, -127))  # no saturation
    hi = o.dequantize_act_mx8(ch, sh)
    assert (np.abs(o.dequantize_act_mx8(ch, sh).reshape(64, 8, 32)) <= 256 * np.exp2(sh.astype(int) - 127)[..., None]).all()
    tot = o.dequantize_act_pieces([(ch, sh), (cl, sl)])
    err = np.abs(tot - A).reshape(64, 8, 32)
    # hi leaves at most 2**-4 of the group max; lo rounds that to 2**-4 of itself
    assert (err <= g[..., None] * 2.0**-8).all()
    assert np.abs(hi - A).max() > np.abs(tot - A).max()


def test_ref_gemm_split2_near_exact():
    rng = np.random.default_rng(6)
    A = o.bf16_bits_to_f32(o.f32_to_bf16_bits(rng.standard_normal((16, 512)).astype(np.float32)))
    Bp, Bs = o.quantize_mxfp4_ocp(rng.standard_normal((512, 128)).astype(np.float32) * 0.02, axis=0)
    exact = A @ o.dequantize_mxfp4(Bp, Bs, axis=0)
    split = o.ref_gemm_mx(A, Bp, Bs, o.MX_SPLIT2)
    assert np.max(np.abs(split - exact)) / np.max(np.abs(exact)) < 2e-3


def test_ref_gemm_mx_close_to_exact():
    rng = np.random.default_rng(4)
    A = rng.standard_normal((16, 128)).astype(np.float32)
    Bp, Bs = o.quantize_mxfp4_ocp(rng.standard_normal((128, 64)).astype(np.float32) * 0.02, axis=0)
    exact = A @ o.dequantize_mxfp4(Bp, Bs, axis=0)
    mx = o.ref_gemm_mx(A, Bp, Bs)
    assert np.max(np.abs(mx - exact)) / np.max(np.abs(exact)) < 0.05
