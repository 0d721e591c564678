"""GPU parity of the format kernels against the oracle: bit-exact (byte/integer work)."""

import numpy as np
import pytest
import torch

import mxfp4_ref as o
from _util import golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mx():
    import mxfp4_b200

    return mxfp4_b200


@pytest.fixture(scope="module")
def g():
    return golden()


def test_quantize_ref_rule_matches_reference_vectors(mx, g):
    tags = sorted({k[:-2] for k in g.files if k.startswith("q_") and k.endswith("_x")})
    for tag in tags:
        ax = 0 if tag.endswith("ax0") else -1
        p, s = mx.quantize_mxfp4(g[tag + "_x"], axis=ax)
        np.testing.assert_array_equal(p, g[tag + "_p"], err_msg=tag)
        np.testing.assert_array_equal(s, g[tag + "_s"], err_msg=tag)


@pytest.mark.parametrize("rule", ["ref", "ocp"])
@pytest.mark.parametrize("axis", [0, 1])
def test_quantize_random_matches_oracle(mx, rule, axis):
    rng = np.random.default_rng(7)
    x = rng.standard_normal((512, 384), dtype=np.float32) * np.exp2(
        rng.integers(-20, 20, size=(512, 384))
    ).astype(np.float32)
    x[:64] *= np.float32(0.02)
    q = o.quantize_mxfp4 if rule == "ref" else o.quantize_mxfp4_ocp
    pr, sr = q(x, axis=axis)
    p, s = mx.quantize_mxfp4(x, axis=axis, rule=rule)
    np.testing.assert_array_equal(s, sr)
    np.testing.assert_array_equal(p, pr)


def _bits_equal_nan_aware(out_f32: np.ndarray, ref_f32: np.ndarray):
    nan = np.isnan(ref_f32)
    np.testing.assert_array_equal(np.isnan(out_f32), nan)
    np.testing.assert_array_equal(out_f32.view(np.uint32)[~nan], ref_f32.view(np.uint32)[~nan])


def test_dequantize_every_scale_byte_bit_exact(mx, g):
    ref = g["dq_out"]
    d32 = mx.dequantize_mxfp4(g["dq_p"], g["dq_s"], axis=0)
    _bits_equal_nan_aware(d32, ref)
    d16 = mx.dequantize_mxfp4(torch.from_numpy(g["dq_p"]), torch.from_numpy(g["dq_s"]), axis=0,
                              dtype=torch.bfloat16)
    ref16 = o.f32_to_bf16_bits(ref)
    got16 = d16.view(torch.int16).cpu().numpy().view(np.uint16)
    nan = np.isnan(ref)
    np.testing.assert_array_equal(got16[~nan], ref16[~nan])
    assert np.isnan(d16.float().cpu().numpy()[nan]).all()


def test_dequantize_nk_layout(mx):
    rng = np.random.default_rng(11)
    N, K = 96, 256
    p = rng.integers(0, 256, size=(N, K // 2), dtype=np.uint8)
    s = rng.integers(90, 160, size=(N, K // 32), dtype=np.uint8)
    _bits_equal_nan_aware(mx.dequantize_mxfp4(p, s, axis=-1), o.dequantize_mxfp4(p, s, axis=-1))


@pytest.mark.parametrize("N,K", [(256, 128), (200, 96), (3072, 3072), (136, 64)])
def test_prepack_matches_host_layout(mx, N, K):
    rng = np.random.default_rng(N + K)
    Bp = rng.integers(0, 256, size=(K // 2, N), dtype=np.uint8)
    Bs = rng.integers(0, 256, size=(K // 32, N), dtype=np.uint8)
    want = o.b200_prepack(Bp, Bs).reshape(-1)
    w = mx.prepack_b200(Bp, Bs, layout="ref")
    np.testing.assert_array_equal(w.data.cpu().numpy(), want)
    # the same weights given row-major ([N, K/2]) and in the strategy-G layout
    w2 = mx.prepack_b200(np.ascontiguousarray(Bp.T), np.ascontiguousarray(Bs.T), layout="nk")
    np.testing.assert_array_equal(w2.data.cpu().numpy(), want)
    if N % 128 == 0:
        gp, gs = o.prepack_b_mxfp4(Bp, Bs)
        w3 = mx.prepack_b200(gp, gs, layout="g", N=N, K=K)
        np.testing.assert_array_equal(w3.data.cpu().numpy(), want)


def test_gemm_dequant_tile_bit_exact(mx, g):
    """The bf16 tile the tensor-core kernel feeds the MMA equals the reference dequant."""
    for Bp, Bs in ((g["dq_p"], g["dq_s"]),
                   o.quantize_mxfp4_ocp(np.random.default_rng(5).standard_normal((3072, 384),
                                                                              dtype=np.float32) * 0.02, axis=0)):
        w = mx.prepack_b200(Bp, Bs)
        got = mx.dequantize_prepacked(w).view(torch.int16).cpu().numpy().view(np.uint16)  # [N, K]
        ref = o.dequantize_mxfp4(Bp, Bs, axis=0).T  # [N, K]
        ref16 = o.f32_to_bf16_bits(np.ascontiguousarray(ref))
        nan = np.isnan(ref)
        np.testing.assert_array_equal(got[~nan], ref16[~nan])
        assert ((got[nan] & 0x7F80) == 0x7F80).all() and ((got[nan] & 0x7F) != 0).all()


def test_prepacked_dequant_matches_plain_dequant_large(mx):
    """Full-size property: LUT dequant == plain dequant on a decode gate+up sized weight."""
    N, K = 57344, 8192
    gen = torch.Generator(device="cuda").manual_seed(0)
    Bp = torch.randint(0, 256, (K // 2, N), dtype=torch.uint8, device="cuda", generator=gen)
    Bs = torch.randint(100, 140, (K // 32, N), dtype=torch.uint8, device="cuda", generator=gen)
    w = mx.prepack_b200(Bp, Bs)
    a = mx.dequantize_prepacked(w)
    b = mx.dequantize_mxfp4(Bp, Bs, axis=0, dtype=torch.bfloat16)
    assert torch.equal(a.view(torch.int16), b.t().contiguous().view(torch.int16))
