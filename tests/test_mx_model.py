"""CPU model of the block-scaled kernels' index arithmetic (gemm_mx.cuh): the tile and
stream-K schedules, the scale-block offsets the producers load, and the epilogues' hi + lo
column mapping, run on the oracle's byte layouts.  It checks that the layouts and the kernels'
offset formulas agree with each other and with oracle.ref_gemm_mx; the tensor-core MMA itself
is modelled as an fp64 matrix product of the decoded tiles."""

import numpy as np
import pytest

import mxfp4_ref as o
from _util import make_case

BK = 128


def _e2m1(nib):
    mag = o.E2M1_MAGNITUDES[nib & 7].astype(np.float64)
    return np.where(nib & 8, -mag, mag)


def _weight_tile(wflat, Np, Kp, nb, kt):
    """Decoded 128 x 128 weight tile (rows nb*128.., k kt*128..) from the MX weight layout."""
    data = wflat[: Np * Kp // 2].reshape(Np, Kp // 2)
    sf = wflat[Np * Kp // 2:].reshape(Np // 128, Kp // 128, 512)
    bytes_ = data[nb * 128:(nb + 1) * 128, kt * 64:(kt + 1) * 64]
    vals = np.empty((128, 128))
    vals[:, 0::2] = _e2m1(bytes_ & 0xF)
    vals[:, 1::2] = _e2m1(bytes_ >> 4)
    blk = sf[nb, kt]  # the kernel's sfa + (nb * k_steps + kt) * 512
    r = np.arange(128)
    for j in range(4):
        vals[:, 32 * j:32 * (j + 1)] *= np.exp2(blk[o.mx_sf_in_block(r, j)].astype(np.float64) - 127)[:, None]
    return vals


def _code_tile(codes, blocks, row0, nrows, kt, sf_block0):
    """Decoded code rows row0.. (nrows) at k kt*128.. with scales from blocks [kt][sf_block0 + r//128]."""
    v = o.e4m3_values()[codes[row0:row0 + nrows, kt * BK:(kt + 1) * BK]].astype(np.float64)
    r = np.arange(nrows)
    for j in range(4):
        s = blocks[kt, sf_block0 + r // 128, o.mx_sf_in_block(r % 128, j)].astype(np.float64)
        v[:, 32 * j:32 * (j + 1)] *= np.exp2(s - 127)[:, None]
    return v


def model_large(A, Bp, Bs, mode):
    M, K = A.shape
    N = Bp.shape[1]
    codes, blocks = o.mx_act_layout(A, mode)
    wflat = o.mx_weight_layout(Bp, Bs)
    Np, Kp = -(-N // 128) * 128, -(-K // BK) * BK
    rows = codes.shape[0]
    m_blocks, n_blocks, k_steps = rows // 256, Np // 128, Kp // BK
    sf_rows = 2 * m_blocks  # the kernel's sf_rows
    act_rows = 128 if mode == o.MX_SPLIT2 else 256
    out = np.zeros((M, N))
    for mb in range(m_blocks):
        for nb in range(n_blocks):
            D = np.zeros((128, 256))
            for kt in range(k_steps):
                w = _weight_tile(wflat, Np, Kp, nb, kt)
                b = _code_tile(codes, blocks.reshape(k_steps, sf_rows, 512), mb * 256, 256, kt, 2 * mb)
                D += w @ b.T
            if mode == o.MX_SPLIT2:
                tile = (D[:, :128] + D[:, 128:]).T  # epilogue: hi columns + lo columns 128 further
            else:
                tile = D.T
            m0, n0 = mb * act_rows, nb * 128
            mm, nn = min(act_rows, M - m0), min(128, N - n0)
            if mm > 0 and nn > 0:
                out[m0:m0 + mm, n0:n0 + nn] = tile[:mm, :nn]
    return out


def model_decode(A, Bp, Bs, mode, grid):
    M, K = A.shape
    N = Bp.shape[1]
    assert M <= 16
    codes, blocks = o.mx_act_layout(A, mode)
    assert codes.shape[0] == 32 and blocks.shape[1] == 1
    wflat = o.mx_weight_layout(Bp, Bs)
    Np, Kp = -(-N // 128) * 128, -(-K // BK) * BK
    n_blocks, k_steps = Np // 128, Kp // BK
    total = n_blocks * k_steps
    ws = np.zeros((M, N))
    for c in range(grid):  # stream-K shares and segments, as gemv_mx_kernel computes them
        s0, s1 = total * c // grid, total * (c + 1) // grid
        s = s0
        while s < s1:
            nb = s // k_steps
            end = min(s1, (nb + 1) * k_steps)
            D = np.zeros((128, 32))
            for st in range(s, end):
                kt = st % k_steps
                D += _weight_tile(wflat, Np, Kp, nb, kt) @ _code_tile(codes, blocks, 0, 32, kt, 0).T
            for q in range(4):
                for lane in range(32):
                    n = nb * 128 + 32 * q + lane
                    if n < N:
                        ws[:, n] += D[32 * q + lane, :M] + D[32 * q + lane, 16:16 + M]
            s = end
    return ws


@pytest.mark.parametrize("mode", [o.MX_Q8, o.MX_SPLIT2])
@pytest.mark.parametrize("M,N,K", [(300, 200, 224), (40, 256, 384)])
def test_large_kernel_model(M, N, K, mode):
    A, Bp, Bs = make_case(M, N, K, seed=M + N)
    ref = o.ref_gemm_mx(A, Bp, Bs, mode)
    got = model_large(A, Bp, Bs, mode)
    assert np.max(np.abs(got - ref)) <= 1e-4 * np.max(np.abs(ref))


@pytest.mark.parametrize("mode", [o.MX_Q8, o.MX_SPLIT2])
@pytest.mark.parametrize("M,N,K,grid", [(1, 200, 384, 5), (16, 512, 256, 3), (7, 384, 640, 7)])
def test_decode_kernel_model(M, N, K, grid, mode):
    A, Bp, Bs = make_case(M, N, K, seed=M * N)
    ref = o.ref_gemm_mx(A, Bp, Bs, mode)
    got = model_decode(A, Bp, Bs, mode, grid)
    assert np.max(np.abs(got - ref)) <= 1e-4 * np.max(np.abs(ref))
