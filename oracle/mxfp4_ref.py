"""CPU oracle for the MXFP4 x BF16 GEMM path.  TEST INFRASTRUCTURE ONLY.

This module restates, in NumPy, the reference package's CPU algorithm
(konradha/cdna3-bench, ``python/mxfp4_cdna3/ref.py``).  It is the checker the
parity tests compare the CUDA path against, and the timed CPU baseline of
``bench.py``.  Nothing in the product package imports it; only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm do.

Parity is pinned: ``tests/test_oracle.py`` checks every function here against
golden vectors produced by importing the reference itself
(``tests/golden/make_golden.py``) and against the reference's own known-answer
tests (``tests/test_smoke.py`` of the reference: zero round trip, the
``[4,-4]*16 -> scale 127 / bytes 0xE6`` bit layout).

Formats (same bytes as the reference):
  * E2M1 nibble = sign<<3 | magnitude index, magnitudes {0,.5,1,1.5,2,3,4,6}.
  * Two nibbles per byte along the quantised axis: even element in the low
    nibble, odd element in the high nibble.
  * One E8M0 scale byte per 32 elements along the axis: value 2**(byte-127).
"""

from __future__ import annotations

import numpy as np

GROUP = 32
E2M1_MAGNITUDES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)

# Decision boundaries between consecutive E2M1 magnitudes (midpoints).
_MIDPOINTS = (E2M1_MAGNITUDES[1:] + E2M1_MAGNITUDES[:-1]) / 2.0


def _groups_last(x: np.ndarray, axis: int) -> tuple[np.ndarray, tuple[int, ...]]:
    x = np.moveaxis(x, axis, -1)
    lead = x.shape[:-1]
    if x.shape[-1] % GROUP:
        raise ValueError(f"axis {axis} length {x.shape[-1]} not divisible by {GROUP}")
    return x.reshape(*lead, x.shape[-1] // GROUP, GROUP), lead


def _pack_nibbles(nib: np.ndarray, lead, n_groups: int, axis: int) -> np.ndarray:
    nib = nib.reshape(*lead, n_groups * GROUP)
    packed = (nib[..., 0::2] & 0xF) | ((nib[..., 1::2] & 0xF) << 4)
    return np.ascontiguousarray(np.moveaxis(packed.astype(np.uint8), -1, axis))


def _nearest_index_ties_low(mag: np.ndarray) -> np.ndarray:
    """Index of the nearest E2M1 magnitude; an exact tie picks the LOWER one.

    Follows ``_nearest_e2m1`` (ref.py:6-11): ``argmin`` of the absolute
    difference returns the first (smallest) index on ties.  A value exactly on
    a midpoint therefore maps down: ``searchsorted(side='left')`` counts the
    midpoints strictly below ``mag``.
    """
    return np.searchsorted(_MIDPOINTS, mag, side="left").astype(np.uint8)


def quantize_mxfp4(x, axis=-1):
    """Reference quantiser (ref.py:14-47).

    scale exponent = ceil(log2(max(amax, 1e-38) / 6)) clipped to [-127, 127];
    elements are divided by 2**exp and mapped to the nearest E2M1 magnitude
    with ties to the lower magnitude.  Returns (packed uint8, scales uint8)
    with the quantised axis halved / divided by 32 respectively.
    """
    x = np.asarray(x, dtype=np.float32)
    g, lead = _groups_last(x, axis)
    amax = np.max(np.abs(g), axis=-1)
    e = np.clip(np.ceil(np.log2(np.maximum(amax, np.float32(1e-38)) / np.float32(6.0))), -127, 127)
    e = e.astype(np.int32)
    scaled = g / np.power(np.float32(2.0), e.astype(np.float32))[..., None]
    idx = _nearest_index_ties_low(np.abs(scaled))
    nib = idx | ((scaled < 0).astype(np.uint8) << 3)
    scales = np.ascontiguousarray(np.moveaxis((e + 127).astype(np.uint8), -1, axis))
    return _pack_nibbles(nib, lead, g.shape[-2], axis), scales


def _rne_index(mag: np.ndarray) -> np.ndarray:
    """Nearest E2M1 magnitude, ties to the even code (OCP MX round-to-nearest-even),
    saturating at 6."""
    lo = np.searchsorted(_MIDPOINTS, mag, side="left")  # ties -> lower
    hi = np.searchsorted(_MIDPOINTS, mag, side="right")  # ties -> upper
    tie = lo != hi
    # on a tie the two candidates are lo (code lo) and hi = lo + 1; pick the even code
    idx = np.where(tie & (lo % 2 == 1), hi, lo)
    return np.minimum(idx, 7).astype(np.uint8)


def quantize_mxfp4_ocp(x, axis=-1):
    """OCP MX v1.0 E2M1 quantiser (the rule the benchmark configs name).

    shared exponent = floor(log2(amax)) - 2 (2 = emax of E2M1), clipped to
    [-127, 127]; an all-zero block gets exponent -127.  Elements are divided by
    2**exp, rounded to nearest-even on the E2M1 grid and saturated at +-6.
    """
    x = np.asarray(x, dtype=np.float32)
    g, lead = _groups_last(x, axis)
    amax = np.max(np.abs(g), axis=-1)
    # floor(log2(amax)) computed exactly from the binary exponent (frexp: amax = m*2**E,
    # m in [0.5, 1)), so blocks whose amax sits one ulp below a power of two are not
    # rounded up by a float32 log2.
    _, E = np.frexp(amax)
    e = (E.astype(np.int64) - 1) - 2
    e = np.where(amax > 0, e, -127)
    e = np.clip(e, -127, 127).astype(np.int32)
    scaled = g / np.power(np.float32(2.0), e.astype(np.float32))[..., None]
    idx = _rne_index(np.abs(scaled))
    nib = idx | ((scaled < 0).astype(np.uint8) << 3)
    scales = np.ascontiguousarray(np.moveaxis((e + 127).astype(np.uint8), -1, axis))
    return _pack_nibbles(nib, lead, g.shape[-2], axis), scales


def dequantize_mxfp4(packed, scales, axis=-1):
    """Reference dequantiser (ref.py:50-72): value = (+-)E2M1[em] * 2**(scale-127) in fp32."""
    packed = np.moveaxis(np.asarray(packed, dtype=np.uint8), axis, -1)
    scales = np.moveaxis(np.asarray(scales, dtype=np.uint8), axis, -1)
    nib = np.empty((*packed.shape[:-1], packed.shape[-1] * 2), dtype=np.uint8)
    nib[..., 0::2] = packed & 0xF
    nib[..., 1::2] = packed >> 4
    val = E2M1_MAGNITUDES[nib & 7] * np.where(nib & 8, np.float32(-1.0), np.float32(1.0))
    with np.errstate(over="ignore", invalid="ignore"):
        mult = np.power(2.0, scales.astype(np.int32) - 127).astype(np.float32)
        lead = val.shape[:-1]
        out = val.reshape(*lead, -1, GROUP) * mult[..., None]
    return np.moveaxis(out.reshape(*lead, -1), -1, axis)


def ref_gemm(A, B_packed, B_scales):
    """Reference GEMM (ref.py:75-78): fp32 A @ dequant(B) with B = [K/2, N] / [K/32, N]."""
    A = np.asarray(A)
    A32 = A if A.dtype == np.float32 else A.astype(np.float32)
    return A32 @ dequantize_mxfp4(B_packed, B_scales, axis=0)


def preshuffle_b(B_packed, B_scales, N_tile=128, K_tile=128):
    """Identity placeholder kept for interface parity (ref.py:81-82)."""
    return np.ascontiguousarray(B_packed), np.ascontiguousarray(B_scales)


def prepack_b_mxfp4(B_packed, B_scales, n_tile=128):
    """Strategy-G prepack of the reference (ref.py:85-101).

    B_prep[nb, K/8, n_tile, 4] (byte b of each 4-byte word = K-byte 4*chunk+b),
    Bs_prep[nb, K/32, n_tile]; both returned flattened.
    """
    B_packed = np.ascontiguousarray(B_packed)
    K2, N = B_packed.shape
    if N % n_tile:
        raise AssertionError("N must be a multiple of n_tile")
    nb = N // n_tile
    bp = B_packed.reshape(K2 // 4, 4, nb, n_tile).transpose(2, 0, 3, 1)
    bs = np.ascontiguousarray(B_scales).reshape(-1, nb, n_tile).transpose(1, 0, 2)
    return np.ascontiguousarray(bp).reshape(-1), np.ascontiguousarray(bs).reshape(-1)


# --------------------------------------------------------------------------------------
# Helpers for the B200 library's own formats (restated on the host for the tests).
# --------------------------------------------------------------------------------------

CHUNK_ROWS = 128  # weight rows (output columns n) per chunk
CHUNK_K = 64  # K elements per chunk
CHUNK_DATA = CHUNK_ROWS * CHUNK_K // 2  # 4096 bytes of nibbles
CHUNK_BYTES = CHUNK_DATA + CHUNK_ROWS * (CHUNK_K // GROUP)  # + 256 scale bytes = 4352


def chunk_data_offset(r, grp, t, b):
    """Byte offset inside a 4352-byte chunk of weight row r (0..127), 32-group grp (0..1),
    word t (0..3) and byte b (0..3) of that row-group, where byte b of word t holds the
    nibble pair for k-pair t + 4*b of the group (low nibble = even k).

    The 16-byte unit of (k = r % 8, t) in the 32-unit block of rows 16a .. 16a+15 (a = r // 16)
    holds word t of (row 16a+k, group 0), (row 16a+k+8, group 0), (row 16a+k, group 1),
    (row 16a+k+8, group 1): the A-fragment words lane (k, t) of an m16n8k16 MMA needs.  It sits
    at unit position 32a + 8t + ((k + 2t) mod 8) (a placement free of shared-memory bank
    conflicts for both kernels' access patterns).
    """
    r = np.asarray(r)
    unit = 32 * (r >> 4) + 8 * t + (((r & 7) + 2 * t) & 7)
    word = 2 * grp + ((r >> 3) & 1)
    return unit * 16 + word * 4 + b


def chunk_scale_offset(r, grp):
    """Byte offset of the E8M0 scale of row r, group grp: 4-byte units 8*w + g after the data
    hold the scales of (row 16w+g, group 0), (16w+g+8, 0), (16w+g, 1), (16w+g+8, 1)."""
    r = np.asarray(r)
    return CHUNK_DATA + 4 * (8 * (r >> 4) + (r & 7)) + 2 * grp + ((r >> 3) & 1)


def b200_prepack(B_packed, B_scales):
    """Host restatement of the B200 prepacked weight layout (the GPU prepack's oracle).

    Input: reference layout B_packed [K/2, N], B_scales [K/32, N].  N is padded to a multiple
    of 128 and K to a multiple of 64 with zero nibbles and scale 127.  Output: uint8
    [N_pad/128, K_pad/64, 4352]; chunk (nb, kb) holds rows nb*128 .. +127 and k in
    kb*64 .. +63 placed by chunk_data_offset / chunk_scale_offset.
    """
    B_packed = np.asarray(B_packed, dtype=np.uint8)
    B_scales = np.asarray(B_scales, dtype=np.uint8)
    K2, N = B_packed.shape
    K = 2 * K2
    Np = -(-N // CHUNK_ROWS) * CHUNK_ROWS
    Kp = -(-K // CHUNK_K) * CHUNK_K
    bp = np.zeros((Kp // 2, Np), dtype=np.uint8)
    bp[:K2, :N] = B_packed
    bs = np.full((Kp // GROUP, Np), 127, dtype=np.uint8)
    bs[: K // GROUP, :N] = B_scales
    nb, kb = Np // CHUNK_ROWS, Kp // CHUNK_K
    d = bp.reshape(kb, 2, 16, nb, CHUNK_ROWS).transpose(3, 0, 4, 1, 2)  # [nb, kb, r, grp, pair]
    s = bs.reshape(kb, 2, nb, CHUNK_ROWS).transpose(2, 0, 3, 1)  # [nb, kb, r, grp]
    r, g, p = np.meshgrid(np.arange(CHUNK_ROWS), np.arange(2), np.arange(16), indexing="ij")
    doff = chunk_data_offset(r, g, p % 4, p // 4)  # pair p = t + 4*b
    r2, g2 = np.meshgrid(np.arange(CHUNK_ROWS), np.arange(2), indexing="ij")
    soff = chunk_scale_offset(r2, g2)
    out = np.empty((nb, kb, CHUNK_BYTES), dtype=np.uint8)
    out[:, :, doff.reshape(-1)] = d.reshape(nb, kb, -1)
    out[:, :, soff.reshape(-1)] = s.reshape(nb, kb, -1)
    return out


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns with round-to-nearest-even (NaN kept quiet)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------------------------------
# Block-scaled path (an extension with no reference counterpart).  The activations are
# quantised to OCP MXFP8 (E4M3 elements, one E8M0 scale per 32 k of a row) and the result is
# dequant(Q8(A)) @ dequant(W).  The E4M3 codec is pinned against torch.float8_e4m3fn in
# tests/test_oracle.py; the scale rule follows the OCP Microscaling Formats v1.0 spec:
# X = 2**(floor(log2(amax)) - emax_elem), emax_elem = 8 for E4M3 (largest normal 448 = 1.75 * 2**8).

E4M3_EMAX = 8
E4M3_MAX = 448.0
MX_BK = 128  # k per 128-row scale block (4 groups of 32)
MX_SF_BLOCK = 512


def e4m3_values() -> np.ndarray:
    """float32 value of every E4M3 (fn variant) code 0..255; 0x7F and 0xFF are NaN."""
    c = np.arange(256)
    s = np.where(c >> 7, -1.0, 1.0)
    e = (c >> 3) & 15
    m = (c & 7).astype(np.float64)
    mag = np.where(e == 0, m * 2.0**-9, (1.0 + m / 8.0) * np.exp2(e - 7.0))
    v = (s * mag).astype(np.float32)
    v[(c & 0x7F) == 0x7F] = np.nan
    return v


def encode_e4m3(x) -> np.ndarray:
    """fp32 -> E4M3 codes: round to nearest, ties to the even code, magnitudes above 448
    saturate to 448 (the cvt.rn.satfinite rule); the sign of x is kept (also for zero)."""
    x = np.asarray(x, dtype=np.float32)
    mags = e4m3_values()[:127].astype(np.float64)  # codes 0..126, ascending
    a = np.minimum(np.abs(x).astype(np.float64), E4M3_MAX)
    hi = np.clip(np.searchsorted(mags, a, side="left"), 0, 126)
    lo = np.clip(hi - 1, 0, 126)
    dlo, dhi = a - mags[lo], mags[hi] - a
    pick_hi = (dhi < dlo) | ((dhi == dlo) & (hi % 2 == 0))
    code = np.where(pick_hi, hi, lo).astype(np.uint8)
    code = np.where(a == mags[hi], hi, code).astype(np.uint8)
    return code | (np.signbit(x).astype(np.uint8) << 7)


def _group_exponent(amax: np.ndarray, below_top: int) -> np.ndarray:
    """floor(log2(amax)) - below_top clipped to [-127, 127]; -127 for an all-zero group."""
    _, E = np.frexp(amax)  # amax = f * 2**E, f in [0.5, 1)
    return np.where(amax > 0, np.clip(E.astype(np.int64) - 1 - below_top, -127, 127), -127)


def _quantize_groups(g: np.ndarray, below_top: int):
    """[..., 32] fp32 groups -> (E4M3 codes, exponents): codes = encode_e4m3(x * 2**-e)."""
    e = _group_exponent(np.abs(g).max(axis=-1), below_top)
    scaled = (g.astype(np.float64) * np.exp2(-e.astype(np.float64))[..., None]).astype(np.float32)
    return encode_e4m3(scaled), e


MX_Q8, MX_SPLIT2 = 0, 1


def quantize_act_mx8(A, mode: int = MX_Q8):
    """MXFP8 quantisation of activations A [M, K] along K (K % 32 == 0).

    mode MX_Q8 (OCP MX): scale exponent e = floor(log2(amax)) - 8, clipped to [-127, 127], an
    all-zero group gets e = -127 (byte 0); codes = encode_e4m3(x * 2**-e) (exact scaling, then
    RNE + saturation at 448).  Returns [(codes uint8 [M, K], scales uint8 [M, K/32])].

    mode MX_SPLIT2: two pieces, A ~ hi + lo.  hi uses e = floor(log2(amax)) - 7 (the group max
    lands in [128, 256), no saturation); lo quantises the exact residual A - dequant(hi) by the
    same rule.  Returns [(hi codes, hi scales), (lo codes, lo scales)].
    """
    A = np.asarray(A, dtype=np.float32)
    M, K = A.shape
    if K % GROUP:
        raise ValueError("K must be a multiple of 32")
    g = A.reshape(M, K // GROUP, GROUP)
    if mode == MX_Q8:
        c, e = _quantize_groups(g, E4M3_EMAX)
        return [(c.reshape(M, K), (e + 127).astype(np.uint8))]
    ch, eh = _quantize_groups(g, E4M3_EMAX - 1)
    vh = e4m3_values()[ch].astype(np.float64) * np.exp2(eh.astype(np.float64))[..., None]
    r = (g.astype(np.float64) - vh).astype(np.float32)  # exact: few significant bits on both sides
    cl, el = _quantize_groups(r, E4M3_EMAX - 1)
    return [(ch.reshape(M, K), (eh + 127).astype(np.uint8)), (cl.reshape(M, K), (el + 127).astype(np.uint8))]


def dequantize_act_mx8(codes, scales) -> np.ndarray:
    codes = np.asarray(codes, dtype=np.uint8)
    M, K = codes.shape
    v = e4m3_values()[codes].reshape(M, K // GROUP, GROUP).astype(np.float64)
    s = np.exp2(np.asarray(scales, dtype=np.float64) - 127.0)
    return (v * s[..., None]).reshape(M, K).astype(np.float32)


def dequantize_act_pieces(pieces) -> np.ndarray:
    """Sum of the dequantised pieces (fp64 sum, rounded to fp32)."""
    tot = sum(dequantize_act_mx8(c, s).astype(np.float64) for c, s in pieces)
    return np.asarray(tot, dtype=np.float32)


def ref_gemm_mx(A, B_packed, B_scales, mode: int = MX_Q8) -> np.ndarray:
    """The block-scaled path's reference: (sum of the dequantised activation pieces) @
    dequant(W) in fp32 (W in the reference layout [K/2, N] + [K/32, N])."""
    return dequantize_act_pieces(quantize_act_mx8(A, mode)) @ dequantize_mxfp4(B_packed, B_scales, axis=0)


def mx_sf_in_block(r, j):
    """Byte of (row r of a 128-row block, 32-k group j of a 128-k step) in a 512-byte scale
    block: 16*(r%32) + 4*(r//32) + j (the tcgen05.cp 32x128b.warpx4 source order)."""
    r = np.asarray(r)
    return 16 * (r & 31) + 4 * ((r >> 5) & 3) + j


def mx_scale_blocks(scales, rows_pad: int, k_pad: int, fill: int, k_major_blocks: bool) -> np.ndarray:
    """Scale bytes [rows, K/32] -> 512-byte blocks.  k_major_blocks=False: [rows_pad/128][k_pad/128]
    (weights); True: [k_pad/128][rows_pad/128] (activations).  Padding bytes = fill."""
    scales = np.asarray(scales, dtype=np.uint8)
    rows, kg = scales.shape
    full = np.full((rows_pad, k_pad // GROUP), fill, dtype=np.uint8)
    full[:rows, :kg] = scales
    rb, kb = rows_pad // 128, k_pad // MX_BK
    r, j = np.meshgrid(np.arange(128), np.arange(4), indexing="ij")
    off = mx_sf_in_block(r, j).reshape(-1)
    src = full.reshape(rb, 128, kb, 4).transpose(0, 2, 1, 3).reshape(rb, kb, 512)  # [rb, kb, r*4+j]
    out = np.empty((rb, kb, 512), dtype=np.uint8)
    out[:, :, off] = src
    return out.transpose(1, 0, 2).copy() if k_major_blocks else out


def mx_weight_layout(B_packed, B_scales) -> np.ndarray:
    """Host restatement of mxfp4_prepack_mx for reference-layout weights: nibbles [Np][Kp/2]
    (row n = weight column n, K contiguous, zero padded) then the scale blocks
    [Np/128][Kp/128] (padding scale 127); flat uint8."""
    B_packed = np.asarray(B_packed, dtype=np.uint8)
    K2, N = B_packed.shape
    K = 2 * K2
    Np, Kp = -(-N // 128) * 128, -(-K // MX_BK) * MX_BK
    data = np.zeros((Np, Kp // 2), dtype=np.uint8)
    data[:N, :K2] = B_packed.T
    sf = mx_scale_blocks(np.asarray(B_scales, dtype=np.uint8).T, Np, Kp, 127, False)
    return np.concatenate([data.reshape(-1), sf.reshape(-1)])


MX_DECODE_M = 16  # M <= 16: the decode kernel's operand of 16 hi + 16 lo rows


def mx_act_rows(M: int, mode: int) -> tuple[int, int]:
    """(group rows G, code rows) of the quantised-activation operand for (M, mode).

    Code row b holds piece p of activation row m, b = (m // G) * 2G + p * G + m % G (pieces
    stacked per G-row group), or b = m with one piece (G = 0):
      M <= 16 (decode kernel), either mode: G = 16, 32 rows (the lo rows are zero for MX_Q8);
      M > 16, MX_Q8:     G = 0, rows = M rounded up to 256;
      M > 16, MX_SPLIT2: G = 128, rows = 2 * (M rounded up to 128).
    """
    if M <= MX_DECODE_M:
        return MX_DECODE_M, 2 * MX_DECODE_M
    if mode == MX_Q8:
        return 0, -(-M // 256) * 256
    return 128, 2 * (-(-M // 128) * 128)


def mx_act_layout(A, mode: int = MX_Q8) -> tuple[np.ndarray, np.ndarray]:
    """Host restatement of mxfp4_quantize_act_mx8(A, mode): codes [rows][Kp] (zero padded) and
    scale blocks [Kp/128][ceil(rows/128)][512] (padding byte 0)."""
    A = np.asarray(A, dtype=np.float32)
    M, K = A.shape
    Kp = -(-K // MX_BK) * MX_BK
    G, rows = mx_act_rows(M, mode)
    pieces = quantize_act_mx8(A, mode)
    codes = np.zeros((rows, Kp), dtype=np.uint8)
    sc = np.zeros((rows, K // GROUP), dtype=np.uint8)
    m = np.arange(M)
    for p, (c, s) in enumerate(pieces):
        b = m if G == 0 else (m // G) * 2 * G + p * G + m % G
        codes[b, :K] = c
        sc[b] = s
    rows_sf = -(-rows // 128) * 128
    return codes, mx_scale_blocks(sc, rows_sf, Kp, 0, True)
