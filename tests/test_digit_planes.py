"""CPU model of the integer digit-plane arithmetic of the decode kernels
(`momij_b200/csrc/token.cu`: tok_encode and the MMA epilogue), checked
against float64: the identities the kernel relies on, at the bit level.

* group exponent E of the largest |x|, X = rint(x * 2^(21-E)) by the
  magic-number rounding fma(x, 2^(21-E), 1.5 * 2^23), exact for bf16 and
  fp16 inputs whose bits lie in the 22-bit window;
* class p enters as Y = X * 4^(3-p); the bytes of
  (bits * 4^(3-p) + (0x808080 - 0x4B400000 * 4^(3-p))) ^ 0x808080 (mod 2^32)
  are the balanced base-256 digits d3, d2, d1 (in [-128, 127]) and d0 of Y;
* the u8 operand of class p is w & (0x03030303 << 2p) = q * 4^p, so the
  digit sums D_d of a group satisfy sum_d 256^(3-d) D_d = 64 * sum q X, with
  |D_d| < 2^20 (16 code bytes of a group per column half, four classes), so
  the folded pairs 256 D0 + D1 and 256 D2 + D3 fit in 32 bits;
* the group's value s * (2^16 (256 D0 + D1) + (256 D2 + D3)) * 2^(E-27) +
  b * sum x equals sum (s q + b) x to fp32 rounding.
"""
from __future__ import annotations

import numpy as np
import pytest

from momij_b200 import synth as S

MAGIC = np.uint32(0x4B400000)  # bits of 1.5 * 2^23


def group_exponent(x32: np.ndarray) -> np.ndarray:
    """Unbiased exponent of each row's largest |x| (0 for an all-zero row),
    clamped below at -100, as the kernel derives it from the float's bits."""
    mx = np.abs(x32).max(axis=1)
    _, e = np.frexp(mx.astype(np.float64))  # mx = f * 2^e, f in [0.5, 1)
    E = np.where(mx > 0, e - 1, 0)
    return np.maximum(E, -100)


def encode(x32: np.ndarray):
    """Rows of 64 float32 values (exact halves) -> E, X, and per class p the
    kernel's digit words e[p] (uint32, bytes d3 d2 d1 d0)."""
    E = group_exponent(x32)
    scale = np.ldexp(np.float32(1), (21 - E)).astype(np.float32)[:, None]
    bits = (x32 * scale + np.float32(12582912.0)).astype(np.float32).view(np.uint32)
    X = bits.astype(np.int64) - int(MAGIC)
    words = []
    for p in range(4):
        mul = np.uint32(1 << (2 * (3 - p)))
        add = np.uint32((0x808080 - int(MAGIC) * int(mul)) & 0xFFFFFFFF)
        with np.errstate(over="ignore"):
            e = (bits * mul + add) ^ np.uint32(0x808080)
        words.append(e)
    return E, X, words


def digits_of(e: np.ndarray) -> np.ndarray:
    """Signed bytes of the digit words: [..., 4] as (d0, d1, d2, d3)."""
    b = e.view(np.uint8).reshape(e.shape + (4,)).astype(np.int8).astype(np.int64)
    return b[..., ::-1]  # byte 3 is d0


def halves(n: int, seed: int, dtype: int, scale_pow: np.ndarray | None = None) -> np.ndarray:
    h = S.normal_half(n, seed, 3, dtype)
    x = S.half_bits_to_f32(h, dtype).reshape(-1, 64)
    if scale_pow is not None:
        x = (x * np.ldexp(1.0, scale_pow)[:, None]).astype(np.float32)
        x = S.half_bits_to_f32(S.f32_to_half_bits(x, dtype), dtype)
    return x


@pytest.mark.parametrize("dtype", [S.DT_BF16, S.DT_F16])
def test_rounding_window_and_balanced_digits(dtype):
    rng = np.random.default_rng(1)
    pw = rng.integers(-20, 12, size=4096) if dtype == S.DT_BF16 else rng.integers(-8, 4, size=4096)
    x = halves(4096 * 64, 2, dtype, pw)
    E, X, words = encode(x)
    xs = x.astype(np.float64) * np.ldexp(1.0, 21 - E)[:, None]
    assert (np.abs(X) < 2 ** 22).all()
    assert (X == np.rint(xs)).all()  # round to nearest even, as the fma does
    for p in range(4):
        d = digits_of(words[p])
        Y = X * 4 ** (3 - p)
        assert ((d[..., 1:] >= -128) & (d[..., 1:] <= 127)).all()
        assert (d[..., 0] * 2 ** 24 + d[..., 1] * 2 ** 16 + d[..., 2] * 2 ** 8 + d[..., 3] == Y).all()


def test_elements_far_below_the_group_maximum_round_into_the_window():
    x = np.zeros((2, 64), np.float32)
    x[:, 0] = 1.0
    x[0, 1:] = np.float32(2.0 ** -30)  # below the 22-bit window: rounds to 0
    x[1, 1:] = np.float32(2.0 ** -12)  # inside it: exact
    E, X, _ = encode(x)
    assert (E == 0).all()
    assert (X[0, 1:] == 0).all() and (X[1, 1:] == 2 ** 9).all()
    assert (X[:, 0] == 2 ** 21).all()


def test_zero_group_and_exponent_clamp():
    x = np.zeros((3, 64), np.float32)
    x[1, 5] = np.float32(2.0 ** -110)  # below the clamp: E = -100, scaled by 2^121
    x[2, 7] = np.float32(-3.0e38)
    E, X, words = encode(x)
    assert E.tolist() == [0, -100, 127]
    assert (X[0] == 0).all() and (digits_of(words[0])[0] == 0).all()
    assert X[1, 5] == 2 ** 11 and X[2, 7] == np.rint(float(np.float32(-3.0e38)) * 2.0 ** (21 - 127))


def test_digit_sums_fold_and_reconstruct_the_group_dot_product():
    """One group of one row: the MMA's digit sums over the group's 16 code
    bytes and four classes, then the epilogue's folded pairs."""
    rng = np.random.default_rng(5)
    G = 2000
    x = halves(G * 64, 9, S.DT_BF16)
    E, X, words = encode(x)
    q = rng.integers(0, 4, size=(G, 64))
    q[:4] = 3  # the largest operand bytes
    # element 4b + p sits in code byte b, bits 2p..2p+1: operand byte q * 4^p
    D = np.zeros((G, 4), np.int64)
    for p in range(4):
        dig = digits_of(words[p])[:, p::4, :]          # [G, 16 bytes, 4 digits]
        opnd = (q[:, p::4] * 4 ** p)[:, :, None]        # u8 operand of class p
        assert (opnd <= 192).all()
        D += (opnd * dig).sum(axis=1)
    assert (np.abs(D) < 2 ** 20).all()
    dh = D[:, 0] * 256 + D[:, 1]
    dl = D[:, 2] * 256 + D[:, 3]
    assert (np.abs(dh) < 2 ** 31).all() and (np.abs(dl) < 2 ** 31).all()
    assert (dh * 65536 + dl == 64 * (q * X).sum(axis=1)).all()
    # the group's value in the kernel's fp32 steps against float64
    s = S.half_bits_to_f32(S.affine_uniform(G, S.SCALE_A, S.SCALE_C, 0, 1)).astype(np.float32)
    b = S.half_bits_to_f32(S.affine_uniform(G, S.BIAS_A, S.BIAS_C, 0, 2)).astype(np.float32)
    fx = np.ldexp(np.float32(1), E - 27).astype(np.float32)
    W = x.sum(axis=1, dtype=np.float32)
    f = (dh.astype(np.float32) * np.float32(65536) + dl.astype(np.float32)).astype(np.float32)
    got = (s * (f * fx) + b * W).astype(np.float64)
    want = ((s.astype(np.float64)[:, None] * q + b.astype(np.float64)[:, None]) * x).sum(axis=1)
    mag = (np.abs(s.astype(np.float64)[:, None] * q) + np.abs(b.astype(np.float64))[:, None]) @ np.ones(64)
    err = np.abs(got - want) / (mag * np.abs(x).max(axis=1))
    assert err.max() < 2e-6, err.max()
