"""Bit-level identities the attention kernels rely on, checked on the CPU.

The kernels themselves are tested on the GPU against the oracle; these tests
pin the arithmetic tricks they use, exhaustively over the codes:

* the UINT8 probability code from the ``+1.5*2^23`` add, permuted under an
  fp16 exponent, reads ``2 + c/512`` (attention.cuh, piper_softmax_role);
* one fused multiply-add with the power-of-two multiples ``512*w`` and
  ``-1024*w`` of the fp16 weight gives ``c*w`` rounded once to fp16, without
  overflow over the weights the kernel can produce (attention.cuh, kPScale);
* an INT8 V code read back from the ``+1.5*2^23`` rounding add converts to
  fp16 exactly, and the two permutes of the V transpose pick one feature of
  two keys from two rows' fp16 pairs (prepass.cuh, pack_codes_f16 and
  quantize_tile).
"""

from __future__ import annotations

import numpy as np


def byte_perm(x: int, y: int, selector: int) -> int:
    """CUDA ``__byte_perm``: result byte i is byte ``(selector >> 4i) & 7`` of (y:x)."""
    b = list(int(x).to_bytes(4, "little")) + list(int(y).to_bytes(4, "little"))
    return int.from_bytes(bytes(b[(selector >> (4 * i)) & 7] for i in range(4)), "little")


def f32_bits(v: float) -> int:
    return int(np.array([v], dtype=np.float32).view(np.uint32)[0])


def halves(word: int) -> np.ndarray:
    return np.array([word], dtype=np.uint32).view(np.float16)


K_BIAS = 12582912.0  # 1.5 * 2^23
K_PSCALE = 32.0      # attention.cuh: kPScale


def test_code_bits_read_as_fp16_two_plus_code_over_512() -> None:
    for c0 in range(256):
        for c1 in (0, 1, 127, 128, 254, 255, (c0 * 37) % 256):
            y0 = f32_bits(K_BIAS + c0)
            y1 = f32_bits(K_BIAS + c1)
            h = halves(byte_perm(y0, y1, 0x6420))
            assert h[0] == np.float16(2 + c0 / 512) and h[1] == np.float16(2 + c1 / 512)


def test_weighting_is_one_rounding_of_code_times_weight() -> None:
    # w_cur = 2^(max - m_ref) lies in (0, 2^8] (lazy rescale threshold 8).
    exps = np.linspace(-30.0, 8.0, 761)
    for e in exps:
        wh = np.float16(2.0 ** e * (K_PSCALE / 255.0))
        a = np.float16(wh * np.float16(512.0))
        b = -np.float16(wh * np.float16(1024.0))
        assert np.isfinite(a) and np.isfinite(b)
        # 512 * w and 1024 * w are exact (powers of two, no overflow).
        assert float(a) == float(wh) * 512.0 and -float(b) == float(wh) * 1024.0
        codes = np.arange(256, dtype=np.float64)
        h = 2.0 + codes / 512.0
        fused = (h * float(a) + float(b)).astype(np.float16)  # exact in float64, one rounding to fp16
        expected = (codes * float(wh)).astype(np.float16)
        assert np.array_equal(fused, expected), e
        assert np.isfinite(fused).all()


def test_int8_codes_convert_to_fp16_exactly() -> None:
    # round_codes leaves t = 1.5*2^23 + c (c the rounded, clamped code);
    # pack_codes_f16 subtracts 1.5*2^23 in fp32 and converts the pair to fp16.
    for c in range(-127, 128):
        t = np.float32(K_BIAS) + np.float32(c)
        assert f32_bits(float(t)) & 0xFF == c & 0xFF  # the byte pack_codes stores
        back = np.float32(t) - np.float32(K_BIAS)
        assert float(back) == c and float(np.float16(back)) == c


def test_v_transpose_permutes_pick_one_feature_of_two_keys() -> None:
    # The V tile holds, per key row, words of fp16 pairs (feature 2p in the low
    # half, 2p + 1 in the high half).  0x5410 takes the low halves of rows k
    # and k + 1, 0x7632 the high halves: feature 2p, then 2p + 1, of both keys.
    rng = np.random.default_rng(3)
    for _ in range(200):
        k0 = rng.integers(-127, 128, size=2).astype(np.float16)
        k1 = rng.integers(-127, 128, size=2).astype(np.float16)
        w0 = int(k0.view(np.uint32)[0])
        w1 = int(k1.view(np.uint32)[0])
        lo = halves(byte_perm(w0, w1, 0x5410))
        hi = halves(byte_perm(w0, w1, 0x7632))
        assert lo[0] == k0[0] and lo[1] == k1[0]
        assert hi[0] == k0[1] and hi[1] == k1[1]


def test_polynomial_exp2_emulated_in_fp32() -> None:
    # CPU restatement of exp2_poly2 (csrc/attention.cuh): each Horner step an
    # fp32 fused multiply-add (emulated through fp64 products); the stated
    # relative-error bound holds over [-125, 0], and below -125 the result is
    # tiny and non-negative.
    import numpy as np

    coeffs = [np.float32(c) for c in (0.001327644451521337, 0.00967553723603487, 0.05550713464617729,
                                      0.24022120237350464, 0.6931469440460205, 1.0000001192092896)]

    def fma(a, b, c):
        return (np.float64(a) * np.float64(b) + np.float64(c)).astype(np.float32)

    def poly(x):
        x = np.maximum(x, np.float32(-126.5)).astype(np.float32)
        t = (x + np.float32(12582912.0)).astype(np.float32)
        u = (t - np.float32(12582912.0)).astype(np.float32)
        f = fma(u, np.float32(-1.0), x)
        p = fma(coeffs[0], f, coeffs[1])
        for c in coeffs[2:]:
            p = fma(p, f, c)
        bits = (t.view(np.uint32).astype(np.uint64) * 0x800000 + p.view(np.uint32).astype(np.uint64)) & 0xFFFFFFFF
        return bits.astype(np.uint32).view(np.float32)

    x = np.linspace(-125.0, 0.0, 1_000_001).astype(np.float32)
    exact = np.exp2(x.astype(np.float64))
    rel = np.abs(poly(x).astype(np.float64) - exact) / exact
    assert rel.max() <= 2.5e-7
    tiny = poly(np.array([-np.inf, -300.0, -126.0], dtype=np.float32)).astype(np.float64)
    assert (tiny >= 0).all() and (tiny <= 2.0**-124).all()
