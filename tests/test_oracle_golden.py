"""Pins the CPU oracle (oracle/hlkv_oracle.c) before anything is checked against it.

1. Known answers restated from the reference's own tests
   (tests/project2/test_dequant.cpp, test_quant_encode.cpp, test_dequant_cuda.cpp).
2. The fixtures in tests/golden/, produced by the reference library itself.
3. The live reference library (oracle/_ref) on larger random inputs, where present.
"""
import math
import os

import numpy as np

from helpers import block_wide_scale_refs
import pytest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden.npz")
FP16, E4M3, E5M2, INT4 = 0, 1, 2, 3


def f32(bits):
    return np.asarray(bits, dtype=np.uint32).view(np.float32)


def ldexp_decode(code: int, ebits: int, mbits: int, bias: int, ieee: bool) -> float:
    """Textbook value of a minifloat code in double precision (test_dequant.cpp:41-57)."""
    sign = (code >> (ebits + mbits)) & 1
    e = (code >> mbits) & ((1 << ebits) - 1)
    m = code & ((1 << mbits) - 1)
    emax = (1 << ebits) - 1
    if ieee and e == emax:
        v = math.inf if m == 0 else math.nan
    elif not ieee and e == emax and m == (1 << mbits) - 1:
        v = math.nan
    elif e == 0:
        v = math.ldexp(m, 1 - bias - mbits)
    else:
        v = math.ldexp((1 << mbits) + m, e - bias - mbits)
    return -v if sign else v


SPECS = {FP16: (5, 10, 15, True, 65536), E4M3: (4, 3, 7, False, 256), E5M2: (5, 2, 15, True, 256)}


@pytest.mark.parametrize("fmt", [FP16, E4M3, E5M2])
def test_exhaustive_decode_matches_textbook(oracle, fmt):
    eb, mb, bias, ieee, n = SPECS[fmt]
    got = oracle.decode(fmt, np.arange(n, dtype=np.uint16))
    for c in range(n):
        want = ldexp_decode(c, eb, mb, bias, ieee)
        if math.isnan(want):
            assert math.isnan(got[c]), hex(c)
        else:
            assert float(got[c]) == want and math.copysign(1, got[c]) == math.copysign(1, want), hex(c)


def test_decode_known_constants(oracle):
    d16 = lambda c: float(oracle.decode(FP16, np.array([c]))[0])  # noqa: E731
    d4 = lambda c: float(oracle.decode(E4M3, np.array([c]))[0])  # noqa: E731
    d5 = lambda c: float(oracle.decode(E5M2, np.array([c]))[0])  # noqa: E731
    assert d16(0x3C00) == 1.0 and d16(0x7BFF) == 65504.0 and d16(0x0001) == 2.0 ** -24
    assert d16(0x0400) == 2.0 ** -14 and d16(0xFC00) == -math.inf
    assert d4(0x7E) == 448.0 and d4(0xFE) == -448.0 and d4(0x38) == 1.0
    assert d4(0x08) == 2.0 ** -6 and d4(0x01) == 2.0 ** -9 and d4(0x78) == 256.0
    assert math.isnan(d4(0x7F)) and math.isnan(d4(0xFF))
    assert d5(0x7B) == 57344.0 and d5(0x3C) == 1.0 and d5(0x01) == 2.0 ** -16
    assert d5(0x7C) == math.inf and all(math.isnan(d5(c)) for c in (0x7D, 0x7E, 0x7F))


def test_int4_low_nibble_first_and_fp16_little_endian(oracle):
    st, out = oracle.dequantize(INT4, np.array([0x21, 0xF0, 0x0E], np.uint8), 5,
                                np.array([[1.0, 0.0]], np.float32), 6)
    assert st == 0 and list(out) == [1, 2, 0, 15, 14]
    st, out = oracle.dequantize(FP16, np.array([0x00, 0x3C, 0x00, 0xC0], np.uint8), 2,
                                np.zeros((0, 2), np.float32), 0)
    assert st == 0 and list(out) == [1.0, -2.0]


def test_int4_fused_affine_single_rounding(oracle):
    st, out = oracle.dequantize(INT4, np.array([0x53, 0xF7], np.uint8), 4,
                                np.array([[0.5, -1.0], [-0.25, 2.0]], np.float32), 2)
    assert st == 0 and list(out) == [0.5, 1.5, 0.25, -1.75]
    scale = np.float32(1.0 + 2.0 ** -23)
    st, out = oracle.dequantize(INT4, np.array([0x0F], np.uint8), 1,
                                np.array([[scale, -15.0]], np.float32), 2)
    assert st == 0 and float(out[0]) == 15.0 * 2.0 ** -23  # a two-step q*s+b would lose it


def test_fp8_multiply_keeps_negative_zero(oracle):
    st, out = oracle.dequantize(E4M3, np.array([0x38, 0xBC, 0x01, 0x80], np.uint8), 4,
                                np.array([[2.0, 0.0], [0.5, 0.0]], np.float32), 2)
    assert st == 0 and list(out[:3]) == [2.0, -3.0, 2.0 ** -10]
    assert out[3] == 0.0 and math.copysign(1, out[3]) < 0


@pytest.mark.parametrize("fmt,sign,max_code", [(FP16, 0x8000, 0x7BFF), (E4M3, 0x80, 0x7E),
                                               (E5M2, 0x80, 0x7B)])
def test_every_code_round_trips_and_midpoints_round_to_even(oracle, fmt, sign, max_code):
    codes = np.arange(2 * sign, dtype=np.uint16)
    vals = oracle.decode(fmt, codes)
    back = oracle.encode(fmt, vals)
    for c in range(2 * sign):
        v = vals[c]
        if np.isnan(v):
            assert np.isnan(oracle.decode(fmt, back[c:c + 1])[0]) and (back[c] & sign) == (c & sign)
        elif np.isinf(v):
            assert back[c] == (c if fmt == FP16 else (c & sign) | max_code)
        else:
            assert back[c] == c, hex(c)
    lo = np.arange(max_code, dtype=np.uint16)
    a, b = oracle.decode(fmt, lo).astype(np.float64), oracle.decode(fmt, lo + 1).astype(np.float64)
    mid = ((a + b) / 2).astype(np.float32)
    assert np.array_equal(mid.astype(np.float64), (a + b) / 2)
    even = np.where(lo % 2 == 0, lo, lo + 1)
    for s in (0, sign):
        m = -mid if s else mid
        assert np.array_equal(oracle.encode(fmt, m), s | even)
        assert np.array_equal(oracle.encode(fmt, np.nextafter(m, np.float32(0))), s | lo)
        away = np.nextafter(m, np.float32(-np.inf if s else np.inf))
        assert np.array_equal(oracle.encode(fmt, away), s | (lo + 1))


def test_encode_special_values(oracle):
    h = lambda x: int(oracle.encode(FP16, np.array([x], np.float32))[0])  # noqa: E731
    e4 = lambda x: int(oracle.encode(E4M3, np.array([x], np.float32))[0])  # noqa: E731
    e5 = lambda x: int(oracle.encode(E5M2, np.array([x], np.float32))[0])  # noqa: E731
    inf, nan = np.inf, np.nan
    assert h(65504.0) == 0x7BFF and h(np.nextafter(np.float32(65520.0), np.float32(0))) == 0x7BFF
    assert h(65520.0) == 0x7C00 and h(1e10) == 0x7C00 and h(-inf) == 0xFC00 and h(nan) == 0x7E00
    assert e4(448.0) == 0x7E and e4(464.0) == 0x7E and e4(465.0) == 0x7E and e4(3e38) == 0x7E
    assert e4(inf) == 0x7E and e4(-inf) == 0xFE and e4(nan) == 0x7F and e4(-nan) == 0xFF
    assert e5(57344.0) == 0x7B and e5(61440.0) == 0x7B and e5(inf) == 0x7B and e5(-1e30) == 0xFB
    assert e5(nan) == 0x7F
    assert h(0.0) == 0 and h(-0.0) == 0x8000 and h(1e-40) == 0 and h(-1e-40) == 0x8000
    assert e4(2.0 ** -10) == 0 and e4(1.5 * 2.0 ** -10) == 1 and e4(-(2.0 ** -30)) == 0x80
    assert e5(2.0 ** -17) == 0 and e5(2.0 ** -16) == 1


def test_fp16_encode_matches_numpy_float16(oracle):
    """Cross-check against an independent binary16 conversion (numpy, RNE), as the reference
    checks against _Float16 (test_quant_encode.cpp:135-147)."""
    xs = np.random.default_rng(12345).integers(0, 2 ** 32, size=2_000_000, dtype=np.uint64)
    xs = xs.astype(np.uint32)
    x = xs.view(np.float32)
    x = x[~np.isnan(x)]
    with np.errstate(over="ignore"):
        want = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(oracle.encode(FP16, x), want)


def test_quantize_known_answers(oracle):
    st, p, packed = oracle.quantize(INT4, np.array([0.0, 7.0, 15.0], np.float32), 4,
                                    packed_init=0xFF)
    assert st == 0 and p[0, 0] == 1.0 and p[0, 1] == 0.0
    assert list(packed) == [0x70, 0x0F]
    st, p, packed = oracle.quantize(E4M3, np.array([0.5, -3.0, 1.0, 0.0], np.float32), 2)
    assert st == 0 and p[0, 0] == np.float32(3.0) / np.float32(448.0)
    assert p[1, 0] == np.float32(1.0) / np.float32(448.0) and p[0, 1] == 0.0
    assert packed[1] == 0xFE and packed[2] == 0x7E
    st, p, _ = oracle.quantize(E5M2, np.zeros(4, np.float32), 4)
    assert st == 0 and p[0, 0] == 1.0


def test_quantize_rejects_bad_arguments_without_writing(oracle):
    inf = np.inf
    def untouched(fmt, x, g, n_params=None, packed_size=None):
        st, p, packed = oracle.quantize(fmt, np.array(x, np.float32), g, n_params, packed_size,
                                        params_init=9.0, packed_init=0xAB)
        assert np.all(p == 9.0) and np.all(packed == 0xAB)
        return st
    assert untouched(INT4, [1, inf, 0, 2], 4) == 1
    assert untouched(E4M3, [1, inf, 0, 2], 4) == 1
    assert untouched(INT4, [-3e38, 3e38, 0, 0], 4) == 1
    assert untouched(INT4, [1, 2, 3, 4], 2, n_params=1) == 1
    assert untouched(INT4, [1, 2, 3, 4], 4, packed_size=1) == 2
    assert untouched(7, [1, 2, 3, 4], 4, n_params=1) == 3
    assert untouched(4, [1, 2, 3, 4], 4, n_params=1) == 3
    st, _, fp16 = oracle.quantize(FP16, np.array([1.0, inf, 0.0, 2.0], np.float32), 0)
    assert st == 0 and (int(fp16[2]) | int(fp16[3]) << 8) == 0x7C00


def test_dequantize_rejects_bad_arguments(oracle):
    packed = np.zeros(64, np.uint8)
    one = np.array([[1.0, 0.0]], np.float32)
    assert oracle.dequantize(9, packed, 4, one, 4)[0] == 3
    assert oracle.dequantize(FP16, packed, 4, np.zeros((0, 2), np.float32), 4)[0] == 1
    assert oracle.dequantize(E4M3, packed, 4, one, 0)[0] == 1
    assert oracle.dequantize(INT4, packed, 4, one, 3)[0] == 1
    assert oracle.dequantize(4, packed, 4, one, 4)[0] == 3
    assert oracle.dequantize(INT4, packed, 8, one, 4)[0] == 1
    assert oracle.dequantize(INT4, packed, 4, np.array([[np.nan, 0.0]], np.float32), 4)[0] == 1
    assert oracle.dequantize(INT4, packed, 4, np.array([[1.0, np.inf]], np.float32), 4)[0] == 1
    assert oracle.dequantize(E5M2, packed, 4, np.array([[1.0, 0.5]], np.float32), 4)[0] == 1
    assert oracle.dequantize(INT4, packed[:1], 4, one, 4)[0] == 2
    assert oracle.dequantize(FP16, packed[:7], 4, np.zeros((0, 2), np.float32), 0)[0] == 2
    st, out = oracle.dequantize(INT4, packed, 4, one, 4, out_size=3)
    assert st == 2 and np.all(out == 7.0)


def test_accuracy_bounds_on_gaussian_data(oracle):
    """quantize -> dequantize stays inside the analytical bound (test_dequant.cpp:261-315)."""
    n = 1 << 14
    for fmt, g, rel, sub in ((E4M3, 128, -4, -10), (E5M2, 128, -3, -17)):
        x = oracle.gaussian(12 + g, n)
        st, p, packed = oracle.quantize(fmt, x, g)
        _, out = oracle.dequantize(fmt, packed, n, p, g)
        scale = np.repeat(p[:, 0], g)[:n].astype(np.float64)
        bound = np.maximum(np.ldexp(np.abs(x), rel), np.ldexp(scale, sub)) + 4 * np.ldexp(np.abs(x) + 1e-30, -23)
        assert np.all(np.abs(out.astype(np.float64) - x) <= bound)
    x = oracle.gaussian(13 + 128, n)
    st, p, packed = oracle.quantize(INT4, x, 128)
    _, out = oracle.dequantize(INT4, packed, n, p, 128)
    scale = np.repeat(p[:, 0], 128)[:n].astype(np.float64)
    assert np.all(np.abs(out - x) <= 0.5 * scale * (1 + 1e-5) + 4 * np.ldexp(np.abs(x) + 1e-30, -23))


# ---- against the reference's own outputs -------------------------------------------------
@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def test_decode_tables_match_golden(oracle, golden):
    for fmt, n in ((0, 65536), (1, 256), (2, 256)):
        got = oracle.decode(fmt, np.arange(n, dtype=np.uint16)).view(np.uint32)
        assert np.array_equal(got, golden[f"decode_{fmt}"]), fmt


def test_encode_matches_golden(oracle, golden):
    x = golden["encode_in"].view(np.float32)
    for fmt in (0, 1, 2):
        assert np.array_equal(oracle.encode(fmt, x), golden[f"encode_{fmt}"]), fmt


def test_fp8_codes_times_kernel_scales_match_golden(oracle, golden):
    codes = np.arange(256, dtype=np.uint8)
    for fmt in (1, 2):
        for k, s in enumerate(golden["k_scales"]):
            st, out = oracle.dequantize_to_fp16(fmt, codes, 256, np.array([[s, 0.0]], np.float32), 256)
            assert st == 0 and np.array_equal(out, golden[f"fp8_scales_{fmt}"][k]), (fmt, s)


def test_quantize_matches_golden(oracle, golden):
    for key in [k for k in golden.files if k.startswith("q_in_")]:
        _, _, fmt, gs = key.split("_")
        fmt, gs = int(fmt), int(gs)
        st, p, packed = oracle.quantize(fmt, golden[key], gs)
        assert st == 0
        assert np.array_equal(p.view(np.uint32), golden[f"q_params_{fmt}_{gs}"].view(np.uint32)), key
        assert np.array_equal(packed, golden[f"q_packed_{fmt}_{gs}"]), key
        _, deq = oracle.dequantize_to_fp16(fmt, packed, golden[key].size, p, gs)
        assert np.array_equal(deq, golden[f"q_fp16_{fmt}_{gs}"]), key


def test_oracle_matches_live_reference(oracle, ref):
    rng = np.random.default_rng(3)
    x = rng.integers(0, 2 ** 32, size=1 << 20, dtype=np.uint64).astype(np.uint32).view(np.float32)
    for fmt in (0, 1, 2):
        assert np.array_equal(oracle.encode(fmt, x), ref.encode(fmt, x))
    for fmt in (0, 1, 2, 3):
        for g in ((0,) if fmt == 0 else (2, 16, 128, 1000)):
            v = oracle.gaussian(7 + g, 4099) * 3
            v[5], v[6] = 0.0, -0.0
            a, b = oracle.quantize(fmt, v, g), ref.quantize(fmt, v, g)
            assert a[0] == b[0] == 0
            assert np.array_equal(a[1].view(np.uint32), b[1].view(np.uint32))
            assert np.array_equal(a[2], b[2])
            assert np.array_equal(oracle.dequantize_to_fp16(fmt, a[2], v.size, a[1], g)[1],
                                  ref.dequantize_to_fp16(fmt, b[2], v.size, b[1], g)[1])


def test_gather_oracle_matches_reference_gather(oracle, ref):
    """The block walk itself: oracle gather == the reference-built gather on random tables."""
    rng = np.random.default_rng(21)
    T, H, D = 4, 2, 64
    rows, elems = 2 * T * H, 2 * T * H * D
    pools = {}
    for f in (0, 1, 2, 3):
        ns = 6
        sb = oracle.slot_bytes_needed(f, T, H, D)
        sb = (sb + 15) // 16 * 16
        buf = np.zeros((ns, sb), np.uint8)
        for s in range(ns):
            x = (rng.standard_normal(elems) * 2).astype(np.float16).astype(np.float32)
            st, p, codes = oracle.quantize(f, x, 0 if f == 0 else D)
            buf[s, :codes.size] = codes
            if f == 3:
                buf[s, codes.size:codes.size + 8 * rows] = p.view(np.uint8).reshape(-1)
            elif f in (1, 2):
                buf[s, codes.size:codes.size + 4 * rows] = p[:, 0].copy().view(np.uint8)
        pools[f] = (buf.reshape(-1), sb, ns)
    n_blocks = 20
    table = np.zeros((n_blocks, 4), np.uint32)
    for i in range(n_blocks):
        f = int(rng.integers(0, 4))
        info = f | (1 << 6) | (int(rng.integers(0, T + 1)) << 10)
        table[i] = (int(rng.integers(0, 6)), info, 0, i)
    table[3] = (0xFFFFFFFF, 15, 0, 3)  # non-executable
    arena = rng.permutation(n_blocks).astype(np.uint32)
    segs = np.array([[0, 5], [5, 0], [5, 9], [14, 8]], np.uint32)  # the last one runs off the arena
    total = int(segs[:, 1].sum())
    a = np.full(total * elems, 0x1111, np.uint16)
    b = np.full(total * elems, 0x1111, np.uint16)
    ea = oracle.gather_dequant(pools, T, H, D, 1, table, arena, segs, a)
    eb = ref.gather_dequant(pools, T, H, D, 1, table, arena, segs, b, threads=3)
    assert ea == eb and ea & 8 and ea & 1
    assert np.array_equal(a, b)


def test_gather_with_block_wide_scales_matches_reference(oracle, ref):
    """Descriptors with scale modes kInlineF32 / kInlineF16Pair (block_descriptor.hpp:61-72):
    the block's rows decode with the descriptor's parameters instead of the per-row ones, as
    one group of the reference's dequantize_reference_to_fp16 (the reference-built gather uses
    the reference's own inline_scale_f32 and decode_fp16); kExternal is rejected (bit 7)."""
    rng = np.random.default_rng(33)
    T, H, D = 4, 2, 64
    rows, elems = 2 * T * H, 2 * T * H * D
    pools = {}
    for f in (0, 1, 2, 3):
        ns = 6
        sb = (oracle.slot_bytes_needed(f, T, H, D) + 15) // 16 * 16
        buf = rng.integers(0, 256, size=(ns, sb), dtype=np.uint8)  # any codes decode
        if f == 3:  # finite per-row parameters for the per-row blocks
            code = oracle.slot_bytes_needed(3, T, H, D) - 8 * rows
            prm = (rng.standard_normal((ns, 2 * rows)) * 2).astype(np.float32)
            buf[:, code:code + 8 * rows] = prm.view(np.uint8)
        elif f in (1, 2):
            code = oracle.slot_bytes_needed(f, T, H, D) - 4 * rows
            prm = np.abs(rng.standard_normal((ns, rows))).astype(np.float32)
            buf[:, code:code + 4 * rows] = prm.view(np.uint8)
        pools[f] = (buf.reshape(-1), sb, ns)
    n_blocks = 40
    table = np.zeros((n_blocks, 4), np.uint32)
    refs = block_wide_scale_refs(rng, n_blocks)
    for i in range(n_blocks):
        f = int(rng.integers(0, 4))
        mode, sref = refs[i] if i % 4 else (0, 0)
        info = f | mode << 4 | (1 << 6) | (int(rng.integers(0, T + 1)) << 10)
        table[i] = (int(rng.integers(0, 6)), info, sref, i)
    table[7] = (1, 1 | 3 << 4 | 1 << 6 | T << 10, 5, 7)  # kExternal: rejected
    arena = rng.permutation(n_blocks).astype(np.uint32)
    segs = np.array([[0, 13], [13, 0], [13, 27]], np.uint32)
    total = int(segs[:, 1].sum())
    a = np.full(total * elems, 0x1111, np.uint16)
    b = np.full(total * elems, 0x1111, np.uint16)
    ea = oracle.gather_dequant(pools, T, H, D, 1, table, arena, segs, a)
    eb = ref.gather_dequant(pools, T, H, D, 1, table, arena, segs, b, threads=3)
    assert ea == eb == 1 << 7
    assert np.array_equal(a, b)
    # both the rejected blocks (untouched) and decoded block-wide blocks are present
    per_block = a.reshape(total, elems)
    assert (per_block == 0x1111).all(axis=1).sum() >= 2
    assert (per_block != 0x1111).all(axis=1).sum() >= 20


def test_quantize_rows_oracle_equals_reference(oracle, ref):
    """The threaded per-row encoders (the decode-append CPU baseline) of the oracle and of
    the reference library agree bit for bit, and each row equals a single quantize call."""
    rng = np.random.default_rng(21)
    x = (rng.standard_normal((777, 128)) * rng.choice([1e-3, 1.0, 50.0], size=(777, 1))).astype(np.float32)
    x[3] = 0.0
    x[4, ::2] = -0.0
    fm = rng.choice([1, 2, 3], size=777).astype(np.uint8)
    res = []
    for impl in (oracle, ref):
        p = np.zeros((777, 2), np.float32)
        c = np.zeros((777, 128), np.uint8)
        assert impl.quantize_rows(fm, x, p, c, threads=5) == 0
        res.append((p.view(np.uint32).copy(), c.copy()))
    assert np.array_equal(res[0][0], res[1][0]) and np.array_equal(res[0][1], res[1][1])
    for r in (0, 3, 4, 500):
        st, p1, c1 = oracle.quantize(int(fm[r]), x[r], 128)
        assert st == 0 and np.array_equal(c1, res[0][1][r][:c1.size])


def _ref_transcode(ref, pools, T, H, D, jobs):
    """The transcode spelled out with the reference library's own calls: per row,
    dequantize_reference_to_fp16 of the source row, then quantize_reference of its
    binary32 values into the destination row (rows of later tokens from zeros)."""
    rows = 2 * T * H
    packed = lambda f, n: 2 * n if f == 0 else (n // 2 if f == 3 else n)
    for ff, fs, tf, ts, vt, fmode, fref in jobs[:, :7]:
        # block-wide source parameters (scale modes 1 and 2), as the reference's decoder
        # would be given them; a job whose parameters it rejects (or mode 3) moves nothing
        wide = None
        if ff != 0 and fmode != 0:
            if fmode > 2:
                continue
            if fmode == 1:
                wide = np.array([[np.uint32(fref).view(np.float32), 0]], np.float32)
            else:
                halves = np.array([fref & 0xFFFF, fref >> 16], np.uint16).view(np.float16).astype(np.float32)
                wide = halves.reshape(1, 2)
            probe = np.zeros(packed(int(ff), D), np.uint8)
            if ref.dequantize_to_fp16(int(ff), probe, D, wide, D)[0] != 0:
                continue
        src_buf, sb_s, _ = pools[int(ff)]
        dst_buf, sb_d, _ = pools[int(tf)]
        src = src_buf[int(fs) * sb_s:(int(fs) + 1) * sb_s]
        dst = dst_buf[int(ts) * sb_d:(int(ts) + 1) * sb_d]
        sc, dc = packed(int(ff), rows * D), packed(int(tf), rows * D)
        for r in range(rows):
            if (r // H) % T < vt:
                codes = src[packed(int(ff), r * D):packed(int(ff), (r + 1) * D)]
                if ff == 0:
                    p = np.zeros((0, 2), np.float32)
                elif wide is not None:
                    p = wide
                elif ff == 3:
                    p = src[sc + 8 * r:sc + 8 * r + 8].view(np.float32).reshape(1, 2)
                else:
                    p = np.array([[src[sc + 4 * r:sc + 4 * r + 4].view(np.float32)[0], 0]], np.float32)
                st, h16 = ref.dequantize_to_fp16(int(ff), codes, D, p, 0 if ff == 0 else D)
                assert st == 0
                x = h16.view(np.float16).astype(np.float32)
            else:
                x = np.zeros(D, np.float32)
            st, p2, c2 = ref.quantize(int(tf), x, 0 if tf == 0 else D)
            if st != 0:
                continue
            dst[packed(int(tf), r * D):packed(int(tf), (r + 1) * D)] = c2
            if tf == 3:
                dst[dc + 8 * r:dc + 8 * r + 8] = p2.reshape(-1).view(np.uint8)
            elif tf != 0:
                dst[dc + 4 * r:dc + 4 * r + 4] = p2[0, :1].view(np.uint8)


def test_transcode_oracle_matches_reference_calls(oracle, ref):
    rng = np.random.default_rng(31)
    T, H, D, n_slots = 4, 2, 64, 6
    rows = 2 * T * H
    pools = {}
    for f in (0, 1, 2, 3):
        sb = oracle.slot_bytes_needed(f, T, H, D)
        sb = (sb + 15) // 16 * 16
        buf = np.zeros(n_slots * sb, np.uint8)
        for s in range(n_slots):   # valid encoded content
            x = (rng.standard_normal((rows, D)) * rng.choice([1e-3, 1, 300])).astype(np.float16).astype(np.float32)
            for r in range(rows):
                st, p, c = oracle.quantize(f, x[r], 0 if f == 0 else D)
                cb = {0: 2 * D, 1: D, 2: D, 3: D // 2}[f]
                buf[s * sb + r * cb:s * sb + (r + 1) * cb] = c
                code_total = {0: 2, 1: 1, 2: 1, 3: 0.5}[f] * rows * D
                o = s * sb + int(code_total)
                if f == 3:
                    buf[o + 8 * r:o + 8 * r + 8] = p.reshape(-1).view(np.uint8)
                elif f != 0:
                    buf[o + 4 * r:o + 4 * r + 4] = p[0, :1].view(np.uint8)
        pools[f] = (buf, sb, n_slots)
    # an FP16 row with Inf: rejected when encoding to FP8/INT4, copied when to FP16
    pools[0][0][2 * D * 3 + 5 * 2:2 * D * 3 + 6 * 2] = np.array([0x7C00], np.uint16).view(np.uint8)
    jobs = []
    slot = {f: 0 for f in range(4)}
    for ff in range(4):
        for tf in range(4):
            if ff == tf:
                continue
            jobs.append([ff, slot[ff] % 3, tf, 3 + slot[tf] % 3, int(rng.integers(0, T + 1)), 0, 0, 0])
            slot[ff] += 1
            slot[tf] += 1
    jobs[0][4] = T  # FP16 slot 0 with the Inf row, all rows valid
    jobs = np.array(jobs, np.uint32)
    a = {f: (b.copy(), sb, ns) for f, (b, sb, ns) in pools.items()}
    b = {f: (b.copy(), sb, ns) for f, (b, sb, ns) in pools.items()}
    err = oracle.transcode(a, T, H, D, jobs)
    _ref_transcode(ref, b, T, H, D, jobs)
    assert err == (1 << 9)
    for f in range(4):
        assert np.array_equal(a[f][0], b[f][0]), f


def test_transcode_block_wide_sources_match_reference_calls(oracle, ref):
    """Sources with block-wide parameters (the job's from_scale_mode / from_scale_ref): the
    oracle equals the reference's own calls given those parameters; jobs whose parameters
    the reference's decoder rejects (non-finite, FP8 bias) or with mode 3 move nothing and
    report HLKV_ERR_SCALE_MODE."""
    rng = np.random.default_rng(37)
    T, H, D, n_slots = 4, 2, 64, 8
    pools = {}
    for f in (0, 1, 2, 3):
        sb = (oracle.slot_bytes_needed(f, T, H, D) + 15) // 16 * 16
        pools[f] = (rng.integers(0, 256, size=n_slots * sb, dtype=np.uint8), sb, n_slots)
    f16 = lambda v: int(np.array([v], np.float16).view(np.uint16)[0])
    f32 = lambda v: int(np.array([v], np.float32).view(np.uint32)[0])
    jobs = np.array([
        [1, 0, 3, 0, T, 1, f32(0.25), 0],                    # E4M3, binary32 scale
        [2, 1, 1, 1, 3, 2, f16(0.5), 0],                     # E5M2, binary16 pair, bias 0
        [3, 2, 1, 2, T, 2, f16(0.125) | f16(-1.5) << 16, 0],  # INT4, scale and bias
        [3, 3, 2, 3, 2, 1, f32(0.01), 0],                    # INT4, binary32 scale, bias 0
        [1, 4, 3, 4, T, 2, f16(1.0) | f16(2.0) << 16, 0],    # FP8 with a bias: rejected
        [3, 5, 1, 5, T, 1, f32(np.inf), 0],                  # non-finite scale: rejected
        [1, 6, 3, 6, T, 3, 9, 0],                            # mode 3: rejected
        [1, 7, 3, 7, T, 0, 0, 0],                            # per-row parameters
    ], np.uint32)
    # per-row parameters of the last source: a finite scale per row
    sb1 = pools[1][1]
    code1 = oracle.slot_bytes_needed(1, T, H, D) - 4 * 2 * T * H
    pools[1][0][7 * sb1 + code1:7 * sb1 + code1 + 4 * 2 * T * H] = \
        np.full(2 * T * H, 0.02, np.float32).view(np.uint8)
    a = {f: (b.copy(), sb, ns) for f, (b, sb, ns) in pools.items()}
    b = {f: (b.copy(), sb, ns) for f, (b, sb, ns) in pools.items()}
    err = oracle.transcode(a, T, H, D, jobs)
    _ref_transcode(ref, b, T, H, D, jobs)
    assert err & (1 << 7)
    for f in range(4):
        assert np.array_equal(a[f][0], b[f][0]), f
    for k in (4, 5, 6):  # the rejected jobs' destination slots are untouched
        tf, ts = int(jobs[k, 2]), int(jobs[k, 3])
        sb = pools[tf][1]
        assert np.array_equal(a[tf][0][ts * sb:(ts + 1) * sb], pools[tf][0][ts * sb:(ts + 1) * sb]), k
