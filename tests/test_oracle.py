"""The CPU oracle against independent restatements and the reference's pins.

The oracle is the checker of every GPU parity test, so it is itself checked
here: codecs exhaustively against the OCP format definitions (written out again
below in plain Python), the generator against a pure-Python splitmix64, the 2:4
compressor against the reference's metadata constant 0x44444444
(tcgen05_sparse_mma/tcgen05_sparse_mma.cu:331) and round trips, and the FP32
GEMM against numpy in float64.
"""
import math

import numpy as np
import torch
import pytest

import oracle

M64 = (1 << 64) - 1


def py_hash(seed, ctr):
    z = (seed + (ctr + 1) * 0x9E3779B97F4A7C15) & M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
    return z ^ (z >> 31)


def py_uniform(seed, ctr):
    u = py_hash(seed, ctr) >> 40
    return float(np.float32((2 * u - (1 << 24)) * 2.0 ** -24))


def py_normal(seed, ctr):
    s = 0
    for i in range(6):
        h = py_hash(seed ^ 0x6A09E667F3BCC909, ctr * 6 + i)
        s += (h >> 40) + ((h >> 16) & 0xFFFFFF)
    return float(np.float32((s - 6 * (1 << 24)) * 2.0 ** -24))


def test_generator_matches_python_restatement():
    L = oracle.lib()
    for seed in (0, 11, 2 ** 63 + 5):
        for ctr in (0, 1, 77, 12345678901):
            assert L.orc_hash(seed, ctr) == py_hash(seed, ctr)
            assert L.orc_uniform(seed, ctr) == py_uniform(seed, ctr)
            assert L.orc_normal(seed, ctr) == py_normal(seed, ctr)


def test_generator_rows_and_shards():
    full = oracle.gen(8, 40, 5, 1)
    part = oracle.gen(3, 40, 5, 1, row0=4)
    assert np.array_equal(full[4:7], part)
    assert np.array_equal(oracle.gen_rows([6, 1], 40, 5, 1), full[[6, 1]])


def test_generator_moments():
    u = oracle.gen(256, 1024, 1, 0)
    assert u.min() >= -1.0 and u.max() < 1.0
    assert abs(u.mean()) < 5e-3 and abs(u.var() - 1 / 3) < 5e-3
    n = oracle.gen(256, 1024, 1, 1)
    assert abs(n.mean()) < 5e-3 and abs(n.var() - 1.0) < 1e-2
    assert np.abs(n).max() < 6.0


# ---------------------------------------------------------------- codecs
def ocp_e4m3(code):
    s, e, m = code >> 7, (code >> 3) & 15, code & 7
    if e == 15 and m == 7:
        return math.nan
    v = 2.0 ** (e - 7) * (1 + m / 8) if e else 2.0 ** -6 * (m / 8)
    return -v if s else v


def ocp_e2m1(code):
    s, e, m = code >> 3, (code >> 1) & 3, code & 1
    v = 2.0 ** (e - 1) * (1 + m / 2) if e else 0.5 * m
    return -v if s else v


def nearest_even(x, codes, value):
    """RNE onto a finite code set with saturation, by brute force."""
    finite = [c for c in codes if not math.isnan(value(c))]
    best = None
    for c in finite:
        d = abs(value(c) - x)
        if best is None or d < best[0] - 1e-300:
            best = (d, c)
        elif abs(d - best[0]) <= 1e-300:
            # tie: prefer the even mantissa (code LSB 0) of the same sign
            if (c & 1) == 0 and (best[1] & 1) == 1:
                best = (d, c)
    return best[1]


def test_e4m3_decode_exhaustive():
    L = oracle.lib()
    for c in range(256):
        want = ocp_e4m3(c)
        got = L.orc_e4m3_to_f32(c)
        assert (math.isnan(want) and math.isnan(got)) or got == want


def test_e4m3_encode_round_trip_and_rne():
    L = oracle.lib()
    for c in range(256):
        v = ocp_e4m3(c)
        if math.isnan(v) or (v == 0 and c == 0x80):
            continue
        assert L.orc_f32_to_e4m3(v) == c
    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.normal(0, 30, 3000), rng.normal(0, 0.01, 1000),
                         [448, 449, 463.9, 464, 465, 1e9, -1e9, 2 ** -10, 3 * 2 ** -11]])
    pos_codes = list(range(0, 127))
    for x in xs.astype(np.float32):
        x = float(x)
        mag = min(abs(x), 448.0)
        c = nearest_even(mag, pos_codes, ocp_e4m3)
        if ocp_e4m3(c) == 0.0:
            c = 0
        want = c | (0x80 if x < 0 and c != 0 else 0)
        got = L.orc_f32_to_e4m3(x)
        assert got == want or (ocp_e4m3(got) == 0 and ocp_e4m3(want) == 0), (x, got, want)


def test_e2m1_exhaustive():
    L = oracle.lib()
    for c in range(16):
        assert L.orc_e2m1_to_f32(c) == ocp_e2m1(c)
    grid = np.arange(-8, 8, 0.0625, dtype=np.float32)
    for x in grid:
        x = float(x)
        c = nearest_even(min(abs(x), 6.0), list(range(8)), ocp_e2m1)
        want = c | (8 if x < 0 and c != 0 else 0)
        got = L.orc_f32_to_e2m1(x)
        assert ocp_e2m1(got) == ocp_e2m1(want), (x, got, want)


def ocp_e5m2(c):
    """E5M2 from its definition: 1-5-2, bias 15, exponent 31 = inf / NaN."""
    s, e, m = c >> 7, (c >> 2) & 31, c & 3
    if e == 31:
        v = math.inf if m == 0 else math.nan
    else:
        v = (1 + m / 4) * 2.0 ** (e - 15) if e else (m / 4) * 2.0 ** -14
    return -v if s else v


def test_e5m2_decode_exhaustive_and_against_torch():
    L = oracle.lib()
    for c in range(256):
        want = ocp_e5m2(c)
        got = L.orc_e5m2_to_f32(c)
        assert (math.isnan(want) and math.isnan(got)) or got == want
    # torch's float8_e5m2 (a third-party codec) decodes the same table
    t = torch.arange(256, dtype=torch.uint8).view(torch.float8_e5m2).float().numpy()
    ours = np.array([L.orc_e5m2_to_f32(c) for c in range(256)], np.float32)
    assert np.array_equal(np.isnan(t), np.isnan(ours))
    assert np.array_equal(t[~np.isnan(t)], ours[~np.isnan(ours)])


def test_e5m2_encode_rne_saturating():
    L = oracle.lib()
    rng = np.random.default_rng(1)
    xs = np.concatenate([rng.normal(0, 300, 3000), rng.normal(0, 1e-4, 1000),
                         [57344, 57345, 61439, 61440, 1e9, -1e9, 1.125, 1.375, 2.0 ** -17]])
    xs = xs.astype(np.float32)
    # within the finite range, torch's round-to-nearest-even conversion agrees
    inr = xs[np.abs(xs) <= 57344]
    t = torch.from_numpy(inr).to(torch.float8_e5m2).view(torch.uint8).numpy()
    got = np.array([L.orc_f32_to_e5m2(float(x)) for x in inr], np.uint8)
    same = (got == t) | ((got & 0x7F) == 0) & ((t & 0x7F) == 0)
    assert same.all(), inr[~same][:5]
    # beyond it the conversion saturates to the largest finite value
    for x in (57345.0, 61440.0, 1e9):
        assert L.orc_f32_to_e5m2(x) == 0x7B and L.orc_f32_to_e5m2(-x) == 0xFB


def test_s8_and_tf32_rounding():
    L = oracle.lib()
    for x, want in ((2.5, 2), (3.5, 4), (-2.5, -2), (-0.5, 0), (126.6, 127), (300.0, 127),
                    (-128.4, -128), (-1e9, -128)):
        assert L.orc_f32_to_s8(x) == want, x
    one = 1.0
    for x, want in ((one + 2 ** -11, one), (one + 3 * 2 ** -11, one + 2 ** -9),
                    (one + 2 ** -12, one), (one + 2 ** -10, one + 2 ** -10), (-1.5, -1.5)):
        assert L.orc_f32_to_tf32(x) == want, x
    rng = np.random.default_rng(2)
    x = rng.normal(0, 1, 4096).astype(np.float32)
    q, d = oracle.quant_elem(x, "tf32")
    assert np.array_equal(q, d) and np.all((q.view(np.uint32) & 0x1FFF) == 0)
    assert np.max(np.abs(q - x) / np.abs(x)) <= 2.0 ** -11


def test_f16_codec_against_numpy():
    # IEEE binary16 restated from its definition agrees with numpy's conversion
    L = oracle.lib()
    rng = np.random.default_rng(5)
    x = np.concatenate([rng.normal(0, 100, 5000), rng.normal(0, 1e-5, 2000),
                        [65504, 65519, 65520, 1e6, 2 ** -24, 3 * 2 ** -25, 2 ** -26]]).astype(np.float32)
    ours = np.array([L.orc_f32_to_f16(float(v)) for v in x], np.uint16)
    with np.errstate(over="ignore"):
        want = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(ours, want)
    codes = np.arange(65536, dtype=np.uint16)
    dec = np.array([L.orc_f16_to_f32(int(c)) for c in codes], np.float32)
    ref = codes.view(np.float16).astype(np.float32)
    same = (dec == ref) | (np.isnan(dec) & np.isnan(ref))
    assert same.all()


def test_u8_rounding():
    L = oracle.lib()
    for x, want in ((2.5, 2), (3.5, 4), (-3.0, 0), (254.5, 254), (255.5, 255), (1e9, 255)):
        assert L.orc_f32_to_u8(x) == want, x


def test_s8_exact_gemm_definition():
    rng = np.random.default_rng(3)
    A = rng.integers(-128, 128, (37, 300)).astype(np.int8)
    B = rng.integers(-128, 128, (23, 300)).astype(np.int8)
    got = oracle.gemm_s8_exact(A, B, 1.0 / 256)
    acc = A.astype(np.int64) @ B.astype(np.int64).T
    # every sum here is below 2^24, so fp32(acc) / 256 is exact and only bf16 rounds
    want, _ = oracle.quant_bf16((acc / 256.0).astype(np.float32))
    assert np.array_equal(got, want)


def ocp_fp6(c, ebits):
    """OCP MX FP6 from its definition: E2M3 (bias 1) or E3M2 (bias 3), no inf / NaN."""
    mbits = 5 - ebits
    bias = 1 if ebits == 2 else 3
    s, e, m = (c >> 5) & 1, (c >> mbits) & ((1 << ebits) - 1), c & ((1 << mbits) - 1)
    v = (1 + m / 2 ** mbits) * 2.0 ** (e - bias) if e else (m / 2 ** mbits) * 2.0 ** (1 - bias)
    return -v if s else v


@pytest.mark.parametrize("name,ebits,maxv", [("e2m3", 2, 7.5), ("e3m2", 3, 28.0)])
def test_fp6_exhaustive_and_rne(name, ebits, maxv):
    L = oracle.lib()
    dec = getattr(L, f"orc_{name}_to_f32")
    enc = getattr(L, f"orc_f32_to_{name}")
    for c in range(64):
        assert dec(c) == ocp_fp6(c, ebits)
        if not (c == 0x20):  # -0 encodes as +0
            assert enc(ocp_fp6(c, ebits)) == c
    pos = list(range(32))
    for x in np.linspace(-2 * maxv, 2 * maxv, 2001, dtype=np.float32):
        x = float(x)
        c = nearest_even(min(abs(x), maxv), pos, lambda k: ocp_fp6(k, ebits))
        want = ocp_fp6(c, ebits) * (-1 if x < 0 else 1)
        assert dec(enc(x)) == want, (name, x)


@pytest.mark.parametrize("fmt,bits", [("e2m1", 4), ("e2m3", 6), ("e3m2", 6)])
def test_sub_byte_packing_order(fmt, bits):
    # element i of each 16-group at bits [bits*i, bits*i + bits), little-endian
    rng = np.random.default_rng(4)
    x = rng.normal(0, 1.5, (3, 64)).astype(np.float32)
    q, d = oracle.quant_sub(x, fmt)
    assert q.shape == (3, 64 * bits // 8)
    L = oracle.lib()
    enc = {"e2m1": L.orc_f32_to_e2m1, "e2m3": L.orc_f32_to_e2m3, "e3m2": L.orc_f32_to_e3m2}[fmt]
    for r in range(3):
        word = int.from_bytes(q[r].tobytes(), "little")
        for i in range(64):
            assert (word >> (bits * i)) & ((1 << bits) - 1) == enc(float(x[r, i]))


def test_bf16_rne():
    L = oracle.lib()
    for x, want in ((1.0, 0x3F80), (1.00390625, 0x3F80), (1.01171875, 0x3F82),
                    (-2.0, 0xC000), (3.0e38, 0x7F62)):
        assert L.orc_f32_to_bf16(x) == want
    x = np.float32(1.0) + np.float32(2 ** -8)  # exact tie between 0x3F80 and 0x3F81 -> even
    assert L.orc_f32_to_bf16(float(x)) == 0x3F80


def test_nvfp4_quantiser_bounds():
    x = oracle.gen(64, 256, 3, 1)
    q, sf, d = oracle.quant_nvfp4(x)
    blocks = x.reshape(64, 16, 16)
    db = d.reshape(64, 16, 16)
    amax = np.abs(blocks).max(axis=2, keepdims=True)
    sv = oracle.e4m3_to_f32(sf).reshape(64, 16, 1)
    # e2m1 grid steps are at most 2 scale units (4 -> 6): rounding error <= 1 scale
    # unit; values beyond 6 scale units (scale rounded down) saturate to 6.
    bound = np.maximum(sv, amax - 6 * sv) + 1e-6
    assert np.all(np.abs(db - blocks) <= bound)
    assert np.array_equal(oracle.e2m1_to_f32(q & 0xF) * oracle.e4m3_to_f32(sf).repeat(8, 1),
                          d.reshape(64, 128, 2)[:, :, 0])


def mx_restated(x, elem):
    """OCP MX v1.0 block-32 quantisation restated with numpy (frexp for the exact
    floor(log2(amax)), ldexp for the power-of-two scaling) and the brute-force RNE
    codecs above: (codes, E8M0 scale bytes)."""
    emax, codes, value, vmax, nbit = {
        "e4m3": (8, list(range(0, 127)), ocp_e4m3, 448.0, 7),
        "e2m1": (2, list(range(8)), ocp_e2m1, 6.0, 3),
        "e5m2": (15, list(range(0, 124)), ocp_e5m2, 57344.0, 7),
        "e2m3": (2, list(range(32)), lambda c: ocp_fp6(c, 2), 7.5, 5),
        "e3m2": (4, list(range(32)), lambda c: ocp_fp6(c, 3), 28.0, 5)}[elem]
    rows, cols = x.shape
    q = np.zeros((rows, cols), np.int64)
    sf = np.zeros((rows, cols // 32), np.int64)
    for r in range(rows):
        for b in range(cols // 32):
            blk = x[r, 32 * b:32 * b + 32]
            amax = float(np.abs(blk).max())
            s = (np.frexp(np.float32(amax))[1] - 1 - emax) if amax > 0 else -127
            s = max(-127, min(127, int(s)))
            sf[r, b] = s + 127
            for i, v in enumerate(blk):
                t = float(np.ldexp(np.float32(v), -s).astype(np.float32))
                c = nearest_even(min(abs(t), vmax), codes, value)
                if value(c) == 0.0:
                    c = 0
                q[r, 32 * b + i] = c | ((1 << nbit) if t < 0 and c != 0 else 0)
    return q, sf


@pytest.mark.parametrize("elem", ["e4m3", "e2m1", "e5m2", "e2m3", "e3m2"])
def test_mx_quantiser_matches_restatement(elem):
    rng = np.random.default_rng(7)
    x = oracle.gen(6, 128, 5, 1)
    # blocks of very different magnitudes, an all-zero block and a subnormal one
    x[1] *= 1e-3
    x[2] *= 300.0
    x[3, :32] = 0.0
    x[4, 32:64] = rng.normal(0, 1e-40, 32).astype(np.float32)
    q, sf, d = oracle.quant_mx(x, elem)
    wq, wsf = mx_restated(x, elem)
    assert np.array_equal(sf.astype(np.int64), wsf)
    got = q.astype(np.int64)
    if elem == "e2m1":
        got = np.stack([got & 0xF, got >> 4], axis=2).reshape(6, 128)
    if elem in ("e2m3", "e3m2"):  # 16 elements per 12 bytes, element i at bits [6i, 6i+6)
        got = np.array([[(int.from_bytes(q[r].tobytes(), "little") >> (6 * i)) & 63
                         for i in range(128)] for r in range(6)], np.int64)
    dec = np.vectorize({"e4m3": ocp_e4m3, "e2m1": ocp_e2m1, "e5m2": ocp_e5m2,
                        "e2m3": lambda c: ocp_fp6(c, 2), "e3m2": lambda c: ocp_fp6(c, 3)}[elem])
    assert np.array_equal(dec(got), dec(wq))
    # dequantised values: code value x 2^(sf - 127), exact
    scale = np.ldexp(np.float32(1.0), wsf.astype(np.int64) - 127).repeat(32, axis=1)
    assert np.array_equal(d, (dec(got) * scale).astype(np.float32))


# ---------------------------------------------------------------- 2:4
def test_metadata_pin_0x44444444():
    d = np.zeros((3, 64), np.uint16)
    d[:, 0::4] = 0x3F80
    d[:, 1::4] = 0x4000
    comp, meta = oracle.compress_24(d)
    assert (meta == 0x44444444).all()
    assert (comp[:, 0::2] == 0x3F80).all() and (comp[:, 1::2] == 0x4000).all()


@pytest.mark.parametrize("pair,nib", [((0, 1), 0x4), ((0, 2), 0x8), ((0, 3), 0xC), ((1, 2), 0x9),
                                      ((1, 3), 0xD), ((2, 3), 0xE)])
def test_metadata_nibbles(pair, nib):
    d = np.zeros((1, 32), np.uint16)
    for g in range(8):
        d[0, 4 * g + pair[0]] = 0x3F80
        d[0, 4 * g + pair[1]] = 0xBF80
    _, meta = oracle.compress_24(d)
    assert meta[0, 0] == int(f"{nib:x}" * 8, 16)


def test_prune_compress_round_trip():
    q = oracle.quant_bf16(oracle.gen(40, 256, 9, 0))[0]
    p = oracle.prune_24(q, 123)
    assert ((p.reshape(40, 64, 4) != 0).sum(axis=2) <= 2).all()
    comp, meta = oracle.compress_24(p)
    assert np.array_equal(oracle.decompress_24(comp, meta, 256), p)
    # rows of a shard prune exactly like the same rows of the whole matrix
    assert np.array_equal(oracle.prune_24(q[10:20], 123, row0=10), p[10:20])


def test_compress_rejects_three_nonzeros():
    d = np.zeros((1, 32), np.uint16)
    d[0, :3] = 0x3F80
    with pytest.raises(ValueError):
        oracle.compress_24(d)


# ---------------------------------------------------------------- GEMM
@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (3, 5, 7), (64, 48, 520), (130, 66, 1031)])
def test_gemm_against_numpy(M, N, K):
    A = oracle.gen(M, K, 1, 0)
    B = oracle.gen(N, K, 2, 0)
    ref = A.astype(np.float64) @ B.astype(np.float64).T
    got = oracle.gemm(A, B, 1.0, threads=3)
    assert np.allclose(got, ref, rtol=1e-5, atol=1e-5 * math.sqrt(K))
    got2 = oracle.gemm(A, B, 0.25, threads=1)
    assert np.allclose(got2, 0.25 * ref, rtol=1e-5, atol=1e-5 * math.sqrt(K))


def test_tolerance_check():
    ref = np.array([1.0, -2.0, 0.0, 4.0], np.float32)
    assert oracle.tolerance_check(ref * 1.005, ref, 1e-2)[0]
    assert not oracle.tolerance_check(ref * 1.05, ref, 1e-2)[0]


def test_gemm_threading_does_not_change_bits():
    # row split (few threads) and column split (many threads, few rows) give the
    # single-thread result bit for bit
    A = oracle.gen(300, 1000, 1, 1)
    B = oracle.gen(333, 1000, 2, 1)
    one = oracle.gemm(A, B, 0.5, 1)
    assert np.array_equal(one, oracle.gemm(A, B, 0.5, 2))
    assert np.array_equal(one, oracle.gemm(A, B, 0.5, 8))
    assert np.array_equal(one[:5], oracle.gemm(A[:5], B, 0.5, 8))


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2", "s8", "u8"])
def test_compress8_round_trip_and_pattern(fmt):
    # 8-bit 2:4: every pruned group holds at most 2 non-zeros at the seeded pair,
    # compress / decompress round-trips the stored codes, and the metadata of the
    # 8-bit compressor uses the 16-bit convention (idx0 | idx1 << 2, idx0 < idx1)
    q, d = oracle.operand(fmt, 16, 256, 3, 1, prune_seed=4)
    nz = (q.view(np.uint8) & oracle.NZ_MASK_8[fmt]) != 0
    assert nz.reshape(16, 64, 4).sum(axis=2).max() <= 2
    assert np.array_equal(d == 0, ~nz) or fmt in ("s8", "u8")
    comp, meta = oracle.compress_24(q, fmt)
    assert comp.shape == (16, 128) and meta.shape == (16, 8)
    back = oracle.decompress_24(comp, meta, 256)
    keep = back.view(np.uint8) & oracle.NZ_MASK_8[fmt]
    assert np.array_equal(keep, q.view(np.uint8) & oracle.NZ_MASK_8[fmt])
    nib = (meta[:, :, None] >> (4 * np.arange(8, dtype=np.uint32))) & 0xF
    assert ((nib & 3) < (nib >> 2)).all()


def test_compress8_pin_and_negative_zero():
    dense = np.zeros((2, 64), np.uint8)
    dense.reshape(2, 16, 4)[:, :, 0] = 0x38
    dense.reshape(2, 16, 4)[:, :, 1] = 0x41
    assert (oracle.compress_24(dense, "e4m3")[1] == 0x44444444).all()
    dense.reshape(2, 16, 4)[:, :, 2] = 0x80  # -0 in e4m3; -128 in s8
    assert (oracle.compress_24(dense, "e4m3")[1] == 0x44444444).all()
    with pytest.raises(ValueError):
        oracle.compress_24(dense.view(np.int8), "s8")


def test_prune8_same_positions_as_prune16():
    # the 8-bit pruner uses the 16-bit one's group counter and hash: on all-nonzero
    # data both keep the same two positions of every group
    ones16 = np.full((8, 128), 0x3F80, np.uint16)
    ones8 = np.full((8, 128), 0x38, np.uint8)
    p16 = oracle.prune_24(ones16, 9, row0=5) != 0
    p8 = oracle.prune_24(ones8, 9, row0=5) != 0
    assert np.array_equal(p16, p8) and p8.reshape(8, 32, 4).sum(axis=2).max() == 2


def test_tolerance_check_holds_both_bounds():
    ref = np.array([10.0, -10.0, 0.01, 1.0], np.float32)  # rms ~ 7.07
    tol = 1e-2
    # 1.5 % off on a large entry: inside tol * (|ref| + rms), outside tol * |ref|
    got = ref.copy()
    got[0] *= 1.015
    ok, worst = oracle.tolerance_check(got, ref, tol)
    assert not ok and 1.4 < worst < 1.6
    assert abs(oracle.relative_error(got, ref) - 0.015) < 1e-6
    # a near-zero entry may be off by tol * rms in absolute terms
    got = ref.copy()
    got[2] += 0.05
    ok, _ = oracle.tolerance_check(got, ref, tol)
    assert ok


def test_tf32_one_of_two_round_trip_and_nibbles():
    # tf32 1:2: one kept element per pair, metadata nibbles 0x4 (element 0) or 0xE
    # (element 1) -- the pair read as four 16-bit halves -- in [rows][K/16] words
    q, d = oracle.operand("tf32", 8, 128, 5, 0, prune_seed=6)
    nz = (q.view(np.uint32) & 0x7FFFFFFF) != 0
    assert nz.reshape(8, 64, 2).sum(axis=2).max() == 1
    comp, meta = oracle.compress_24(q)
    assert comp.shape == (8, 64) and meta.shape == (8, 8)
    nib = (meta[:, :, None] >> (4 * np.arange(8, dtype=np.uint32))) & 0xF
    assert set(np.unique(nib)) <= {0x4, 0xE}
    assert np.array_equal(oracle.decompress_24(comp, meta, 128).view(np.uint32) & 0x7FFFFFFF,
                          q.view(np.uint32) & 0x7FFFFFFF)
    two = np.ones((1, 16), np.float32)
    with pytest.raises(ValueError):
        oracle.compress_24(two)


def test_mx_block64_scale_is_the_larger_block32_scale():
    # one E8M0 per 64 elements (the 2:4-sparse MX GEMM's block) = the larger of the two
    # 32-element scales, since s = floor(log2(amax)) - emax is monotone in amax
    x = oracle.gen(8, 512, 3, 1)
    for elem in ("e4m3", "e5m2"):
        _, s32, _ = oracle.quant_mx(x, elem)
        q, s64, d = oracle.quant_mx(x, elem, 64)
        assert np.array_equal(s64, np.maximum(s32[:, 0::2], s32[:, 1::2]))
        scale = np.ldexp(1.0, s64.astype(np.int32) - 127).repeat(64, axis=1)
        ref = oracle.e4m3_to_f32(q) if elem == "e4m3" else None
        if ref is not None:
            assert np.array_equal(d, (ref * scale).astype(np.float32))


def test_block_scaled_operands_and_pair_compression():
    # every block-scaled operand name resolves to its quantiser (a name table shared
    # with the byte-wise compressor must not capture one)
    for fmt, sf_cols in (("mxf8", 8), ("mxf4", 8), ("nvfp4", 16), ("mx_e5m2", 8),
                         ("mx64_e4m3", 4), ("nvfp4_32", 8)):
        q, d, sf = oracle.operand(fmt, 4, 256, 3, 1)
        assert sf.shape == (4, sf_cols) and d.shape == (4, 256)
    # 4:8 in pairs: 2 of every 4 bytes of packed e2m1 kept, metadata over the bytes
    q, d, sf = oracle.operand("mx64_e2m1", 4, 256, 3, 1, prune_seed=5)
    comp, meta = oracle.compress_24(q, "mxf4")
    assert comp.shape == (4, 64) and meta.shape == (4, 4)
    back = oracle.decompress_24(comp, meta, 128)
    assert np.array_equal(np.where(back & 0x77, back, 0), np.where(q & 0x77, q, 0))
