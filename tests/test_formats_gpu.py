"""GPU parity of the GEMM on the remaining dense tcgen05 kinds, through the C ABI:
int8 (kind::i8, s32 accumulator), tf32 (kind::tf32), and the f8f6f4 element types
e5m2, e2m1, e2m3 and e3m2 (the last three packed in memory and unpacked by the
TMA into the MMA's 16-byte chunks).  The reference runs these element types only
as MMA issue loops (umma_throughput/umma_tput.cu:68-75 MMAFormat::S8 / F4;
tcgen05_sparse_mma/Makefile:64-103 tf32 / e5m2 / e2m3 / e3m2 / e2m1), never
reading D back.

int8 is checked bit for bit: its accumulation is exact and C is a defined
rounding of it (fp32(acc) to nearest even, times alpha in fp32, bf16 to nearest
even).  tf32 is held to the bf16 tolerance and e5m2 to the fp8 tolerance.
"""
import numpy as np
import pytest
import torch

import b2g
import oracle
from gpu_util import ALPHA, FMT, TOL, bf16_tensor_to_f32, device_operand, host_operand, to_np_u16

pytestmark = pytest.mark.gpu


def stored_bytes(fmt, t):
    if fmt == "tf32":
        return t.contiguous().cpu().numpy().view(np.float32)
    a = t.contiguous().view(torch.uint8).cpu().numpy()
    return a.view(np.int8) if fmt == "s8" else (a.view(np.uint16) if fmt == "f16" else a)


def check(engine, fmt, M, N, K, seed_a=11, seed_b=22, b_fmt=None, **kw):
    b_fmt = b_fmt or fmt
    A, _ = device_operand(engine, fmt, M, K, seed_a)
    B, _ = device_operand(engine, b_fmt, N, K, seed_b)
    C = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    if b_fmt != fmt:
        kw["b_format"] = FMT[b_fmt]
    engine.gemm(A, B, C, FMT[fmt], alpha=ALPHA[fmt], **kw)
    engine.check()
    qa, da = host_operand(fmt, M, K, seed_a)
    qb, db = host_operand(b_fmt, N, K, seed_b)
    # the device quantiser must produce the oracle's operands bit for bit
    assert np.array_equal(stored_bytes(fmt, A).view(qa.dtype), qa)
    assert np.array_equal(stored_bytes(b_fmt, B).view(qb.dtype), qb)
    if fmt in ("s8", "u8"):
        want = oracle.gemm_s8_exact(qa, qb, ALPHA[fmt])
        got = to_np_u16(C)
        bad = np.argwhere(got != want)
        assert bad.size == 0, f"{fmt} {M}x{N}x{K} {kw}: {len(bad)} entries differ, first {bad[:3]}"
        return
    ref = oracle.gemm(da, db, ALPHA[fmt])
    got = bf16_tensor_to_f32(C)
    assert not np.isnan(got).any(), "C has unwritten entries"
    ok, worst = oracle.tolerance_check(got, ref, TOL[fmt])
    assert ok, f"{fmt} {M}x{N}x{K} {kw}: worst error ratio {worst:.3f}"


BYTE_FORMATS = ["s8", "u8", "tf32", "e5m2", "f16"]
SUB_FORMATS = ["e2m1", "e2m3", "e3m2"]  # K, lda, ldb multiples of 128
FORMATS = BYTE_FORMATS + SUB_FORMATS


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("cg,tile_n", [(1, 64), (1, 128), (1, 256), (2, 128), (2, 256)])
def test_tiles(engine, fmt, cg, tile_n):
    check(engine, fmt, 512, 512, 1024, cta_group=cg, tile_n=tile_n)


@pytest.mark.parametrize("fmt", BYTE_FORMATS)
@pytest.mark.parametrize("cg", [1, 2])
@pytest.mark.parametrize("M,N,K", [(300, 200, 528), (257, 196, 64), (129, 8, 16), (1, 1000, 2064)])
def test_ragged(engine, fmt, cg, M, N, K):
    check(engine, fmt, M, N, K, cta_group=cg)


@pytest.mark.parametrize("fmt", SUB_FORMATS)
@pytest.mark.parametrize("cg", [1, 2])
@pytest.mark.parametrize("M,N,K", [(300, 200, 512), (257, 196, 128), (129, 8, 128), (1, 1000, 2048)])
def test_ragged_sub_byte(engine, fmt, cg, M, N, K):
    check(engine, fmt, M, N, K, cta_group=cg)


@pytest.mark.parametrize("fmt", SUB_FORMATS)
def test_sub_byte_full_grid(engine, fmt):
    # the full 74-pair grid, several waves, on packed operands
    check(engine, fmt, 2048, 2048, 1024, cta_group=2, tile_n=256)


@pytest.mark.parametrize("fmt", FORMATS)
def test_persistent_small_grid_and_stages(engine, fmt):
    # a few CTAs walk many tiles (ring wrap-around, both TMEM buffers), shallow ring
    check(engine, fmt, 1024, 768, 512, cta_group=2, max_ctas=4, stages=2)
    check(engine, fmt, 1024, 768, 512, cta_group=1, max_ctas=3)


@pytest.mark.parametrize("fmt", ["tf32", "e5m2", "e2m1", "e3m2"])
def test_split_tail(engine, fmt):
    # 20 tiles on 16 pairs: the last wave's 4 tiles are cut into 2 K ranges
    check(engine, fmt, 1280, 1024, 2048, cta_group=2, tile_n=256, max_ctas=32, split_tail=2)


@pytest.mark.parametrize("fmt", ["s8", "u8"])
def test_i8_large_accumulator_is_exact(engine, fmt):
    # K = 16384: u8 sums reach ~3e8, far above fp32's 2^24 integer range; the s32
    # accumulator keeps them exact and C is their defined rounding
    check(engine, fmt, 256, 256, 16384, cta_group=2)


@pytest.mark.parametrize("fmt", FORMATS)
def test_host_path(engine, fmt):
    # b2g_gemm_host: host operands in, host C out, same values as the device path
    M, N, K = 640, 512, 768
    A, _ = device_operand(engine, fmt, M, K, 11)
    B, _ = device_operand(engine, fmt, N, K, 22)
    Cd = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    engine.gemm(A, B, Cd, FMT[fmt], alpha=ALPHA[fmt], split_tail=1)
    engine.check()
    Ah, Bh = A.cpu().pin_memory(), B.cpu().pin_memory()
    Ch = torch.empty((M, N), dtype=torch.bfloat16).pin_memory()
    engine.gemm_host(Ah, Bh, Ch, FMT[fmt], alpha=ALPHA[fmt])
    assert torch.equal(Ch.view(torch.int16), Cd.cpu().view(torch.int16))



# A and B of different kind::f8f6f4 element types (the reference's f8f6f4 pair table,
# tcgen05_sparse_mma/benchmark.py:103-107): each operand keeps its own packing
MIXES = [("e4m3", "e2m1"), ("e2m1", "e4m3"), ("e5m2", "e3m2"), ("e2m3", "e2m1"),
         ("e4m3", "e5m2"), ("e3m2", "e2m3")]


@pytest.mark.parametrize("a_fmt,b_fmt", MIXES)
@pytest.mark.parametrize("cg,tile_n", [(1, 128), (2, 256)])
def test_f8f6f4_type_mixes(engine, a_fmt, b_fmt, cg, tile_n):
    check(engine, a_fmt, 512, 384, 1024, b_fmt=b_fmt, cta_group=cg, tile_n=tile_n)


@pytest.mark.parametrize("a_fmt,b_fmt", [("e4m3", "e2m1"), ("e2m3", "e5m2")])
def test_f8f6f4_type_mix_ragged_and_split(engine, a_fmt, b_fmt):
    check(engine, a_fmt, 300, 200, 512, b_fmt=b_fmt, cta_group=2)
    check(engine, a_fmt, 1280, 1024, 2048, b_fmt=b_fmt, cta_group=2, tile_n=256, max_ctas=32,
          split_tail=2)


# OCP MX block scaling (one E8M0 per 32 K) on every kind::f8f6f4 element type, through
# kind::mxf8f6f4 (the reference's mxf8f6f4 pair table, tcgen05_sparse_mma/benchmark.py:
# 103-116); e4m3 x e4m3 is B2G_FMT_MXF8, tested with the block-scaled formats
MX_BITS = {"e4m3": 8, "e5m2": 8, "e2m1": 4, "e2m3": 6, "e3m2": 6}


def mx_operand(engine, elem, rows, cols, seed):
    x = torch.empty(rows, cols, dtype=torch.float32, device="cuda")
    engine.fill(x, seed, 1)
    q = torch.empty(rows, cols * MX_BITS[elem] // 8, dtype=torch.uint8, device="cuda")
    sf = torch.empty(rows, cols // 32, dtype=torch.uint8, device="cuda")
    engine.quantize_mx(FMT[elem], x, q, sf)
    return q, sf


def check_mx(engine, a_elem, b_elem, M, N, K, **kw):
    A, sfa = mx_operand(engine, a_elem, M, K, 11)
    B, sfb = mx_operand(engine, b_elem, N, K, 22)
    C = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    if b_elem != a_elem:
        kw["b_format"] = FMT[b_elem]
    engine.gemm(A, B, C, FMT[a_elem], sfa=sfa, sfb=sfb, mx_scale=1, **kw)
    engine.check()
    qa, da, sa = oracle.operand("mx_" + a_elem, M, K, 11, 1)
    qb, db, sb = oracle.operand("mx_" + b_elem, N, K, 22, 1)
    assert np.array_equal(A.cpu().numpy(), qa) and np.array_equal(sfa.cpu().numpy(), sa)
    assert np.array_equal(B.cpu().numpy(), qb) and np.array_equal(sfb.cpu().numpy(), sb)
    got = bf16_tensor_to_f32(C)
    assert not np.isnan(got).any(), "C has unwritten entries"
    ok, worst = oracle.tolerance_check(got, oracle.gemm(da, db), 5e-2)
    assert ok, f"mx {a_elem}x{b_elem} {M}x{N}x{K} {kw}: worst error ratio {worst:.3f}"


@pytest.mark.parametrize("elem", ["e5m2", "e2m1", "e2m3", "e3m2", "e4m3"])
@pytest.mark.parametrize("kw", [dict(cta_group=1, tile_n=128), dict(cta_group=2, tile_n=224),
                                dict(cta_group=2, tile_n=224, m_sub=1)])
def test_mx_element_types(engine, elem, kw):
    check_mx(engine, elem, elem, 512, 448, 1024, **kw)


@pytest.mark.parametrize("a_elem,b_elem", [("e4m3", "e2m1"), ("e2m3", "e5m2"), ("e3m2", "e2m1")])
def test_mx_type_mixes(engine, a_elem, b_elem):
    check_mx(engine, a_elem, b_elem, 512, 448, 1024, cta_group=2)


@pytest.mark.parametrize("elem", ["e5m2", "e2m3"])
def test_mx_ragged(engine, elem):
    check_mx(engine, elem, elem, 300, 200, 512, cta_group=2)
    check_mx(engine, elem, elem, 129, 40, 128, cta_group=1)


@pytest.mark.parametrize("a_fmt,b_fmt", [("e2m1", "e2m1"), ("e4m3", "e2m3"), ("f16", "f16")])
def test_dense_two_subtiles_other_types(engine, a_fmt, b_fmt):
    check(engine, a_fmt, 1000, 900, 1024, b_fmt=b_fmt, cta_group=2, tile_n=224, m_sub=2)
