"""GPU parity of 2:4-sparse A on the block-scaled kind::mxf8f6f4
(tcgen05.mma.sp ... kind::mxf8f6f4.block_scale): MX e4m3 / e5m2 operands, A pruned
2:4 on its stored codes.  A sparse MMA spans 64 dense K and applies ONE E8M0 scale
per row of A and of B to all of them (measured on the B200: the scale byte the MMA
names weighs both 32-element halves), so these operands carry one scale per 64 K
(b2g_quantize_mx_block with block 64), the OCP MX block of the 32 kept elements.

The reference issues this form only in its single-tile rate probe, with constant
metadata (0x44444444) and constant scale factors
(tcgen05_sparse_mma/tcgen05_sparse_mma.cu:104-105,196-202,320-332; REPORT.md:58-74
gives mxf8f6f4's granularity as 2:4).  Here the operand is quantised on the
device (b2g_quantize_mx), pruned (b2g_prune_24_format on the codes) and
compressed (b2g_compress_24_format), and independently by the CPU oracle: codes,
scales, compressed values and metadata must agree bit for bit.  C must match the
oracle's FP32 GEMM over the dequantised pruned A within the fp8 tolerance (5e-2).
The cases cover all four scale bytes of a ring slot's group and K over several
ring slots.
"""
import numpy as np
import pytest
import torch

import b2g
import oracle
from gpu_util import TOL, bf16_tensor_to_f32, to_np_u8

pytestmark = pytest.mark.gpu
SEED_A, SEED_B, SEED_P = 71, 72, 73
ELEM = {"e4m3": b2g.FMT_E4M3, "e5m2": b2g.FMT_E5M2}


def mx_codes(engine, elem, rows, K, seed):
    x = torch.empty(rows, K, dtype=torch.float32, device="cuda")
    engine.fill(x, seed, 1)
    q = torch.empty(rows, K, dtype=torch.uint8, device="cuda")
    sf = torch.empty(rows, K // 64, dtype=torch.uint8, device="cuda")
    engine.quantize_mx(ELEM[elem], x, q, sf, block=64)
    return q, sf


def check_sparse_mx(engine, elem, M, N, K, layout=0, **kw):
    A, sfa = mx_codes(engine, elem, M, K, SEED_A)
    engine.prune_24(A, SEED_P, fmt=ELEM[elem])
    comp = torch.empty(M, K // 2, dtype=torch.uint8, device="cuda")
    meta = torch.empty(M, K // 32, dtype=torch.int32, device="cuda")
    engine.compress_24(A, comp, meta, fmt=ELEM[elem])
    B, sfb = mx_codes(engine, elem, N, K, SEED_B)
    engine.check()
    qa, da, sa = oracle.operand("mx64_" + elem, M, K, SEED_A, 1, prune_seed=SEED_P)
    qb, db, sb = oracle.operand("mx64_" + elem, N, K, SEED_B, 1)
    rc, rm = oracle.compress_24(qa, elem)
    assert np.array_equal(to_np_u8(A), qa) and np.array_equal(to_np_u8(sfa), sa)
    assert np.array_equal(to_np_u8(comp), rc.view(np.uint8))
    assert np.array_equal(meta.cpu().numpy().view(np.uint32), rm)
    assert np.array_equal(to_np_u8(B), qb) and np.array_equal(to_np_u8(sfb), sb)
    mkw = dict(meta=meta)
    if layout == 1:
        ready = torch.empty(engine.sparse_meta_bytes(M, K, fmt=ELEM[elem]) // 4,
                            dtype=torch.int32, device="cuda")
        engine.sparse_meta_prepare(meta, M, K, ready, fmt=ELEM[elem])
        mkw = dict(meta=ready, meta_layout=1)
    C = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    engine.gemm(comp, B, C, ELEM[elem], sparse=1, K=K, sfa=sfa, sfb=sfb, mx_scale=1, **mkw, **kw)
    engine.check()
    got = bf16_tensor_to_f32(C)
    assert not np.isnan(got).any(), "C has unwritten entries"
    ok, worst = oracle.tolerance_check(got, oracle.gemm(da, db), TOL["mxf8"])
    assert ok, f"sparse MX {elem} {M}x{N}x{K} {kw}: worst ratio {worst:.3f}"
    return C


@pytest.mark.parametrize("elem", ["e4m3", "e5m2"])
@pytest.mark.parametrize("cg", [1, 2])
def test_sparse_mx_small(engine, elem, cg):
    check_sparse_mx(engine, elem, 256, 256, 512, cta_group=cg)


@pytest.mark.parametrize("cg,tile_n", [(1, 64), (1, 128), (1, 224), (2, 128), (2, 224)])
def test_sparse_mx_tiles(engine, cg, tile_n):
    check_sparse_mx(engine, "e4m3", 512, 448, 1024, cta_group=cg, tile_n=tile_n)


@pytest.mark.parametrize("cg", [1, 2])
@pytest.mark.parametrize("M,N,K", [(300, 200, 576), (129, 40, 64), (640, 1000, 2112)])
def test_sparse_mx_ragged(engine, cg, M, N, K):
    check_sparse_mx(engine, "e4m3", M, N, K, cta_group=cg)


@pytest.mark.parametrize("cg,tile_n", [(1, 128), (2, 192)])
def test_sparse_mx_two_subtiles(engine, cg, tile_n):
    check_sparse_mx(engine, "e4m3", 1024, 448, 1024, cta_group=cg, tile_n=tile_n, m_sub=2)


def test_sparse_mx_small_grid_stages_prepared_metadata(engine):
    check_sparse_mx(engine, "e4m3", 1024, 672, 2048, cta_group=2, max_ctas=4, stages=2)
    check_sparse_mx(engine, "e5m2", 640, 448, 1536, layout=1, cta_group=2)


def test_sparse_mx_mxf8_format_code(engine):
    # B2G_FMT_MXF8 names e4m3 with MX scales: the same GEMM as E4M3 + mx_scale
    M, N, K = 384, 320, 1024
    A, sfa = mx_codes(engine, "e4m3", M, K, SEED_A)
    engine.prune_24(A, SEED_P, fmt=b2g.FMT_MXF8)
    comp = torch.empty(M, K // 2, dtype=torch.uint8, device="cuda")
    meta = torch.empty(M, K // 32, dtype=torch.int32, device="cuda")
    engine.compress_24(A, comp, meta, fmt=b2g.FMT_MXF8)
    B, sfb = mx_codes(engine, "e4m3", N, K, SEED_B)
    C0 = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    C1 = torch.empty_like(C0)
    engine.gemm(comp, B, C0, b2g.FMT_MXF8, sparse=1, K=K, sfa=sfa, sfb=sfb, meta=meta)
    engine.gemm(comp, B, C1, b2g.FMT_E4M3, sparse=1, K=K, sfa=sfa, sfb=sfb, meta=meta, mx_scale=1)
    engine.check()
    assert torch.equal(C0.view(torch.int16), C1.view(torch.int16))
