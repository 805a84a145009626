"""GPU parity of structured-sparse A on kind::mxf4nvf4 with ue4m3 scales
(tcgen05.mma.sp ... kind::mxf4nvf4.block_scale.block16): NVFP4 packed e2m1
operands, A sparse 4:8 in pairs.

The reference issues kind::mxf4nvf4 .sp only as a build target of its rate probe
(with E8M0 scales, block32) and the constant metadata word 0x44444444
(tcgen05_sparse_mma/tcgen05_sparse_mma.cu:105-108,327-332; REPORT.md:58-74 gives
mxf4nvf4's granularity as "4:8 in pairs").  In
pairs means a byte of packed e2m1 (two elements) is the unit: 2 of every 4 bytes
are kept, so the compressor, the metadata words and the TMEM layout are the 8-bit
ones over the bytes (K / 2 of them).  A sparse MMA spans 128 dense K and reads four
ue4m3 scales per row, as the dense block16 MMA does for its 64, so each scale
covers 32 dense K: the operands carry one scale per 32 elements
(b2g_quantize_nvfp4_block with block 32).  Codes, scales, compressed bytes and
metadata must agree with the CPU oracle bit for bit, and C must match the oracle's
FP32 GEMM over the dequantised pruned A within the fp4 tolerance (5e-2).  The
scale-factor blocks take 48 TMEM columns per ring slot, so the default tile is 192
columns.
"""
import numpy as np
import pytest
import torch

import b2g
import oracle
from gpu_util import TOL, bf16_tensor_to_f32, to_np_u8

pytestmark = pytest.mark.gpu
SEED_A, SEED_B, SEED_P = 95, 96, 97


def nvfp4_codes(engine, rows, K, seed):
    x = torch.empty(rows, K, dtype=torch.float32, device="cuda")
    engine.fill(x, seed, 1)
    q = torch.empty(rows, K // 2, dtype=torch.uint8, device="cuda")
    sf = torch.empty(rows, K // 32, dtype=torch.uint8, device="cuda")
    engine.quantize_nvfp4(x, q, sf, block=32)
    return q, sf


def check_sparse_nvfp4(engine, M, N, K, layout=0, **kw):
    A, sfa = nvfp4_codes(engine, M, K, SEED_A)
    engine.prune_24(A, SEED_P, fmt=b2g.FMT_NVFP4)
    comp = torch.empty(M, K // 4, dtype=torch.uint8, device="cuda")
    meta = torch.empty(M, K // 64, dtype=torch.int32, device="cuda")
    engine.compress_24(A, comp, meta, fmt=b2g.FMT_NVFP4)
    B, sfb = nvfp4_codes(engine, N, K, SEED_B)
    engine.check()
    qa, da, sa = oracle.operand("nvfp4_32", M, K, SEED_A, 1, prune_seed=SEED_P)
    qb, db, sb = oracle.operand("nvfp4_32", N, K, SEED_B, 1)
    rc, rm = oracle.compress_24(qa, "mxf4")
    assert np.array_equal(to_np_u8(A), qa) and np.array_equal(to_np_u8(sfa), sa)
    assert np.array_equal(to_np_u8(comp), rc), "compressed A differs"
    assert np.array_equal(meta.cpu().numpy().view(np.uint32), rm), "metadata differs"
    assert np.array_equal(to_np_u8(B), qb) and np.array_equal(to_np_u8(sfb), sb)
    mkw = dict(meta=meta)
    if layout == 1:
        ready = torch.empty(engine.sparse_meta_bytes(M, K, fmt=b2g.FMT_NVFP4) // 4,
                            dtype=torch.int32, device="cuda")
        engine.sparse_meta_prepare(meta, M, K, ready, fmt=b2g.FMT_NVFP4)
        mkw = dict(meta=ready, meta_layout=1)
    C = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    engine.gemm(comp, B, C, b2g.FMT_NVFP4, sparse=1, K=K, sfa=sfa, sfb=sfb, **mkw, **kw)
    engine.check()
    got = bf16_tensor_to_f32(C)
    assert not np.isnan(got).any(), "C has unwritten entries"
    ok, worst = oracle.tolerance_check(got, oracle.gemm(da, db), TOL["nvfp4"])
    assert ok, f"sparse NVFP4 {M}x{N}x{K} {kw}: worst ratio {worst:.3f}"


@pytest.mark.parametrize("cg", [1, 2])
def test_sparse_nvfp4_small(engine, cg):
    check_sparse_nvfp4(engine, 256, 256, 1024, cta_group=cg)


@pytest.mark.parametrize("cg,tile_n", [(1, 64), (1, 192), (2, 128), (2, 192)])
def test_sparse_nvfp4_tiles(engine, cg, tile_n):
    check_sparse_nvfp4(engine, 512, 448, 2048, cta_group=cg, tile_n=tile_n)


@pytest.mark.parametrize("cg", [1, 2])
@pytest.mark.parametrize("M,N,K", [(300, 200, 576), (129, 40, 64), (640, 1000, 2112)])
def test_sparse_nvfp4_ragged(engine, cg, M, N, K):
    check_sparse_nvfp4(engine, M, N, K, cta_group=cg)


def test_sparse_nvfp4_two_subtiles_small_grid_prepared_metadata(engine):
    check_sparse_nvfp4(engine, 1024, 448, 2048, cta_group=2, tile_n=192, m_sub=2)
    check_sparse_nvfp4(engine, 1024, 672, 2048, cta_group=2, max_ctas=4, stages=2)
    check_sparse_nvfp4(engine, 640, 448, 1536, layout=1, cta_group=2)
