"""GPU parity of 2:4-sparse A on the sub-byte element types of kind::f8f6f4: e2m1
(fp4), e2m3 and e3m2 (fp6), stored packed in HBM and unpacked by the TMA into the
MMA's byte-per-element layout (tcgen05.mma.sp ... kind::f8f6f4).

The reference issues kind::f8f6f4 .sp for every element type of its table with the
constant metadata word 0x44444444 (tcgen05_sparse_mma/tcgen05_sparse_mma.cu:88-111,
327-332; tcgen05_sparse_mma/REPORT.md:58-74: f8f6f4 is 2:4, selector 0).  Here the
packed operand is built on the device (seeded codes, seeded 2:4 pruning of the
packed codes, b2g_compress_24_format) and independently by the CPU oracle: pruned
codes, compressed codes and metadata must agree bit for bit, and C must match the
oracle's FP32 GEMM over the pruned A within the fp4 / fp6 tolerance (5e-2).
"""
import numpy as np
import pytest
import torch

import b2g
import oracle
from gpu_util import FMT, SUB_BITS, TOL, bf16_tensor_to_f32, device_operand, to_np_u8

pytestmark = pytest.mark.gpu
SEED_A, SEED_B, SEED_P = 81, 82, 83


def check_sparse_sub(engine, fmt, M, N, K, b_fmt=None, layout=0, **kw):
    bits = SUB_BITS[fmt]
    A, _ = device_operand(engine, fmt, M, K, SEED_A)  # packed codes
    engine.prune_24(A, SEED_P, fmt=FMT[fmt])
    comp = torch.empty(M, K // 2 * bits // 8, dtype=torch.uint8, device="cuda")
    meta = torch.empty(M, K // 32, dtype=torch.int32, device="cuda")
    engine.compress_24(A, comp, meta, fmt=FMT[fmt])
    b_fmt = b_fmt or fmt
    B, _ = device_operand(engine, b_fmt, N, K, SEED_B)
    engine.check()
    qa, da = oracle.operand(fmt, M, K, SEED_A, 1, prune_seed=SEED_P)
    rc, rm = oracle.compress_24(qa, fmt)
    assert np.array_equal(to_np_u8(A), qa), "pruned A differs from the oracle's"
    assert np.array_equal(to_np_u8(comp), rc), "compressed A differs"
    assert np.array_equal(meta.cpu().numpy().view(np.uint32), rm), "metadata differs"
    db = oracle.operand(b_fmt, N, K, SEED_B, 1)[1]
    mkw = dict(meta=meta)
    if layout == 1:
        ready = torch.empty(engine.sparse_meta_bytes(M, K, fmt=FMT[fmt]) // 4, dtype=torch.int32,
                            device="cuda")
        engine.sparse_meta_prepare(meta, M, K, ready, fmt=FMT[fmt])
        mkw = dict(meta=ready, meta_layout=1)
    if b_fmt != fmt:
        kw["b_format"] = FMT[b_fmt]
    C = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    engine.gemm(comp, B, C, FMT[fmt], sparse=1, K=K, **mkw, **kw)
    engine.check()
    got = bf16_tensor_to_f32(C)
    assert not np.isnan(got).any(), "C has unwritten entries"
    ok, worst = oracle.tolerance_check(got, oracle.gemm(da, db), TOL[fmt])
    assert ok, f"sparse {fmt} {M}x{N}x{K} {kw}: worst ratio {worst:.3f}"


@pytest.mark.parametrize("fmt", ["e2m1", "e2m3", "e3m2"])
@pytest.mark.parametrize("cg", [1, 2])
def test_sparse_sub_small(engine, fmt, cg):
    check_sparse_sub(engine, fmt, 256, 256, 512, cta_group=cg)


@pytest.mark.parametrize("fmt", ["e2m1", "e3m2"])
@pytest.mark.parametrize("cg,tile_n", [(1, 64), (1, 224), (2, 128), (2, 224)])
def test_sparse_sub_tiles(engine, fmt, cg, tile_n):
    check_sparse_sub(engine, fmt, 512, 448, 1024, cta_group=cg, tile_n=tile_n)


@pytest.mark.parametrize("fmt", ["e2m1", "e2m3"])
@pytest.mark.parametrize("cg", [1, 2])
@pytest.mark.parametrize("M,N,K", [(300, 200, 512), (129, 40, 256), (640, 1000, 2304)])
def test_sparse_sub_ragged(engine, fmt, cg, M, N, K):
    check_sparse_sub(engine, fmt, M, N, K, cta_group=cg)


@pytest.mark.parametrize("fmt", ["e2m1", "e3m2"])
def test_sparse_sub_two_subtiles_and_prepared_metadata(engine, fmt):
    check_sparse_sub(engine, fmt, 1024, 448, 1024, cta_group=2, tile_n=224, m_sub=2)
    check_sparse_sub(engine, fmt, 640, 448, 1536, layout=1, cta_group=2)


@pytest.mark.parametrize("a,b", [("e2m1", "e4m3"), ("e3m2", "e2m1")])
def test_sparse_sub_type_mix(engine, a, b):
    # kind::f8f6f4 takes any A x B pair of its element types, with sparse A too
    check_sparse_sub(engine, a, 384, 320, 1024, b_fmt=b, cta_group=2)
