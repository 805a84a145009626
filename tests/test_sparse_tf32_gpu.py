"""GPU parity of structured-sparse A on kind::tf32 (tcgen05.mma.sp, 1:2 sparsity).

The reference issues `tcgen05.mma.sp ... kind::tf32` only in its rate probe, with the
constant metadata word 0x44444444 (tcgen05_sparse_mma/tcgen05_sparse_mma.cu:88-111,
327-332; tcgen05_sparse_mma/REPORT.md:58-74 gives tf32's granularity as 1:2).  The
sparse MMA reads a pair of tf32 elements as a group of four 16-bit halves, so the
metadata keeps halves {0, 1} (0x4, element 0) or {2, 3} (0xE, element 1) of every
pair, and the engine's TMEM layout of it is the 16-bit one of twice the K.  The
operand is built on the device (seeded tf32 A, seeded 1:2 pruning,
b2g_compress_24_format) and by the CPU oracle; pruned words, compressed words and
metadata must agree bit for bit, and C must match the oracle's FP32 GEMM over the
pruned A within the tf32 tolerance (the bf16 bar, 1e-2).
"""
import numpy as np
import pytest
import torch

import b2g
import oracle
from gpu_util import TOL, bf16_tensor_to_f32, device_operand
from test_sparse_gpu import ready_layout

pytestmark = pytest.mark.gpu
SEED_A, SEED_B, SEED_P = 61, 62, 63


def tf32_sparse_operands(engine, M, N, K):
    A, _ = device_operand(engine, "tf32", M, K, SEED_A)
    engine.prune_24(A, SEED_P, fmt=b2g.FMT_TF32)
    comp = torch.empty(M, K // 2, dtype=torch.float32, device="cuda")
    meta = torch.empty(M, K // 16, dtype=torch.int32, device="cuda")
    engine.compress_24(A, comp, meta, fmt=b2g.FMT_TF32)
    B, _ = device_operand(engine, "tf32", N, K, SEED_B)
    engine.check()
    return A, comp, meta, B


def u32(t):
    return t.contiguous().view(torch.int32).cpu().numpy().view(np.uint32)


def check_tf32_sparse(engine, M, N, K, layout=0, **kw):
    A, comp, meta, B = tf32_sparse_operands(engine, M, N, K)
    qa, da = oracle.operand("tf32", M, K, SEED_A, 0, prune_seed=SEED_P)
    rc, rm = oracle.compress_24(qa)
    assert np.array_equal(u32(A), qa.view(np.uint32)), "pruned A differs from the oracle's"
    assert np.array_equal(u32(comp), rc.view(np.uint32)), "compressed A differs"
    assert np.array_equal(u32(meta), rm), "metadata differs"
    db = oracle.operand("tf32", N, K, SEED_B, 0)[1]
    mkw = dict(meta=meta)
    if layout == 1:
        ready = torch.empty(engine.sparse_meta_bytes(M, K, fmt=b2g.FMT_TF32) // 4,
                            dtype=torch.int32, device="cuda")
        engine.sparse_meta_prepare(meta, M, K, ready, fmt=b2g.FMT_TF32)
        mkw = dict(meta=ready, meta_layout=1)
    C = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    engine.gemm(comp, B, C, b2g.FMT_TF32, sparse=1, K=K, **mkw, **kw)
    engine.check()
    got = bf16_tensor_to_f32(C)
    assert not np.isnan(got).any()
    ok, worst = oracle.tolerance_check(got, oracle.gemm(da, db), TOL["tf32"])
    assert ok, f"sparse tf32 {M}x{N}x{K} {kw}: worst ratio {worst:.3f}"


@pytest.mark.parametrize("cg", [1, 2])
def test_tf32_sparse_small(engine, cg):
    check_tf32_sparse(engine, 256, 256, 256, cta_group=cg)


@pytest.mark.parametrize("cg,tile_n", [(1, 64), (1, 224), (2, 128), (2, 224)])
def test_tf32_sparse_tiles(engine, cg, tile_n):
    check_tf32_sparse(engine, 512, 448, 1024, cta_group=cg, tile_n=tile_n)


@pytest.mark.parametrize("cg", [1, 2])
@pytest.mark.parametrize("M,N,K", [(300, 200, 544), (129, 40, 32), (640, 1000, 2080)])
def test_tf32_sparse_ragged(engine, cg, M, N, K):
    check_tf32_sparse(engine, M, N, K, cta_group=cg)


@pytest.mark.parametrize("cg,tile_n", [(1, 224), (2, 224)])
def test_tf32_sparse_two_subtiles(engine, cg, tile_n):
    check_tf32_sparse(engine, 1024, 448, 1024, cta_group=cg, tile_n=tile_n, m_sub=2)


def test_tf32_sparse_prepared_metadata(engine):
    check_tf32_sparse(engine, 640, 448, 1536, layout=1, cta_group=2)


def test_tf32_meta_ready_is_the_16bit_layout_of_twice_k(engine):
    M, K = 200, 176  # canonical [M][K/16] words: the 16-bit layout of 2 K
    rng = np.random.default_rng(9)
    canon = rng.integers(0, 2 ** 32, size=(M, K // 16), dtype=np.uint64).astype(np.uint32)
    dev = torch.from_numpy(canon.view(np.int32)).cuda()
    ready = torch.empty(engine.sparse_meta_bytes(M, K, fmt=b2g.FMT_TF32) // 4, dtype=torch.int32,
                        device="cuda")
    engine.sparse_meta_prepare(dev, M, K, ready, fmt=b2g.FMT_TF32)
    engine.check()
    assert np.array_equal(u32(ready).reshape(-1), ready_layout(canon, M, 2 * K).reshape(-1))
