"""GPU parity of the NVFP4 block-scaled GEMM (kind::mxf4nvf4.block_scale.block16):
e2m1 operands packed two per byte, one ue4m3 scale per 16 K elements, fp32
accumulate, bf16 C.  Operands are quantised on the device (bit-exact with the
oracle, tests/test_datagen_gpu.py); C is compared with the oracle's FP32 GEMM
over the dequantised operands within the fp4 tolerance (5e-2)."""
import numpy as np
import pytest
import torch

import b2g
import oracle
from gpu_util import TOL, bf16_tensor_to_f32, to_np_u8

pytestmark = pytest.mark.gpu
SEED_A, SEED_B = 51, 52


def nvfp4_operand(engine, rows, K, seed, row0=0):
    x = torch.empty(rows, K, dtype=torch.float32, device="cuda")
    engine.fill(x, seed, 1, row0=row0)
    q = torch.empty(rows, K // 2, dtype=torch.uint8, device="cuda")
    sf = torch.empty(rows, K // 16, dtype=torch.uint8, device="cuda")
    engine.quantize(b2g.FMT_NVFP4, x, q, sf)
    return q, sf


def check_nvfp4(engine, M, N, K, **kw):
    A, sfa = nvfp4_operand(engine, M, K, SEED_A)
    B, sfb = nvfp4_operand(engine, N, K, SEED_B)
    C = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    engine.gemm(A, B, C, b2g.FMT_NVFP4, sfa=sfa, sfb=sfb, **kw)
    engine.check()
    qa, da, sa = oracle.operand("nvfp4", M, K, SEED_A, 1)
    qb, db, sb = oracle.operand("nvfp4", N, K, SEED_B, 1)
    assert np.array_equal(to_np_u8(A), qa) and np.array_equal(to_np_u8(sfa), sa)
    ref = oracle.gemm(da, db)
    got = bf16_tensor_to_f32(C)
    assert not np.isnan(got).any()
    ok, worst = oracle.tolerance_check(got, ref, TOL["nvfp4"])
    assert ok, f"nvfp4 {M}x{N}x{K} {kw}: worst ratio {worst:.3f}"
    return C


@pytest.mark.parametrize("cg", [1, 2])
def test_nvfp4_small(engine, cg):
    check_nvfp4(engine, 256, 192, 256, cta_group=cg)


@pytest.mark.parametrize("cg,tile_n", [(1, 64), (1, 128), (1, 224), (2, 64), (2, 128), (2, 224)])
def test_nvfp4_tiles(engine, cg, tile_n):
    check_nvfp4(engine, 384, 512, 1024, cta_group=cg, tile_n=tile_n)


@pytest.mark.parametrize("cg", [1, 2])
@pytest.mark.parametrize("M,N,K", [(300, 200, 544), (129, 40, 32), (640, 1000, 2080)])
def test_nvfp4_ragged(engine, cg, M, N, K):
    check_nvfp4(engine, M, N, K, cta_group=cg)


@pytest.mark.parametrize("cg", [1, 2])
def test_nvfp4_persistent_small_grid(engine, cg):
    check_nvfp4(engine, 1024, 768, 512, cta_group=cg, max_ctas=4)


# two 128-row A sub-tiles per CTA share one B tile and its scale factors
@pytest.mark.parametrize("cg,tile_n", [(1, 64), (1, 224), (2, 128), (2, 224)])
def test_nvfp4_two_subtiles(engine, cg, tile_n):
    check_nvfp4(engine, 1024, 448, 1024, cta_group=cg, tile_n=tile_n, m_sub=2)


@pytest.mark.parametrize("cg", [1, 2])
@pytest.mark.parametrize("M,N,K", [(300, 200, 544), (129, 40, 32), (640, 1000, 2080)])
def test_nvfp4_two_subtiles_ragged(engine, cg, M, N, K):
    check_nvfp4(engine, M, N, K, cta_group=cg, m_sub=2)


def test_nvfp4_two_subtiles_small_grid_matches_one(engine):
    C1 = check_nvfp4(engine, 2048, 672, 1024, cta_group=2, m_sub=1, split_tail=1)
    C2 = check_nvfp4(engine, 2048, 672, 1024, cta_group=2, m_sub=2, max_ctas=6)
    assert torch.equal(C1, C2)


def test_nvfp4_rejects_tile_without_tmem_room(engine):
    A, sfa = nvfp4_operand(engine, 256, 256, SEED_A)
    C = torch.empty(256, 256, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(b2g.B2GError) as e:
        engine.gemm(A, A, C, b2g.FMT_NVFP4, sfa=sfa, sfb=sfa, tile_n=256)
    assert e.value.status == 1


@pytest.mark.parametrize("cg", [2, 1])
def test_nvfp4_full_size_cfg4_sampled(engine, cg):
    # BASELINE cfg4: M = N = K = 16384
    M = N = K = 16384
    A, sfa = nvfp4_operand(engine, M, K, SEED_A)
    B, sfb = nvfp4_operand(engine, N, K, SEED_B)
    C = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    engine.gemm(A, B, C, b2g.FMT_NVFP4, sfa=sfa, sfb=sfb, cta_group=cg)
    engine.check()
    rng = np.random.default_rng(4)
    rows = np.sort(rng.choice(M, 12, replace=False))
    cols = np.sort(rng.choice(N, 12, replace=False))
    da = np.stack([oracle.operand("nvfp4", 1, K, SEED_A, 1, int(r))[1][0] for r in rows])
    db = np.stack([oracle.operand("nvfp4", 1, K, SEED_B, 1, int(c))[1][0] for c in cols])
    ref = oracle.gemm(da, db)
    got = bf16_tensor_to_f32(C[torch.as_tensor(rows, device="cuda")][:, torch.as_tensor(cols, device="cuda")])
    ok, worst = oracle.tolerance_check(got, ref, TOL["nvfp4"])
    assert ok, f"cfg4 sampled worst ratio {worst:.3f}"
    assert not torch.isnan(C).any()


def test_nvfp4_scratch_growth_keeps_other_handle_buffers():
    # growing a fresh handle's scale-factor scratch must leave the probe's result
    # buffer alone: probe, grow the scratch twice with NVFP4 calls, probe again
    eng = b2g.Engine(0)
    try:
        eng.probe_mma(kind=1, a_type=1, b_type=1, cta_group=1, m=128, n=256, k=16, depth=4, iters=10)
        check_nvfp4(eng, 256, 256, 256, cta_group=2)
        check_nvfp4(eng, 2304, 256, 2048, cta_group=2)
        cyc, tot, _ = eng.probe_mma(kind=1, a_type=1, b_type=1, cta_group=1, m=128, n=256, k=16,
                                    depth=4, iters=10)
        assert tot == 40 and cyc > 0
    finally:
        eng.close()
