"""GPU parity of the OCP MX block-scaled GEMMs: MXFP8 (e4m3 operands,
kind::mxf8f6f4.block_scale) and MXFP4 (packed e2m1, kind::mxf4.block_scale.block32),
one E8M0 scale per 32 K elements, fp32 accumulate, bf16 C.

Operands are quantised on the device (bit-exact with the oracle,
tests/test_datagen_gpu.py); C is compared with the oracle's FP32 GEMM over the
dequantised operands within the 5e-2 tolerance.  One tcgen05.cp of a 32-row x
16-byte block carries the scales of 4 MXFP8 MMAs (or 2 MXFP4 MMAs); each MMA
selects its byte with the scale-factor ids of the instruction descriptor, so the
parity cases cover every byte position (K spans several ring slots).
"""
import numpy as np
import pytest
import torch

import b2g
import oracle
from gpu_util import FMT, TOL, bf16_tensor_to_f32, to_np_u8

pytestmark = pytest.mark.gpu
SEED_A, SEED_B = 61, 62


def mx_operand(engine, fmt, rows, K, seed, row0=0):
    x = torch.empty(rows, K, dtype=torch.float32, device="cuda")
    engine.fill(x, seed, 1, row0=row0)
    q = torch.empty(rows, K if fmt == "mxf8" else K // 2, dtype=torch.uint8, device="cuda")
    sf = torch.empty(rows, K // 32, dtype=torch.uint8, device="cuda")
    engine.quantize(FMT[fmt], x, q, sf)
    return q, sf


def check_mx(engine, fmt, M, N, K, **kw):
    A, sfa = mx_operand(engine, fmt, M, K, SEED_A)
    B, sfb = mx_operand(engine, fmt, N, K, SEED_B)
    C = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    engine.gemm(A, B, C, FMT[fmt], sfa=sfa, sfb=sfb, **kw)
    engine.check()
    qa, da, sa = oracle.operand(fmt, M, K, SEED_A, 1)
    qb, db, sb = oracle.operand(fmt, N, K, SEED_B, 1)
    assert np.array_equal(to_np_u8(A), qa) and np.array_equal(to_np_u8(sfa), sa)
    ref = oracle.gemm(da, db)
    got = bf16_tensor_to_f32(C)
    assert not np.isnan(got).any()
    ok, worst = oracle.tolerance_check(got, ref, TOL[fmt])
    assert ok, f"{fmt} {M}x{N}x{K} {kw}: worst ratio {worst:.3f}"
    return C


@pytest.mark.parametrize("fmt", ["mxf8", "mxf4"])
@pytest.mark.parametrize("cg", [1, 2])
def test_mx_small(engine, fmt, cg):
    check_mx(engine, fmt, 256, 192, 512, cta_group=cg)


@pytest.mark.parametrize("fmt", ["mxf8", "mxf4"])
@pytest.mark.parametrize("cg,tile_n", [(1, 64), (1, 224), (2, 128), (2, 224)])
def test_mx_tiles(engine, fmt, cg, tile_n):
    check_mx(engine, fmt, 384, 512, 1024, cta_group=cg, tile_n=tile_n)


@pytest.mark.parametrize("fmt", ["mxf8", "mxf4"])
@pytest.mark.parametrize("cg", [1, 2])
@pytest.mark.parametrize("M,N,K", [(300, 200, 544), (129, 40, 32), (640, 1000, 2080)])
def test_mx_ragged(engine, fmt, cg, M, N, K):
    check_mx(engine, fmt, M, N, K, cta_group=cg)


@pytest.mark.parametrize("fmt", ["mxf8", "mxf4"])
@pytest.mark.parametrize("cg", [1, 2])
def test_mx_two_subtiles_and_small_grid(engine, fmt, cg):
    C1 = check_mx(engine, fmt, 2048, 672, 1024, cta_group=cg, m_sub=1, split_tail=1)
    C2 = check_mx(engine, fmt, 2048, 672, 1024, cta_group=cg, m_sub=2, max_ctas=6)
    assert torch.equal(C1, C2)


@pytest.mark.parametrize("fmt", ["mxf8", "mxf4"])
def test_mx_host_path(engine, fmt):
    M, N, K = 2048, 448, 1024
    A, sfa = mx_operand(engine, fmt, M, K, SEED_A)
    B, sfb = mx_operand(engine, fmt, N, K, SEED_B)
    C = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    engine.gemm(A, B, C, FMT[fmt], sfa=sfa, sfb=sfb, split_tail=1)
    engine.check()
    hC = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()
    engine.gemm_host(A.cpu().pin_memory(), B.cpu().pin_memory(), hC, FMT[fmt],
                     sfa=sfa.cpu().pin_memory(), sfb=sfb.cpu().pin_memory())
    assert torch.equal(hC, C.cpu())


@pytest.mark.parametrize("fmt", ["mxf8", "mxf4"])
def test_mx_full_size_sampled(engine, fmt):
    M = N = K = 8192
    A, sfa = mx_operand(engine, fmt, M, K, SEED_A)
    B, sfb = mx_operand(engine, fmt, N, K, SEED_B)
    C = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    engine.gemm(A, B, C, FMT[fmt], sfa=sfa, sfb=sfb)
    engine.check()
    rng = np.random.default_rng(11)
    rows = np.sort(rng.choice(M, 12, replace=False))
    cols = np.sort(rng.choice(N, 12, replace=False))
    da = np.stack([oracle.operand(fmt, 1, K, SEED_A, 1, int(r))[1][0] for r in rows])
    db = np.stack([oracle.operand(fmt, 1, K, SEED_B, 1, int(c))[1][0] for c in cols])
    ref = oracle.gemm(da, db)
    got = bf16_tensor_to_f32(C[torch.as_tensor(rows, device="cuda")][:, torch.as_tensor(cols, device="cuda")])
    ok, worst = oracle.tolerance_check(got, ref, TOL[fmt])
    assert ok, f"{fmt} 8192^3 sampled worst ratio {worst:.3f}"
