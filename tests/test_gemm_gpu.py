"""GPU parity of the dense tcgen05 GEMM (bf16, fp8 e4m3; cta_group 1 and 2)
against the CPU oracle, through the C ABI.

Small and ragged shapes are checked element by element against the oracle's
FP32 GEMM over the dequantised operands; the BASELINE full sizes (4096^3 bf16,
8192^3 e4m3) are checked on a seeded sample of rows x columns of C that the
oracle recomputes from regenerated operand rows, plus a size-independent
linearity property.
"""
import numpy as np
import pytest
import torch

import oracle
from gpu_util import (ALPHA, CFG1_B_ROW0, CFG1_SEED, FMT, TOL, bf16_tensor_to_f32,
                      device_operand, host_operand, host_rows, to_np_u16, to_np_u8)

pytestmark = pytest.mark.gpu


def run_gemm(engine, fmt, M, N, K, seed_a=11, seed_b=22, b_row0=0, **kw):
    A, _ = device_operand(engine, fmt, M, K, seed_a)
    B, _ = device_operand(engine, fmt, N, K, seed_b, row0=b_row0)
    C = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    engine.gemm(A, B, C, FMT[fmt], alpha=ALPHA[fmt], **kw)
    engine.check()
    return A, B, C


def check_small(engine, fmt, M, N, K, **kw):
    A, B, C = run_gemm(engine, fmt, M, N, K, **kw)
    qa, da = host_operand(fmt, M, K, 11)
    qb, db = host_operand(fmt, N, K, 22)
    # the device-side operands must be the oracle's, bit for bit
    if fmt == "bf16":
        assert np.array_equal(to_np_u16(A), qa) and np.array_equal(to_np_u16(B), qb)
    else:
        assert np.array_equal(to_np_u8(A), qa) and np.array_equal(to_np_u8(B), qb)
    ref = oracle.gemm(da, db, ALPHA[fmt])
    got = bf16_tensor_to_f32(C)
    assert not np.isnan(got).any(), "C has unwritten entries"
    ok, worst = oracle.tolerance_check(got, ref, TOL[fmt])
    assert ok, f"{fmt} {M}x{N}x{K} {kw}: worst error ratio {worst:.3f}"


@pytest.mark.parametrize("fmt", ["bf16", "e4m3"])
@pytest.mark.parametrize("cg", [1, 2])
def test_gemm_square_small(engine, fmt, cg):
    check_small(engine, fmt, 256, 256, 256, cta_group=cg)


@pytest.mark.parametrize("fmt", ["bf16", "e4m3"])
@pytest.mark.parametrize("cg,tile_n", [(1, 64), (1, 128), (1, 256), (2, 128), (2, 256)])
def test_gemm_tiles(engine, fmt, cg, tile_n):
    check_small(engine, fmt, 512, 512, 1024, cta_group=cg, tile_n=tile_n)


@pytest.mark.parametrize("fmt", ["bf16", "e4m3"])
@pytest.mark.parametrize("stages", [2, 3, 5, 7])
def test_gemm_stages(engine, fmt, stages):
    check_small(engine, fmt, 384, 512, 768, cta_group=2, tile_n=256, stages=stages)


@pytest.mark.parametrize("fmt", ["bf16", "e4m3"])
@pytest.mark.parametrize("cg", [1, 2])
@pytest.mark.parametrize("M,N,K", [(300, 200, 528), (257, 196, 64), (129, 8, 16), (1, 1000, 2064)])
def test_gemm_ragged(engine, fmt, cg, M, N, K):
    check_small(engine, fmt, M, N, K, cta_group=cg)


@pytest.mark.parametrize("fmt", ["bf16", "e4m3"])
def test_gemm_persistent_small_grid(engine, fmt):
    # a few CTAs walk many tiles: exercises ring wrap-around and both TMEM buffers
    check_small(engine, fmt, 1024, 768, 512, cta_group=2, max_ctas=4)
    check_small(engine, fmt, 1024, 768, 512, cta_group=1, max_ctas=3)


@pytest.mark.parametrize("fmt,size,cg", [("bf16", 4096, 2), ("bf16", 4096, 1), ("e4m3", 8192, 2),
                                          ("e4m3", 8192, 1), ("bf16", 8192, 2)])
def test_gemm_full_size_sampled(engine, fmt, size, cg):
    M = N = K = size
    # cfg1 (bf16 4096^3) is drawn from seed 0 as BASELINE states; cfg2 keeps 11 / 22.
    # At 8192^3 with cta_group 2 the planner takes 512 x 256 pair tiles (two A sub-tiles
    # per CTA, one accumulator; bf16 through the streaming epilogue)
    sa, sb, b0 = (CFG1_SEED, CFG1_SEED, CFG1_B_ROW0) if fmt == "bf16" else (11, 22, 0)
    A, B, C = run_gemm(engine, fmt, M, N, K, seed_a=sa, seed_b=sb, b_row0=b0, cta_group=cg)
    rng = np.random.default_rng(size + cg)
    rows = np.sort(rng.choice(M, 24, replace=False))
    cols = np.sort(rng.choice(N, 24, replace=False))
    da = host_rows(fmt, rows, K, sa)
    db = host_rows(fmt, cols + b0, K, sb)
    ref = oracle.gemm(da, db, ALPHA[fmt])
    got = bf16_tensor_to_f32(C[torch.as_tensor(rows, device="cuda")][:, torch.as_tensor(cols, device="cuda")])
    ok, worst = oracle.tolerance_check(got, ref, TOL[fmt])
    assert ok, f"sampled {fmt} {size}^3 cg{cg}: worst ratio {worst:.3f}"
    # linearity: C . x == alpha * A . (B^T . x) for a seeded x, on every row
    x = torch.from_numpy(oracle.gen(1, N, 99, 0)[0]).cuda().double()
    lhs = C.double() @ x
    if fmt == "bf16":
        Ad, Bd = A.double(), B.double()
    else:
        Ad = A.view(torch.float8_e4m3fn).double()
        Bd = B.view(torch.float8_e4m3fn).double()
    rhs = ALPHA[fmt] * (Ad @ (Bd.t() @ x))
    rel = ((lhs - rhs).norm() / rhs.norm()).item()
    assert rel < 5e-3, f"linearity residual {rel:.2e}"
    assert not torch.isnan(C).any()


# TS operands: A is copied SMEM -> TMEM (tcgen05.cp) and the MMA reads it there
@pytest.mark.parametrize("fmt", ["bf16", "e4m3"])
@pytest.mark.parametrize("cg,tile_n", [(1, 64), (1, 224), (2, 128), (2, 224)])
def test_gemm_ts_operands(engine, fmt, cg, tile_n):
    check_small(engine, fmt, 512, 448, 1024, cta_group=cg, tile_n=tile_n, ab_mode=1)


@pytest.mark.parametrize("fmt", ["bf16", "e4m3"])
@pytest.mark.parametrize("M,N,K", [(300, 200, 528), (129, 8, 16)])
def test_gemm_ts_ragged(engine, fmt, M, N, K):
    check_small(engine, fmt, M, N, K, cta_group=2, ab_mode=1)
    check_small(engine, fmt, M, N, K, cta_group=1, ab_mode=1, max_ctas=2)


@pytest.mark.parametrize("fmt", ["bf16", "e4m3"])
def test_gemm_ts_matches_ss_bitwise(engine, fmt):
    # same tiles, same K order: TS and SS accumulate identically
    M, N, K = 1024, 896, 2048
    _, _, c_ss = run_gemm(engine, fmt, M, N, K, cta_group=2, tile_n=224)
    _, _, c_ts = run_gemm(engine, fmt, M, N, K, cta_group=2, tile_n=224, ab_mode=1)
    assert torch.equal(c_ss, c_ts)


# Split tail: the last, partial wave's tiles are cut into K ranges on idle
# clusters; split 0 adds the others' fp32 partials.  max_ctas makes the tail.
@pytest.mark.parametrize("fmt", ["bf16", "e4m3"])
@pytest.mark.parametrize("cg,tile_n,max_ctas,split", [(2, 256, 10, 0), (2, 256, 10, 2), (2, 128, 20, 3),
                                                      (1, 128, 7, 0), (1, 256, 5, 4)])
def test_gemm_split_tail(engine, fmt, cg, tile_n, max_ctas, split):
    check_small(engine, fmt, 1024, 1024, 2048, cta_group=cg, tile_n=tile_n, max_ctas=max_ctas,
                split_tail=split)


@pytest.mark.parametrize("fmt", ["bf16", "e4m3"])
def test_gemm_split_tail_repeated_calls(engine, fmt):
    # each launch stamps its flags with a new epoch: a second call with other
    # operands must wait for its own partials, not the first call's
    M = N = 1024
    K = 2048
    A, _ = device_operand(engine, fmt, M, K, 11)
    B1, _ = device_operand(engine, fmt, N, K, 22)
    B2, _ = device_operand(engine, fmt, N, K, 33)
    C1 = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    C2 = torch.empty_like(C1)
    kw = dict(alpha=ALPHA[fmt], cta_group=2, tile_n=256, max_ctas=10)
    for _ in range(3):
        engine.gemm(A, B1, C1, FMT[fmt], **kw)
        engine.gemm(A, B2, C2, FMT[fmt], **kw)
    engine.check()
    da = host_operand(fmt, M, K, 11)[1]
    for C, seed in ((C1, 22), (C2, 33)):
        ref = oracle.gemm(da, host_operand(fmt, N, K, seed)[1], ALPHA[fmt])
        ok, worst = oracle.tolerance_check(bf16_tensor_to_f32(C), ref, TOL[fmt])
        assert ok, f"seed {seed}: worst ratio {worst:.3f}"


def test_gemm_split_tail_off_matches_whole_tiles_bitwise(engine):
    # split_tail=1 keeps whole tiles: identical to a grid with no tail at all
    M = N = 1024
    K = 2048
    _, _, c_off = run_gemm(engine, "bf16", M, N, K, cta_group=2, tile_n=256, max_ctas=10, split_tail=1)
    _, _, c_whole = run_gemm(engine, "bf16", M, N, K, cta_group=2, tile_n=256, max_ctas=16)
    assert torch.equal(c_off, c_whole)


@pytest.mark.parametrize("raster_m", [1, 3, 16])
def test_gemm_raster_groups(engine, raster_m):
    check_small(engine, "e4m3", 1024, 1280, 256, cta_group=2, tile_n=128, raster_m=raster_m)


def test_gemm_rejects_bad_arguments(engine):
    import b2g

    A = torch.zeros(128, 100, dtype=torch.bfloat16, device="cuda")  # K=100: 200 B rows, not 16B
    B = torch.zeros(128, 100, dtype=torch.bfloat16, device="cuda")
    C = torch.zeros(128, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(b2g.B2GError) as e:
        engine.gemm(A, B, C, b2g.FMT_BF16)
    assert e.value.status == 1
    A = torch.zeros(128, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(b2g.B2GError):
        engine.gemm(A, A, C, b2g.FMT_BF16, tile_n=48)
    with pytest.raises(b2g.B2GError):
        engine.gemm(A, A, C, b2g.FMT_BF16, stages=9)
    with pytest.raises(b2g.B2GError) as e:
        engine.gemm(A, A, C, b2g.FMT_BF16, ab_mode=2)
    assert e.value.status == 1
    with pytest.raises(b2g.B2GError) as e:
        engine.gemm(A, A, C, b2g.FMT_BF16, split_tail=5)
    assert e.value.status == 1


@pytest.mark.parametrize("fmt", ["bf16", "e4m3"])
@pytest.mark.parametrize("cg,tile_n", [(2, 256), (2, 224), (2, 192), (1, 256), (1, 128)])
def test_gemm_two_subtiles(engine, fmt, cg, tile_n):
    # dense m_sub = 2: two 128-row A sub-tiles per CTA share each B slot (one
    # accumulator buffer, the 8-warp epilogue); ragged M and N, several waves
    check_small(engine, fmt, 1000, 900, 1024, cta_group=cg, tile_n=tile_n, m_sub=2)
    check_small(engine, fmt, 1024, 768, 512, cta_group=cg, tile_n=tile_n, m_sub=2, max_ctas=4)
