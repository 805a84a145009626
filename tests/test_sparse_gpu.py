"""GPU parity of the 2:4 structured-sparse bf16 GEMM (tcgen05.mma.sp, kind::f16).

The sparse operand is built on the device (seeded bf16 A, seeded 2:4 pruning,
b2g_compress_24) and independently by the CPU oracle; the compressed values and
metadata must agree bit for bit, and C must match the oracle's FP32 GEMM over
the pruned dense A within the bf16 tolerance.  The engine's TMEM-ready metadata
layout (b2g_sparse_meta_prepare) is checked word for word against a restatement
of its definition below.
"""
import numpy as np
import pytest
import torch

import b2g
import oracle
from gpu_util import TOL, bf16_tensor_to_f32, to_np_u16

pytestmark = pytest.mark.gpu
SEED_A, SEED_B, SEED_P = 31, 32, 33


def sparse_operands(engine, M, N, K):
    x = torch.empty(M, K, dtype=torch.float32, device="cuda")
    engine.fill(x, SEED_A, 0)
    A = torch.empty(M, K, dtype=torch.bfloat16, device="cuda")
    engine.quantize(b2g.FMT_BF16, x, A)
    engine.prune_24(A, SEED_P)
    comp = torch.empty(M, K // 2, dtype=torch.bfloat16, device="cuda")
    meta = torch.empty(M, K // 32, dtype=torch.int32, device="cuda")
    engine.compress_24(A, comp, meta)
    y = torch.empty(N, K, dtype=torch.float32, device="cuda")
    engine.fill(y, SEED_B, 0)
    B = torch.empty(N, K, dtype=torch.bfloat16, device="cuda")
    engine.quantize(b2g.FMT_BF16, y, B)
    engine.check()
    return A, comp, meta, B


def host_sparse_rows(rows, K, seed=SEED_A):
    """Dequantised pruned rows of A from the oracle (fp32)."""
    out = np.empty((len(rows), K), np.float32)
    for i, r in enumerate(rows):
        q, _ = oracle.operand("bf16", 1, K, seed, 0, int(r), prune_seed=SEED_P)
        out[i] = oracle.bf16_to_f32(q)[0]
    return out


def check_sparse(engine, M, N, K, **kw):
    A, comp, meta, B = sparse_operands(engine, M, N, K)
    q, da = oracle.operand("bf16", M, K, SEED_A, 0, prune_seed=SEED_P)
    rc, rm = oracle.compress_24(q)
    assert np.array_equal(to_np_u16(A), q)
    assert np.array_equal(to_np_u16(comp), rc)
    assert np.array_equal(meta.cpu().numpy().view(np.uint32), rm)
    db = oracle.operand("bf16", N, K, SEED_B, 0)[1]
    C = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    engine.gemm(comp, B, C, b2g.FMT_BF16, sparse=1, meta=meta, K=K, **kw)
    engine.check()
    ref = oracle.gemm(da, db)
    got = bf16_tensor_to_f32(C)
    assert not np.isnan(got).any()
    ok, worst = oracle.tolerance_check(got, ref, TOL["bf16"])
    assert ok, f"sparse {M}x{N}x{K} {kw}: worst ratio {worst:.3f}"
    return A, comp, meta, B, C


def ready_layout(meta_canon: np.ndarray, M: int, K: int) -> np.ndarray:
    """Restatement of the engine's TMEM-ready metadata layout (datagen.cu)."""
    kw = K // 32
    rb_n, kb_n = (M + 127) // 128, (K + 127) // 128
    out = np.empty((rb_n, kb_n, 128, 4), np.uint32)
    pad = np.uint32(0x44444444)
    for rb in range(rb_n):
        for kb in range(kb_n):
            for L in range(128):
                m2, k1, m0 = L >> 4, (L >> 3) & 1, L & 7
                r_lo = rb * 128 + m2 * 16 + m0
                r_hi = r_lo + 8
                for c in range(4):
                    ch = kb * 4 + c
                    wl = meta_canon[r_lo, ch] if (r_lo < M and ch < kw) else pad
                    wh = meta_canon[r_hi, ch] if (r_hi < M and ch < kw) else pad
                    lo = (int(wl) >> (16 * k1)) & 0xFFFF
                    hi = (int(wh) >> (16 * k1)) & 0xFFFF
                    out[rb, kb, L, c] = lo | (hi << 16)
    return out


def test_meta_ready_layout_matches_definition(engine):
    M, K = 200, 352  # ragged: padding rows and K blocks
    rng = np.random.default_rng(5)
    canon = rng.integers(0, 2 ** 32, size=(M, K // 32), dtype=np.uint64).astype(np.uint32)
    dev = torch.from_numpy(canon.view(np.int32)).cuda()
    ready = torch.empty(engine.sparse_meta_bytes(M, K) // 4, dtype=torch.int32, device="cuda")
    engine.sparse_meta_prepare(dev, M, K, ready)
    engine.check()
    got = ready.cpu().numpy().view(np.uint32).reshape(-1)
    assert np.array_equal(got, ready_layout(canon, M, K).reshape(-1))


@pytest.mark.parametrize("cg", [1, 2])
def test_sparse_small(engine, cg):
    check_sparse(engine, 256, 256, 256, cta_group=cg)


@pytest.mark.parametrize("cg,tile_n", [(1, 64), (1, 128), (1, 224), (2, 128), (2, 224)])
def test_sparse_tiles(engine, cg, tile_n):
    check_sparse(engine, 512, 448, 1024, cta_group=cg, tile_n=tile_n)


@pytest.mark.parametrize("cg", [1, 2])
@pytest.mark.parametrize("M,N,K", [(300, 200, 544), (129, 40, 32), (640, 1000, 2080)])
def test_sparse_ragged(engine, cg, M, N, K):
    check_sparse(engine, M, N, K, cta_group=cg)


# two 128-row A sub-tiles per CTA sharing one B tile (one TMEM accumulator buffer)
@pytest.mark.parametrize("cg,tile_n", [(1, 64), (1, 224), (2, 128), (2, 224)])
def test_sparse_two_subtiles(engine, cg, tile_n):
    check_sparse(engine, 1024, 448, 1024, cta_group=cg, tile_n=tile_n, m_sub=2)


@pytest.mark.parametrize("cg", [1, 2])
@pytest.mark.parametrize("M,N,K", [(300, 200, 544), (129, 40, 32), (640, 1000, 2080)])
def test_sparse_two_subtiles_ragged(engine, cg, M, N, K):
    check_sparse(engine, M, N, K, cta_group=cg, m_sub=2)


def test_sparse_two_subtiles_small_grid_matches_one(engine):
    # few clusters walk many tiles through the single accumulator buffer; the
    # per-element K order is the same as with one sub-tile, so C is bit-identical
    M, N, K = 2048, 672, 1024
    A, comp, meta, B, C1 = check_sparse(engine, M, N, K, cta_group=2, m_sub=1, split_tail=1)
    C2 = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    engine.gemm(comp, B, C2, b2g.FMT_BF16, sparse=1, meta=meta, K=K, cta_group=2, m_sub=2,
                max_ctas=6)
    engine.check()
    assert torch.equal(C1, C2)


def test_sparse_prepared_meta_and_small_grid(engine):
    M, N, K = 1024, 672, 512
    A, comp, meta, B, C = check_sparse(engine, M, N, K, cta_group=2, max_ctas=4)
    ready = torch.empty(engine.sparse_meta_bytes(M, K) // 4, dtype=torch.int32, device="cuda")
    engine.sparse_meta_prepare(meta, M, K, ready)
    C2 = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    engine.gemm(comp, B, C2, b2g.FMT_BF16, sparse=1, meta=ready, meta_layout=1, K=K, split_tail=1)
    engine.check()
    assert torch.equal(C, C2)


def test_sparse_equals_dense_on_pruned_operand(engine):
    # the sparse path and the dense path over the pruned A compute the same C
    M, N, K = 512, 512, 2048
    A, comp, meta, B, C = check_sparse(engine, M, N, K)
    Cd = torch.empty_like(C)
    engine.gemm(A, B, Cd, b2g.FMT_BF16)
    engine.check()
    d = (C.float() - Cd.float()).abs().max().item()
    scale = Cd.float().abs().max().item()
    assert d <= 1e-2 * scale


def test_sparse_full_size_cfg3_sampled(engine):
    # BASELINE cfg3: M = N = 8192, K = 16384
    M, N, K = 8192, 8192, 16384
    A, comp, meta, B = sparse_operands(engine, M, N, K)
    C = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    engine.gemm(comp, B, C, b2g.FMT_BF16, sparse=1, meta=meta, K=K)
    engine.check()
    rng = np.random.default_rng(3)
    rows = np.sort(rng.choice(M, 16, replace=False))
    cols = np.sort(rng.choice(N, 16, replace=False))
    da = host_sparse_rows(rows, K)
    db = np.stack([oracle.operand("bf16", 1, K, SEED_B, 0, int(c))[1][0] for c in cols])
    ref = oracle.gemm(da, db)
    got = bf16_tensor_to_f32(C[torch.as_tensor(rows, device="cuda")][:, torch.as_tensor(cols, device="cuda")])
    ok, worst = oracle.tolerance_check(got, ref, TOL["bf16"])
    assert ok, f"cfg3 sampled worst ratio {worst:.3f}"
    x = torch.from_numpy(oracle.gen(1, N, 99, 0)[0]).cuda().double()
    lhs = C.double() @ x
    rhs = A.double() @ (B.double().t() @ x)
    assert ((lhs - rhs).norm() / rhs.norm()).item() < 5e-3


def test_sparse_rejects_bad_m_sub(engine):
    M, N, K = 256, 256, 256
    A, comp, meta, B = sparse_operands(engine, M, N, K)
    C = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(b2g.B2GError) as e:
        engine.gemm(comp, B, C, b2g.FMT_BF16, sparse=1, meta=meta, K=K, m_sub=3)
    assert e.value.status == 1
    with pytest.raises(b2g.B2GError) as e:
        engine.gemm(A, B, C, b2g.FMT_BF16, m_sub=2, ab_mode=1)  # dense two sub-tiles: SS only
    assert e.value.status == 4
    with pytest.raises(b2g.B2GError) as e:  # 2 x 256 accumulator columns leave no TMEM
        engine.gemm(comp, B, C, b2g.FMT_BF16, sparse=1, meta=meta, K=K, m_sub=2, tile_n=256)
    assert e.value.status == 1


@pytest.mark.parametrize("cg,m_sub", [(1, 1), (2, 1), (2, 2)])
def test_sparse_fp16(engine, cg, m_sub):
    # kind::f16 .sp with fp16 operands (type code 0): same prune / compress (16-bit
    # patterns), the oracle decodes the codes as IEEE binary16
    M, N, K = 640, 448, 1024
    x = torch.empty(M, K, dtype=torch.float32, device="cuda")
    engine.fill(x, SEED_A, 0)
    A = torch.empty(M, K, dtype=torch.float16, device="cuda")
    engine.quantize(b2g.FMT_F16, x, A)
    engine.prune_24(A, SEED_P)
    comp = torch.empty(M, K // 2, dtype=torch.float16, device="cuda")
    meta = torch.empty(M, K // 32, dtype=torch.int32, device="cuda")
    engine.compress_24(A, comp, meta)
    y = torch.empty(N, K, dtype=torch.float32, device="cuda")
    engine.fill(y, SEED_B, 0)
    B = torch.empty(N, K, dtype=torch.float16, device="cuda")
    engine.quantize(b2g.FMT_F16, y, B)
    C = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    engine.gemm(comp, B, C, b2g.FMT_F16, sparse=1, meta=meta, K=K, cta_group=cg, m_sub=m_sub)
    engine.check()
    qa, da = oracle.operand("f16", M, K, SEED_A, 0, prune_seed=SEED_P)
    assert np.array_equal(A.cpu().numpy().view(np.uint16), qa)
    rc, rm = oracle.compress_24(qa)
    assert np.array_equal(comp.cpu().numpy().view(np.uint16), rc)
    assert np.array_equal(meta.cpu().numpy().view(np.uint32), rm)
    db = oracle.operand("f16", N, K, SEED_B, 0)[1]
    got = bf16_tensor_to_f32(C)
    ok, worst = oracle.tolerance_check(got, oracle.gemm(da, db), TOL["bf16"])
    assert ok, f"sparse fp16 cg{cg} m_sub {m_sub}: worst ratio {worst:.3f}"
