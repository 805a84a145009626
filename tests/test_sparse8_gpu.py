"""GPU parity of 2:4 structured-sparse A on the 8-bit kinds: tcgen05.mma.sp with
kind::f8f6f4 (e4m3, e5m2) and kind::i8 (s8, u8).

The reference issues these sparse forms only in its single-tile rate probe, with
the constant metadata word 0x44444444
(tcgen05_sparse_mma/tcgen05_sparse_mma.cu:88-111,327-332,343-483).  Here the
sparse operand is built on the device (seeded codes, seeded 2:4 pruning of the
stored bytes, b2g_compress_24_format) and independently by the CPU oracle: the
pruned codes, the compressed values and the metadata must agree bit for bit.
C must match the oracle's FP32 GEMM over the pruned dense A within the fp8
tolerance (5e-2), and for the integer kinds equal the exact int8 GEMM bit for
bit.  The engine's TMEM-ready layout of 8-bit metadata is checked word for word
against a restatement of its definition.
"""
import numpy as np
import pytest
import torch

import b2g
import oracle
from gpu_util import ALPHA, FMT, TOL, bf16_tensor_to_f32, device_operand, host_rows, to_np_u16

pytestmark = pytest.mark.gpu
SEED_A, SEED_B, SEED_P = 51, 52, 53
FLOAT8 = ("e4m3", "e5m2")
INT8 = ("s8", "u8")


def sparse8_operands(engine, fmt, M, N, K):
    A, _ = device_operand(engine, fmt, M, K, SEED_A)  # stored codes, one byte each
    engine.prune_24(A, SEED_P, fmt=FMT[fmt])
    comp = torch.empty(M, K // 2, dtype=torch.uint8, device="cuda")
    meta = torch.empty(M, K // 32, dtype=torch.int32, device="cuda")
    engine.compress_24(A, comp, meta, fmt=FMT[fmt])
    B, _ = device_operand(engine, fmt, N, K, SEED_B)
    engine.check()
    return A, comp, meta, B


def u8(t):
    return t.contiguous().view(torch.uint8).cpu().numpy()


def check_sparse8(engine, fmt, M, N, K, layout=0, **kw):
    A, comp, meta, B = sparse8_operands(engine, fmt, M, N, K)
    qa, da = oracle.operand(fmt, M, K, SEED_A, 1, prune_seed=SEED_P)
    rc, rm = oracle.compress_24(qa, fmt)
    assert np.array_equal(u8(A), qa.view(np.uint8)), "pruned A differs from the oracle's"
    assert np.array_equal(u8(comp), rc.view(np.uint8)), "compressed A differs"
    assert np.array_equal(meta.cpu().numpy().view(np.uint32), rm), "metadata differs"
    qb, db = oracle.operand(fmt, N, K, SEED_B, 1)
    mkw = dict(meta=meta)
    if layout == 1:
        ready = torch.empty(engine.sparse_meta_bytes(M, K, fmt=FMT[fmt]) // 4, dtype=torch.int32,
                            device="cuda")
        engine.sparse_meta_prepare(meta, M, K, ready, fmt=FMT[fmt])
        mkw = dict(meta=ready, meta_layout=1)
    C = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    engine.gemm(comp, B, C, FMT[fmt], sparse=1, K=K, alpha=ALPHA[fmt], **mkw, **kw)
    engine.check()
    if fmt in INT8:
        want = oracle.gemm_s8_exact(qa, qb, ALPHA[fmt])
        assert np.array_equal(to_np_u16(C), want), f"sparse {fmt} {M}x{N}x{K} {kw}: not bit-exact"
    else:
        got = bf16_tensor_to_f32(C)
        assert not np.isnan(got).any()
        ok, worst = oracle.tolerance_check(got, oracle.gemm(da, db, ALPHA[fmt]), TOL[fmt])
        assert ok, f"sparse {fmt} {M}x{N}x{K} {kw}: worst ratio {worst:.3f}"
    return A, comp, meta, B, C


@pytest.mark.parametrize("fmt", FLOAT8 + INT8)
@pytest.mark.parametrize("cg", [1, 2])
def test_sparse8_small(engine, fmt, cg):
    check_sparse8(engine, fmt, 256, 256, 512, cta_group=cg)


@pytest.mark.parametrize("fmt", ["e4m3", "s8"])
@pytest.mark.parametrize("cg,tile_n", [(1, 64), (1, 128), (1, 224), (2, 128), (2, 224)])
def test_sparse8_tiles(engine, fmt, cg, tile_n):
    check_sparse8(engine, fmt, 512, 448, 1024, cta_group=cg, tile_n=tile_n)


@pytest.mark.parametrize("fmt", ["e4m3", "s8"])
@pytest.mark.parametrize("cg", [1, 2])
@pytest.mark.parametrize("M,N,K", [(300, 200, 544), (129, 40, 32), (640, 1000, 2080)])
def test_sparse8_ragged(engine, fmt, cg, M, N, K):
    check_sparse8(engine, fmt, M, N, K, cta_group=cg)


# two 128-row A sub-tiles per CTA sharing one B tile (one accumulator buffer; the
# 8-warp epilogue, which converts the s32 accumulator of kind::i8 itself)
@pytest.mark.parametrize("fmt", ["e4m3", "s8", "u8"])
@pytest.mark.parametrize("cg,tile_n", [(1, 64), (1, 224), (2, 128), (2, 224)])
def test_sparse8_two_subtiles(engine, fmt, cg, tile_n):
    check_sparse8(engine, fmt, 1024, 448, 1024, cta_group=cg, tile_n=tile_n, m_sub=2)


@pytest.mark.parametrize("fmt", ["e4m3", "s8"])
def test_sparse8_persistent_small_grid_and_stages(engine, fmt):
    check_sparse8(engine, fmt, 1024, 672, 2048, cta_group=2, max_ctas=4, stages=2)
    # (a 224-column cta_group::1 tile takes 76 KB per 8-bit sparse slot: 3 do not fit)
    check_sparse8(engine, fmt, 768, 448, 1536, cta_group=1, tile_n=128, max_ctas=3, stages=3)


@pytest.mark.parametrize("fmt", ["e4m3", "u8"])
def test_sparse8_prepared_metadata(engine, fmt):
    check_sparse8(engine, fmt, 640, 448, 1536, layout=1, cta_group=2)


def ready_layout8(canon: np.ndarray, M: int, K: int) -> np.ndarray:
    """Restatement of the engine's TMEM-ready layout of 8-bit metadata (datagen.cu):
    per [128-row block][256-K slot], two halves of [128 lanes][4 words]; lane L of
    half h holds canonical words 8 kb + 4 h .. + 3 of row 128 rb + L."""
    kw = K // 32
    rb_n, kb_n = (M + 127) // 128, (K + 255) // 256
    out = np.full((rb_n, kb_n, 2, 128, 4), 0x44444444, np.uint32)
    for rb in range(rb_n):
        for kb in range(kb_n):
            for h in range(2):
                for c in range(4):
                    ch = kb * 8 + 4 * h + c
                    if ch >= kw:
                        continue
                    rows = np.arange(rb * 128, min(M, rb * 128 + 128))
                    out[rb, kb, h, :len(rows), c] = canon[rows, ch]
    return out


def test_meta_ready_layout8_matches_definition(engine):
    M, K = 200, 608  # ragged: padding rows, a partial K slot
    rng = np.random.default_rng(7)
    canon = rng.integers(0, 2 ** 32, size=(M, K // 32), dtype=np.uint64).astype(np.uint32)
    dev = torch.from_numpy(canon.view(np.int32)).cuda()
    nbytes = engine.sparse_meta_bytes(M, K, fmt=b2g.FMT_E4M3)
    assert nbytes == 2 * 3 * 4096
    ready = torch.empty(nbytes // 4, dtype=torch.int32, device="cuda")
    engine.sparse_meta_prepare(dev, M, K, ready, fmt=b2g.FMT_E4M3)
    engine.check()
    got = ready.cpu().numpy().view(np.uint32).reshape(-1)
    assert np.array_equal(got, ready_layout8(canon, M, K).reshape(-1))


@pytest.mark.parametrize("fmt", FLOAT8 + INT8)
def test_compress8_pin_0x44444444(engine, fmt):
    # every group keeps elements 0 and 1: the reference's constant metadata word
    # (tcgen05_sparse_mma.cu:331), whatever the 8-bit format
    M, K = 64, 256
    dense = torch.zeros(M, K, dtype=torch.uint8, device="cuda")
    dense.view(M, K // 4, 4)[:, :, 0] = 0x38  # 1.0 in e4m3; a non-zero code in every format
    dense.view(M, K // 4, 4)[:, :, 1] = 0x41
    comp = torch.empty(M, K // 2, dtype=torch.uint8, device="cuda")
    meta = torch.empty(M, K // 32, dtype=torch.int32, device="cuda")
    engine.compress_24(dense, comp, meta, fmt=FMT[fmt])
    engine.check()
    assert (meta.cpu().numpy().view(np.uint32) == 0x44444444).all()
    c = comp.cpu().numpy().reshape(M, K // 4, 2)
    assert (c[:, :, 0] == 0x38).all() and (c[:, :, 1] == 0x41).all()


def test_compress8_fp8_negative_zero_is_zero(engine):
    # e4m3 0x80 is -0: it may share a group with two non-zeros; for s8 it is -128
    M, K = 8, 64
    dense = torch.zeros(M, K, dtype=torch.uint8, device="cuda")
    g = dense.view(M, K // 4, 4)
    g[:, :, 1] = 0x38
    g[:, :, 2] = 0x80
    g[:, :, 3] = 0x41
    comp = torch.empty(M, K // 2, dtype=torch.uint8, device="cuda")
    meta = torch.empty(M, K // 32, dtype=torch.int32, device="cuda")
    engine.compress_24(dense, comp, meta, fmt=b2g.FMT_E4M3)
    engine.check()  # no more than 2 non-zeros per group
    assert (meta.cpu().numpy().view(np.uint32) == 0xDDDDDDDD).all()  # idx 1 | 3 << 2
    engine.compress_24(dense, comp, meta, fmt=b2g.FMT_S8)
    with pytest.raises(b2g.B2GError) as e:  # 0x80 is -128 for s8: three non-zeros
        engine.check()
    assert e.value.status == 1


def test_sparse8_cfg3_shape_e4m3_sampled(engine):
    # the cfg3 shape (8192 x 8192 x 16384) on kind::f8f6f4: a seeded sample of C
    # against the oracle, plus the linearity property over every row
    M = N = 8192
    K = 16384
    fmt = "e4m3"
    A, comp, meta, B = sparse8_operands(engine, fmt, M, N, K)
    C = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    engine.gemm(comp, B, C, FMT[fmt], sparse=1, meta=meta, K=K, alpha=ALPHA[fmt])
    engine.check()
    rng = np.random.default_rng(8)
    rows = np.sort(rng.choice(M, 24, replace=False))
    cols = np.sort(rng.choice(N, 24, replace=False))
    da = np.stack([oracle.operand(fmt, 1, K, SEED_A, 1, int(r), prune_seed=SEED_P)[1][0] for r in rows])
    db = host_rows(fmt, cols, K, SEED_B)
    got = bf16_tensor_to_f32(C[torch.as_tensor(rows, device="cuda")][:, torch.as_tensor(cols, device="cuda")])
    ok, worst = oracle.tolerance_check(got, oracle.gemm(da, db, ALPHA[fmt]), TOL[fmt])
    assert ok, f"sampled sparse e4m3 8192x8192x16384: worst ratio {worst:.3f}"
    x = torch.from_numpy(oracle.gen(1, N, 99, 0)[0]).cuda().double()
    Ad = A.view(torch.float8_e4m3fn).double()
    rhs = ALPHA[fmt] * (Ad @ (B.view(torch.float8_e4m3fn).double().t() @ x))
    rel = ((C.double() @ x - rhs).norm() / rhs.norm()).item()
    assert rel < 5e-3, f"linearity residual {rel:.2e}"


def test_sparse8_host_pipeline_matches_device(engine):
    # b2g_gemm_host on pinned host buffers (prepared metadata: the engine layout's
    # row blocks of 256-K slots are cut per row chunk) gives the device call's C
    fmt = "e4m3"
    M, N, K = 1536, 1024, 1024
    A, comp, meta, B = sparse8_operands(engine, fmt, M, N, K)
    ready = torch.empty(engine.sparse_meta_bytes(M, K, fmt=FMT[fmt]) // 4, dtype=torch.int32,
                        device="cuda")
    engine.sparse_meta_prepare(meta, M, K, ready, fmt=FMT[fmt])
    C = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    kw = dict(sparse=1, K=K, alpha=ALPHA[fmt], meta_layout=1, cta_group=2, split_tail=1)
    engine.gemm(comp, B, C, FMT[fmt], meta=ready, **kw)
    engine.check()
    hC = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()
    engine.gemm_host(comp.cpu().pin_memory(), B.cpu().pin_memory(), hC, FMT[fmt],
                     meta=ready.cpu().pin_memory(), **kw)
    assert torch.equal(hC, C.cpu())
