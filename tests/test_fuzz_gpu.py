"""Seeded randomised GEMM parity: shapes, formats and every tile option drawn at
random (cta_group, tile_n, m_sub, split_tail, stages, max_ctas, TS operands), each
case checked against the CPU oracle within its format's tolerance.  The draws
respect the engine's documented limits (TMA 16-byte rows, TMEM room); a draw the
engine rejects must be rejected with B2G_ERR_INVALID / UNSUPPORTED, never run."""
import numpy as np
import pytest
import torch

import b2g
import oracle
from gpu_util import ALPHA, DIST, FMT, TOL, bf16_tensor_to_f32, device_operand, to_np_u16
from test_mx_gpu import mx_operand
from test_nvfp4_gpu import nvfp4_operand
from test_sparse_gpu import SEED_A as SP_A, SEED_B as SP_B, SEED_P, sparse_operands

pytestmark = pytest.mark.gpu

FORMATS = ["bf16", "e4m3", "nvfp4", "mxf8", "mxf4", "sparse"]


def draw(rng):
    fmt = FORMATS[rng.integers(len(FORMATS))]
    kq = {"bf16": 16, "e4m3": 16, "nvfp4": 32, "mxf8": 32, "mxf4": 32, "sparse": 32}[fmt]
    M = int(rng.integers(1, 1300))
    N = int(rng.integers(1, 40)) * 8
    K = int(rng.integers(1, 48)) * kq
    kw = {"cta_group": int(rng.choice([0, 1, 2]))}
    cg = kw["cta_group"] or (2 if M >= 256 else 1)
    wide = [t for t in (64, 96, 128, 160, 192, 224, 256) if t % (16 * cg) == 0 and t % 32 == 0]
    if fmt != "bf16" and fmt != "e4m3":
        wide = [t for t in wide if t <= 224]
    kw["tile_n"] = int(rng.choice([0] + wide))
    if fmt in ("nvfp4", "mxf8", "mxf4", "sparse"):
        kw["m_sub"] = int(rng.choice([0, 1, 2]))
    elif rng.random() < 0.3 and (kw["tile_n"] or 256) <= 224:
        kw["ab_mode"] = 1
    elif rng.random() < 0.3:
        kw["m_sub"] = 2  # dense: two A sub-tiles per CTA (SS), any tile_n up to 256
    kw["split_tail"] = int(rng.choice([0, 1, 2, 3, 4]))
    if rng.random() < 0.4:
        kw["max_ctas"] = int(rng.integers(1, 40)) * cg
    if rng.random() < 0.3:
        kw["stages"] = int(rng.integers(2, 5))
    return fmt, M, N, K, kw


@pytest.mark.parametrize("case", range(48))
def test_fuzz_parity(engine, case):
    rng = np.random.default_rng(1000 + case)
    fmt, M, N, K, kw = draw(rng)
    C = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    if fmt == "sparse":
        A, comp, meta, B = sparse_operands(engine, M, N, K)
        args = (comp, B, C, b2g.FMT_BF16)
        kw.update(sparse=1, meta=meta, K=K)
        da = oracle.operand("bf16", M, K, SP_A, 0, prune_seed=SEED_P)[1]
        db = oracle.operand("bf16", N, K, SP_B, 0)[1]
        tol, alpha = TOL["bf16"], 1.0
    elif fmt in ("nvfp4", "mxf8", "mxf4"):
        mk = (lambda r, s: nvfp4_operand(engine, r, K, s)) if fmt == "nvfp4" else \
             (lambda r, s: mx_operand(engine, fmt, r, K, s))
        (A, sfa), (B, sfb) = mk(M, 71), mk(N, 72)
        args = (A, B, C, FMT[fmt])
        kw.update(sfa=sfa, sfb=sfb)
        da = oracle.operand(fmt, M, K, 71, 1)[1]
        db = oracle.operand(fmt, N, K, 72, 1)[1]
        tol, alpha = TOL[fmt], 1.0
    else:
        A, _ = device_operand(engine, fmt, M, K, 71)
        B, _ = device_operand(engine, fmt, N, K, 72)
        args = (A, B, C, FMT[fmt])
        da = oracle.operand(fmt, M, K, 71, 1 if fmt == "e4m3" else 0)[1]
        db = oracle.operand(fmt, N, K, 72, 1 if fmt == "e4m3" else 0)[1]
        tol, alpha = TOL[fmt], ALPHA[fmt]
        kw["alpha"] = alpha
    try:
        engine.gemm(*args, **kw)
    except b2g.B2GError as e:
        # only the documented limits may refuse a draw (e.g. a ring too deep for SMEM)
        assert e.status in (1, 4), e
        pytest.skip(f"{fmt} {M}x{N}x{K} {kw.get('tile_n')}: refused ({e})")
    engine.check()
    got = bf16_tensor_to_f32(C)
    assert not np.isnan(got).any(), f"{fmt} {M}x{N}x{K} {kw}: unwritten entries"
    ok, worst = oracle.tolerance_check(got, oracle.gemm(da, db, alpha), tol)
    assert ok, f"{fmt} {M}x{N}x{K} {dict((k, v) for k, v in kw.items() if not hasattr(v, 'shape'))}: worst ratio {worst:.3f}"


# ---------------------------------------------------------------- the other kinds
F8 = ["e4m3", "e5m2", "e2m1", "e2m3", "e3m2"]
MX_BITS = {"e4m3": 8, "e5m2": 8, "e2m1": 4, "e2m3": 6, "e3m2": 6}
KINDS = ["s8", "u8", "tf32", "f16", "f8pair", "mxpair"]


def mx_elem_operand(engine, elem, rows, cols, seed):
    x = torch.empty(rows, cols, dtype=torch.float32, device="cuda")
    engine.fill(x, seed, 1)
    q = torch.empty(rows, cols * MX_BITS[elem] // 8, dtype=torch.uint8, device="cuda")
    sf = torch.empty(rows, cols // 32, dtype=torch.uint8, device="cuda")
    engine.quantize_mx(FMT[elem], x, q, sf)
    return q, sf


def draw_kind(rng):
    kind = KINDS[rng.integers(len(KINDS))]
    a = b = None
    if kind in ("f8pair", "mxpair"):
        a, b = F8[rng.integers(5)], F8[rng.integers(5)]
    sub_byte = a in ("e2m1", "e2m3", "e3m2") or b in ("e2m1", "e2m3", "e3m2")
    kq = 128 if sub_byte else (32 if kind == "mxpair" else 16)
    M = int(rng.integers(1, 1300))
    N = int(rng.integers(1, 40)) * 8
    K = int(rng.integers(1, 24)) * kq
    kw = {"cta_group": int(rng.choice([0, 1, 2]))}
    cg = kw["cta_group"] or (2 if M >= 256 else 1)
    wide = [t for t in (64, 96, 128, 160, 192, 224, 256) if t % (16 * cg) == 0 and t % 32 == 0]
    if kind == "mxpair":
        wide = [t for t in wide if t <= 224]
    kw["tile_n"] = int(rng.choice([0] + wide))
    if kind in ("mxpair", "f16", "f8pair") and rng.random() < 0.4 and 0 < kw["tile_n"] <= 224:
        kw["m_sub"] = 2
    kw["split_tail"] = int(rng.choice([0, 1, 2, 3, 4]))
    if rng.random() < 0.4:
        kw["max_ctas"] = int(rng.integers(1, 40)) * cg
    if rng.random() < 0.3:
        kw["stages"] = int(rng.integers(2, 5))
    return kind, a, b, M, N, K, kw


@pytest.mark.parametrize("case", range(48))
def test_fuzz_other_kinds(engine, case):
    rng = np.random.default_rng(5000 + case)
    kind, a, b, M, N, K, kw = draw_kind(rng)
    C = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    exact = False
    if kind == "mxpair":
        (A, sfa), (B, sfb) = mx_elem_operand(engine, a, M, K, 81), mx_elem_operand(engine, b, N, K, 82)
        args = (A, B, C, FMT[a])
        kw.update(sfa=sfa, sfb=sfb, mx_scale=1, b_format=FMT[b])
        da = oracle.operand("mx_" + a, M, K, 81, 1)[1]
        db = oracle.operand("mx_" + b, N, K, 82, 1)[1]
        tol, alpha = 5e-2, 1.0
    else:
        fa, fb = (a, b) if kind == "f8pair" else (kind, kind)
        A, _ = device_operand(engine, fa, M, K, 81)
        B, _ = device_operand(engine, fb, N, K, 82)
        args = (A, B, C, FMT[fa])
        if fb != fa:
            kw["b_format"] = FMT[fb]
        qa, da = oracle.operand(fa, M, K, 81, DIST[fa])[:2]
        qb, db = oracle.operand(fb, N, K, 82, DIST[fb])[:2]
        tol, alpha = TOL[fa], ALPHA[fa]
        exact = fa in ("s8", "u8")
        kw["alpha"] = alpha
    try:
        engine.gemm(*args, **kw)
    except b2g.B2GError as e:
        assert e.status in (1, 4), e
        pytest.skip(f"{kind} {a}/{b} {M}x{N}x{K}: refused ({e})")
    engine.check()
    desc = f"{kind} {a}/{b} {M}x{N}x{K} " + str({k: v for k, v in kw.items() if not hasattr(v, 'shape')})
    if exact:
        assert np.array_equal(to_np_u16(C), oracle.gemm_s8_exact(qa, qb, alpha)), desc
        return
    got = bf16_tensor_to_f32(C)
    assert not np.isnan(got).any(), f"{desc}: unwritten entries"
    ok, worst = oracle.tolerance_check(got, oracle.gemm(da, db, alpha), tol)
    assert ok, f"{desc}: worst ratio {worst:.3f}"


# ---------------------------------------------------------------- structured-sparse A
# every sparse form of the GEMM: 2:4 on bf16 / fp16 / the 8-bit and fp4 / fp6 types,
# MX e4m3 / e5m2 (one scale per 64 K), MXFP4 in pairs, tf32 1:2; the .ws.sp form,
# prepared metadata and the tile options drawn at random
SPARSE_KINDS = ["bf16", "e4m3", "e5m2", "s8", "u8", "tf32", "e2m1", "e2m3", "e3m2", "mx_e4m3",
                "mx_e5m2", "mxf4"]


def draw_sparse(rng):
    kind = SPARSE_KINDS[rng.integers(len(SPARSE_KINDS))]
    kq = {"e2m1": 256, "e2m3": 256, "e3m2": 256, "mx_e4m3": 64, "mx_e5m2": 64, "mxf4": 64}.get(kind, 32)
    M = int(rng.integers(1, 1100))
    N = int(rng.integers(1, 40)) * 8
    K = int(rng.integers(1, 12)) * kq
    kw = {}
    layout = int(rng.random() < 0.3) if kind != "bf16" else 0
    if kind not in ("mx_e4m3", "mx_e5m2", "mxf4") and rng.random() < 0.2:
        kw.update(instruction=1, tile_n=int(rng.choice([64, 128])))  # .ws.sp, cta_group::1
    else:
        kw["cta_group"] = int(rng.choice([0, 1, 2]))
        cg = kw["cta_group"] or (2 if M >= 256 else 1)
        wide = [t for t in (64, 96, 128, 160, 192, 224) if t % (16 * cg) == 0 and t % 32 == 0]
        kw["tile_n"] = int(rng.choice([0] + wide))
        if rng.random() < 0.4 and 0 < kw["tile_n"] <= (192 if kind.startswith("mx") else 224):
            kw["m_sub"] = 2
        if rng.random() < 0.4:
            kw["max_ctas"] = int(rng.integers(1, 40)) * cg
    kw["split_tail"] = int(rng.choice([0, 1, 2, 3, 4]))
    if rng.random() < 0.3:
        kw["stages"] = int(rng.integers(2, 5))
    return kind, M, N, K, layout, kw


@pytest.mark.parametrize("case", range(40))
def test_fuzz_sparse_kinds(engine, case):
    from test_sparse8_gpu import check_sparse8
    from test_sparse_gpu import check_sparse
    from test_sparse_mx_gpu import check_sparse_mx
    from test_sparse_mxf4_gpu import check_sparse_mxf4
    from test_sparse_sub_gpu import check_sparse_sub
    from test_sparse_tf32_gpu import check_tf32_sparse

    rng = np.random.default_rng(7000 + case)
    kind, M, N, K, layout, kw = draw_sparse(rng)
    try:
        if kind == "bf16":
            check_sparse(engine, M, N, K, **kw)
        elif kind in ("e4m3", "e5m2", "s8", "u8"):
            check_sparse8(engine, kind, M, N, K, layout=layout, **kw)
        elif kind == "tf32":
            check_tf32_sparse(engine, M, N, K, layout=layout, **kw)
        elif kind in ("e2m1", "e2m3", "e3m2"):
            check_sparse_sub(engine, kind, M, N, K, layout=layout, **kw)
        elif kind == "mxf4":
            check_sparse_mxf4(engine, M, N, K, layout=layout, **kw)
        else:
            check_sparse_mx(engine, kind[3:], M, N, K, layout=layout, **kw)
    except b2g.B2GError as e:
        # only the documented limits may refuse a draw (a ring too deep for SMEM,
        # tile_n and sub-tiles beyond TMEM)
        assert e.status in (1, 4), e
        pytest.skip(f"sparse {kind} {M}x{N}x{K} {kw}: refused ({e})")
