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
from gpu_util import ALPHA, FMT, TOL, bf16_tensor_to_f32, device_operand
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
