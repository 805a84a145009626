"""b2g_gemm_host (the end-to-end entry point on HOST buffers) on the GPU.

The call copies the operands in, runs the GEMM and copies C out, pipelined over
512-row chunks of M on separate copy streams.  C must equal, bit for bit, what
b2g_gemm computes from the same operands already on the device (whole tiles,
same K order), and the oracle within the format's tolerance.
"""
import numpy as np
import pytest
import torch

import b2g
import oracle
from gpu_util import ALPHA, FMT, TOL, bf16_tensor_to_f32, device_operand, host_operand
from test_nvfp4_gpu import SEED_A as NV_A, SEED_B as NV_B, nvfp4_operand
from test_sparse_gpu import sparse_operands

pytestmark = pytest.mark.gpu


def pinned(t):
    return t.cpu().pin_memory()


@pytest.mark.parametrize("fmt", ["bf16", "e4m3"])
@pytest.mark.parametrize("M", [2560, 1100, 300])
def test_host_dense_matches_device_and_oracle(engine, fmt, M):
    N, K = 384, 512
    A, _ = device_operand(engine, fmt, M, K, 11)
    B, _ = device_operand(engine, fmt, N, K, 22)
    C = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    engine.gemm(A, B, C, FMT[fmt], alpha=ALPHA[fmt], split_tail=1)
    engine.check()
    hC = torch.full((M, N), float("nan"), dtype=torch.bfloat16).pin_memory()
    engine.gemm_host(pinned(A), pinned(B), hC, FMT[fmt], alpha=ALPHA[fmt])
    assert torch.equal(hC, C.cpu())
    ref = oracle.gemm(host_operand(fmt, M, K, 11)[1], host_operand(fmt, N, K, 22)[1], ALPHA[fmt])
    ok, worst = oracle.tolerance_check(bf16_tensor_to_f32(hC), ref, TOL[fmt])
    assert ok, f"worst ratio {worst:.3f}"


def test_host_pageable_buffers(engine):
    # pageable host memory: the copies are staged by the driver, results the same
    M, N, K = 1536, 256, 256
    A, _ = device_operand(engine, "bf16", M, K, 11)
    B, _ = device_operand(engine, "bf16", N, K, 22)
    C = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    engine.gemm(A, B, C, b2g.FMT_BF16, split_tail=1)
    hC = torch.empty(M, N, dtype=torch.bfloat16)
    engine.gemm_host(A.cpu(), B.cpu(), hC, b2g.FMT_BF16)
    assert torch.equal(hC, C.cpu())


@pytest.mark.parametrize("layout", [0, 1])
def test_host_sparse(engine, layout):
    M, N, K = 2048, 448, 1024
    A, comp, meta, B = sparse_operands(engine, M, N, K)
    m = meta
    if layout == 1:
        m = torch.empty(engine.sparse_meta_bytes(M, K) // 4, dtype=torch.int32, device="cuda")
        engine.sparse_meta_prepare(meta, M, K, m)
    C = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    engine.gemm(comp, B, C, b2g.FMT_BF16, sparse=1, meta=m, meta_layout=layout, K=K, split_tail=1)
    engine.check()
    hC = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()
    engine.gemm_host(pinned(comp), pinned(B), hC, b2g.FMT_BF16, sparse=1, meta=pinned(m),
                     meta_layout=layout, K=K)
    assert torch.equal(hC, C.cpu())


def test_host_nvfp4(engine):
    M, N, K = 2048, 448, 1024
    A, sfa = nvfp4_operand(engine, M, K, NV_A)
    B, sfb = nvfp4_operand(engine, N, K, NV_B)
    C = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    engine.gemm(A, B, C, b2g.FMT_NVFP4, sfa=sfa, sfb=sfb, split_tail=1)
    engine.check()
    hC = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()
    engine.gemm_host(pinned(A), pinned(B), hC, b2g.FMT_NVFP4, sfa=pinned(sfa), sfb=pinned(sfb))
    assert torch.equal(hC, C.cpu())
    ref = oracle.gemm(oracle.operand("nvfp4", M, K, NV_A, 1)[1], oracle.operand("nvfp4", N, K, NV_B, 1)[1])
    ok, worst = oracle.tolerance_check(bf16_tensor_to_f32(hC), ref, TOL["nvfp4"])
    assert ok, f"worst ratio {worst:.3f}"


def test_host_repeated_calls_reuse_the_pipeline(engine):
    M, N, K = 2048, 256, 256
    outs = []
    for seed in (5, 6, 7):
        A, _ = device_operand(engine, "bf16", M, K, seed)
        B, _ = device_operand(engine, "bf16", N, K, 22)
        C = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        engine.gemm(A, B, C, b2g.FMT_BF16, split_tail=1)
        hC = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()
        engine.gemm_host(pinned(A), pinned(B), hC, b2g.FMT_BF16)
        assert torch.equal(hC, C.cpu())
        outs.append(hC)
    assert not torch.equal(outs[0], outs[1])
