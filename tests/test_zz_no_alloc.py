"""b2g_gemm_sparse_noalloc: the 2:4 sparse GEMM for callers that cannot allocate.

Callers such as plugins inside a framework that owns all device memory, or
latency-critical loops where cudaMalloc / cudaFree may synchronise the device,
cannot create a b2g handle (handles own device memory) or let b2g_gemm grow its
scratch.  This entry point takes no handle and allocates nothing; its scratch
is a static device array of the library.  The test calls it through the C ABI,
twice in a row, and compares each result with the existing entry point
(b2g_gemm, sparse, canonical metadata) and with the CPU oracle's FP32 GEMM,
within the bf16 tolerance of the other parity tests.  It is collected last so
that a run that stops at the first failure has already run every other test; it
also passes alone in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import b2g
import oracle
from b2g import _lib
from gpu_util import TOL, bf16_tensor_to_f32

pytestmark = pytest.mark.gpu


def _sparse_inputs(engine, M, N, K):
    x = torch.empty(M, K, dtype=torch.float32, device="cuda")
    engine.fill(x, 41, 0)
    A = torch.empty(M, K, dtype=torch.bfloat16, device="cuda")
    engine.quantize(b2g.FMT_BF16, x, A)
    engine.prune_24(A, 43)
    comp = torch.empty(M, K // 2, dtype=torch.bfloat16, device="cuda")
    meta = torch.empty(M, K // 32, dtype=torch.int32, device="cuda")
    engine.compress_24(A, comp, meta)
    y = torch.empty(N, K, dtype=torch.float32, device="cuda")
    engine.fill(y, 42, 0)
    B = torch.empty(N, K, dtype=torch.bfloat16, device="cuda")
    engine.quantize(b2g.FMT_BF16, y, B)
    engine.check()
    return comp, meta, B


def _noalloc(comp, meta, B, Cout, K):
    lib = _lib.load()
    d = b2g.Engine._desc(comp, B, Cout, b2g.FMT_BF16, K=K, sparse=1, meta=meta)
    msg = C.c_char_p()
    st = lib.b2g_gemm_sparse_noalloc(C.byref(d), int(torch.cuda.current_stream().cuda_stream),
                                     C.byref(msg))
    return st, (msg.value.decode() if msg.value else "")


# the CUDA driver hands out device memory in 2 MiB granules, so a cudaMalloc
# that the call kept would lower the device's free memory by at least this much
ALLOC_GRANULE = 2 << 20


@pytest.mark.parametrize("M,N,K", [(512, 448, 1024), (300, 200, 544)])
def test_noalloc_matches_b2g_gemm_twice(engine, M, N, K):
    comp, meta, B = _sparse_inputs(engine, M, N, K)
    ref = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    engine.gemm(comp, B, ref, b2g.FMT_BF16, sparse=1, meta=meta, K=K)
    engine.check()
    ref_np = bf16_tensor_to_f32(ref)
    # the same operands from the CPU oracle's generator, prune and FP32 GEMM
    host = oracle.gemm(oracle.operand("bf16", M, K, 41, 0, prune_seed=43)[1],
                       oracle.operand("bf16", N, K, 42, 0)[1])
    torch_allocated = torch.cuda.memory_allocated()
    for call in range(2):
        out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        st, msg = _noalloc(comp, meta, B, out, K)
        free_after = torch.cuda.mem_get_info()[0]
        assert st == 0, f"call {call}: status {st}: {msg}"
        got = bf16_tensor_to_f32(out)
        assert not np.isnan(got).any()
        ok, worst = oracle.tolerance_check(got, ref_np, TOL["bf16"])
        assert ok, f"call {call}: worst ratio {worst:.3f} against b2g_gemm"
        ok, worst = oracle.tolerance_check(got, host, TOL["bf16"])
        assert ok, f"call {call}: worst ratio {worst:.3f} against the CPU oracle"
        # After the first call, which loads the library module that holds the static
        # array (16 MiB of device memory, kept until exit), a call keeps no device
        # memory (a tolerance below one allocation granule, since the counter is
        # device-wide)
        if call == 1:
            assert free_after > free_before - ALLOC_GRANULE, (free_before, free_after)
        del out
    assert torch.cuda.memory_allocated() == torch_allocated


def test_noalloc_rejects_oversize_problem():
    # 8192 x 32768 needs 32 MiB of metadata scratch, above the 16 MiB array;
    # rejected before any pointer is touched
    lib = _lib.load()
    d = _lib.GemmDesc()
    d.format, d.sparse, d.meta_layout = b2g.FMT_BF16, 1, 0
    d.M, d.N, d.K = 8192, 256, 32768
    d.lda, d.ldb, d.ldc = 16384, 32768, 256
    d.A = d.B = d.C = d.meta = 256
    msg = C.c_char_p()
    st = lib.b2g_gemm_sparse_noalloc(C.byref(d), 0, C.byref(msg))
    assert st == 1
    assert b"16 MiB" in msg.value


def test_noalloc_limit_counts_whole_128_blocks():
    # M * K = 133971936 is below 2^27, but the engine layout rounds both to
    # 128: ceil(8193 / 128) * ceil(16352 / 128) = 65 * 128 = 8320 blocks of 2 KiB,
    # above the 8192 that fit; rejected before any pointer is touched
    lib = _lib.load()
    d = _lib.GemmDesc()
    d.format, d.sparse, d.meta_layout = b2g.FMT_BF16, 1, 0
    d.M, d.N, d.K = 8193, 256, 16352
    d.lda, d.ldb, d.ldc = 8176, 16352, 256
    d.A = d.B = d.C = d.meta = 256
    msg = C.c_char_p()
    st = lib.b2g_gemm_sparse_noalloc(C.byref(d), 0, C.byref(msg))
    assert st == 1
    assert b"ceil(M/128) * ceil(K/128)" in msg.value
