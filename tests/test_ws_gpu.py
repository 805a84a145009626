"""GPU parity of the GEMM on the weight-stationary MMA form, tcgen05.mma.ws and
tcgen05.mma.ws.sp (b2g_gemm_desc.instruction = 1).

The reference issues `.ws` and `.ws.sp` only in its single-tile rate probe
(tcgen05_sparse_mma/tcgen05_sparse_mma.cu:80-81,343-483, INSTRUCTION=ws), for the
kinds without block scaling and cta_group::1 only; it never reads D back.  Here
the same forms drive whole GEMMs (128-row tiles, N 64 / 128 / 256) on every
dense kind (tf32, f16 with bf16 and fp16, f8f6f4 element types, i8) and on the
structured-sparse kinds, and C must match the CPU oracle within each format's
tolerance (bit-exact for the integer kinds), like the ordinary form's tests.
"""
import pytest

from test_formats_gpu import check as check_dense
from test_sparse8_gpu import check_sparse8
from test_sparse_gpu import check_sparse
from test_sparse_tf32_gpu import check_tf32_sparse

pytestmark = pytest.mark.gpu
WS = dict(instruction=1)


@pytest.mark.parametrize("fmt", ["bf16", "f16", "tf32", "e4m3", "e5m2", "s8", "u8", "e2m1",
                                 "e3m2"])
@pytest.mark.parametrize("tile_n", [64, 128, 256])
def test_ws_dense_tiles(engine, fmt, tile_n):
    check_dense(engine, fmt, 512, 512, 1024, tile_n=tile_n, **WS)


@pytest.mark.parametrize("fmt", ["bf16", "tf32", "e4m3", "s8"])
@pytest.mark.parametrize("M,N,K", [(300, 200, 528), (129, 8, 16), (1, 1000, 2064)])
def test_ws_dense_ragged(engine, fmt, M, N, K):
    check_dense(engine, fmt, M, N, K, **WS)


def test_ws_dense_small_grid_stages_and_split_tail(engine):
    # a persistent grid of 3 CTAs, a 2-deep ring, and a split last wave
    check_dense(engine, "bf16", 640, 512, 2048, tile_n=128, max_ctas=3, stages=2, **WS)
    check_dense(engine, "e4m3", 384, 256, 4096, tile_n=256, split_tail=4, **WS)


@pytest.mark.parametrize("tile_n", [64, 128])
def test_ws_sparse_bf16(engine, tile_n):
    check_sparse(engine, 512, 448, 1024, tile_n=tile_n, **WS)


@pytest.mark.parametrize("M,N,K", [(300, 200, 544), (129, 40, 32)])
def test_ws_sparse_bf16_ragged(engine, M, N, K):
    check_sparse(engine, M, N, K, **WS)


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2", "s8", "u8"])
@pytest.mark.parametrize("tile_n", [64, 128])
def test_ws_sparse8(engine, fmt, tile_n):
    check_sparse8(engine, fmt, 512, 448, 1024, tile_n=tile_n, **WS)


def test_ws_sparse8_prepared_metadata(engine):
    check_sparse8(engine, "e4m3", 640, 448, 1536, layout=1, **WS)


@pytest.mark.parametrize("tile_n", [64, 128])
def test_ws_sparse_tf32(engine, tile_n):
    check_tf32_sparse(engine, 512, 448, 1024, tile_n=tile_n, **WS)

