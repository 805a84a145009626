"""GPU generators, quantisers and the 2:4 compressor must equal the CPU oracle
bit for bit (integer / byte work: the bar is exact equality)."""
import numpy as np
import pytest
import torch

import b2g
import oracle
from gpu_util import to_np_u16, to_np_u8

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dist", [0, 1])
@pytest.mark.parametrize("rows,cols", [(1, 1), (7, 333), (64, 1024)])
def test_fill_matches_oracle(engine, dist, rows, cols):
    x = torch.empty(rows, cols, dtype=torch.float32, device="cuda")
    engine.fill(x, 1234, dist)
    ref = oracle.gen(rows, cols, 1234, dist)
    assert np.array_equal(x.cpu().numpy().view(np.uint32), ref.view(np.uint32))


def _special_values():
    v = [0.0, -0.0, 1e-30, -1e-30, 448.0, 464.0, 465.0, 480.0, 1e6, -1e6, 0.25, 0.75, 1.25,
         1.75, 2.5, 3.5, 5.0, 6.0, 7.0, -5.0, 2 ** -6, 2 ** -9, 2 ** -10, 3 * 2 ** -11,
         2 ** -7 + 2 ** -11]
    return np.array(v * 4, np.float32)[:96]


@pytest.mark.parametrize("fmt", ["bf16", "e4m3"])
def test_quantise_matches_oracle(engine, fmt):
    x = np.concatenate([oracle.gen(1, 4000, 5, 1)[0] * 50, _special_values()]).astype(np.float32)
    x = x[: (x.size // 16) * 16].reshape(16, -1)
    xt = torch.from_numpy(x).cuda()
    if fmt == "bf16":
        q = torch.empty(x.shape, dtype=torch.bfloat16, device="cuda")
        engine.quantize(b2g.FMT_BF16, xt, q)
        assert np.array_equal(to_np_u16(q), oracle.quant_bf16(x)[0])
    else:
        q = torch.empty(x.shape, dtype=torch.uint8, device="cuda")
        engine.quantize(b2g.FMT_E4M3, xt, q)
        assert np.array_equal(to_np_u8(q), oracle.quant_e4m3(x)[0])


def test_quantise_nvfp4_matches_oracle(engine):
    x = oracle.gen(32, 256, 77, 1)
    x[0, :16] = 0.0                    # all-zero block -> scale 0, codes 0
    x[1, :16] = np.linspace(-6, 6, 16)  # exact grid points
    x[2, :16] *= 1e-4                   # tiny block (subnormal e4m3 scale)
    xt = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    q = torch.empty(32, 128, dtype=torch.uint8, device="cuda")
    sf = torch.empty(32, 16, dtype=torch.uint8, device="cuda")
    engine.quantize(b2g.FMT_NVFP4, xt, q, sf)
    rq, rsf, _ = oracle.quant_nvfp4(x)
    assert np.array_equal(to_np_u8(sf), rsf)
    assert np.array_equal(to_np_u8(q), rq)


@pytest.mark.parametrize("fmt,elem", [("mxf8", "e4m3"), ("mxf4", "e2m1")])
def test_quantise_mx_matches_oracle(engine, fmt, elem):
    x = oracle.gen(32, 256, 78, 1)
    x[0, :32] = 0.0                      # all-zero block -> E8M0 0 (2^-127), codes 0
    x[1, :32] *= 1e-30                   # tiny block
    x[2, 32:64] *= 3e4                   # large block: saturation at the top of the range
    x[3, 64:96] = np.float32(2.0) ** -140  # fp32 subnormal block
    xt = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    q = torch.empty(32, 256 if elem == "e4m3" else 128, dtype=torch.uint8, device="cuda")
    sf = torch.empty(32, 8, dtype=torch.uint8, device="cuda")
    engine.quantize(b2g.FMT_MXF8 if fmt == "mxf8" else b2g.FMT_MXF4, xt, q, sf)
    engine.check()
    rq, rsf, _ = oracle.quant_mx(x, elem)
    assert np.array_equal(to_np_u8(sf), rsf)
    assert np.array_equal(to_np_u8(q), rq)


def test_prune_and_compress_match_oracle(engine):
    rows, K = 96, 512
    x = torch.empty(rows, K, dtype=torch.float32, device="cuda")
    engine.fill(x, 3, 0)
    q = torch.empty(rows, K, dtype=torch.bfloat16, device="cuda")
    engine.quantize(b2g.FMT_BF16, x, q)
    engine.prune_24(q, 4)
    ref_q = oracle.prune_24(oracle.quant_bf16(oracle.gen(rows, K, 3, 0))[0], 4)
    assert np.array_equal(to_np_u16(q), ref_q)
    comp = torch.empty(rows, K // 2, dtype=torch.bfloat16, device="cuda")
    meta = torch.empty(rows, K // 32, dtype=torch.int32, device="cuda")
    engine.compress_24(q, comp, meta)
    engine.check()
    rc, rm = oracle.compress_24(ref_q)
    assert np.array_equal(to_np_u16(comp), rc)
    assert np.array_equal(meta.cpu().numpy().view(np.uint32), rm)


def test_compress_pin_0x44444444(engine):
    # kept indices {0,1} in every group -> nibble 0b0100 -> word 0x44444444,
    # the metadata constant of tcgen05_sparse_mma/tcgen05_sparse_mma.cu:331
    d = np.zeros((4, 64), np.uint16)
    d[:, 0::4] = 0x3F80
    d[:, 1::4] = 0xBF80
    dt = torch.from_numpy(d.view(np.int16)).cuda().view(torch.bfloat16)
    comp = torch.empty(4, 32, dtype=torch.bfloat16, device="cuda")
    meta = torch.empty(4, 2, dtype=torch.int32, device="cuda")
    engine.compress_24(dt, comp, meta)
    engine.check()
    assert (meta.cpu().numpy().view(np.uint32) == 0x44444444).all()


def test_compress_rejects_dense_group(engine):
    d = torch.ones(2, 32, dtype=torch.bfloat16, device="cuda")
    comp = torch.empty(2, 16, dtype=torch.bfloat16, device="cuda")
    meta = torch.empty(2, 1, dtype=torch.int32, device="cuda")
    engine.compress_24(d, comp, meta)
    with pytest.raises(b2g.B2GError) as e:
        engine.check()
    assert e.value.status == 1
