"""Helpers shared by the GPU parity tests: seeded operands built on the device by
libb2g and, independently, on the host by the CPU oracle."""
import numpy as np
import torch

import b2g
import oracle

# Per-format tolerance of C against the oracle (north star): bf16 1e-2, fp8 and
# fp4 5e-2 after dequantisation.  The check is |got - ref| <= tol*(|ref| + rms(ref)).
# tf32 is held to the bf16 bar; e5m2 to the fp8 bar.  int8 (s8) is bit-exact: its
# accumulation is exact and C is a defined rounding of it.
TOL = {"bf16": 1e-2, "e4m3": 5e-2, "nvfp4": 5e-2, "mxf8": 5e-2, "mxf4": 5e-2,
       "tf32": 1e-2, "e5m2": 5e-2, "s8": 0.0, "e2m1": 5e-2, "e2m3": 5e-2, "e3m2": 5e-2,
       "f16": 1e-2, "u8": 0.0}
FMT = {"bf16": b2g.FMT_BF16, "e4m3": b2g.FMT_E4M3, "nvfp4": b2g.FMT_NVFP4,
       "mxf8": b2g.FMT_MXF8, "mxf4": b2g.FMT_MXF4, "tf32": b2g.FMT_TF32,
       "e5m2": b2g.FMT_E5M2, "s8": b2g.FMT_S8, "e2m1": b2g.FMT_E2M1, "e2m3": b2g.FMT_E2M3,
       "e3m2": b2g.FMT_E3M2, "f16": b2g.FMT_F16, "u8": b2g.FMT_U8}
# distributions of the BASELINE configs: bf16 uniform[-1,1], fp8 / fp4 normal(0,1)
DIST = {"bf16": 0, "e4m3": 1, "nvfp4": 1, "mxf8": 1, "mxf4": 1, "tf32": 0, "e5m2": 1, "s8": 1,
        "e2m1": 1, "e2m3": 1, "e3m2": 1, "f16": 0, "u8": 1}
# per-tensor scale 1/64 for A and for B in the fp8 config -> alpha = 1/4096
ALPHA = {"bf16": 1.0, "e4m3": 1.0 / 4096.0, "nvfp4": 1.0, "mxf8": 1.0, "mxf4": 1.0,
         "tf32": 1.0, "e5m2": 1.0, "s8": 1.0 / 1024.0, "e2m1": 1.0, "e2m3": 1.0, "e3m2": 1.0,
         "f16": 1.0, "u8": 1.0 / 65536.0}
# packed bits per element of the sub-byte f8f6f4 formats
SUB_BITS = {"e2m1": 4, "e2m3": 6, "e3m2": 6}


def to_np_u16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def to_np_u8(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.uint8).cpu().numpy()


def bf16_tensor_to_f32(t: torch.Tensor) -> np.ndarray:
    return oracle.bf16_to_f32(to_np_u16(t))


# BASELINE cfg1 draws A and B "from seed 0": A is rows [0, M) and B rows
# [CFG1_B_ROW0, CFG1_B_ROW0 + N) of the seed-0 stream, disjoint slices of one
# generator (the same seed at the same rows would make B a copy of A)
CFG1_SEED = 0
CFG1_B_ROW0 = 1 << 20


def device_operand(engine, fmt: str, rows: int, cols: int, seed: int, row0: int = 0):
    """Stored operand on cuda:0 (bf16 tensor, or uint8 bytes for e4m3 / packed nvfp4):
    rows [row0, row0 + rows) of the seeded generator's stream."""
    x = torch.empty(rows, cols, dtype=torch.float32, device="cuda")
    engine.fill(x, seed, DIST[fmt], row0=row0)
    if fmt == "bf16":
        q = torch.empty(rows, cols, dtype=torch.bfloat16, device="cuda")
        engine.quantize(b2g.FMT_BF16, x, q)
        return q, None
    if fmt in ("e4m3", "e5m2", "s8", "u8"):
        q = torch.empty(rows, cols, dtype=torch.uint8, device="cuda")
        if fmt in ("s8", "u8"):
            x.mul_(oracle.S8_PRESCALE)  # fp32 multiply by a power of two: exact
        if fmt == "u8":
            x.add_(oracle.U8_OFFSET)  # fp32 add, rounded as the oracle's numpy add
        engine.quantize(FMT[fmt], x, q)
        return q, None
    if fmt == "f16":
        q = torch.empty(rows, cols, dtype=torch.float16, device="cuda")
        engine.quantize(b2g.FMT_F16, x, q)
        return q, None
    if fmt == "tf32":
        q = torch.empty(rows, cols, dtype=torch.float32, device="cuda")
        engine.quantize(b2g.FMT_TF32, x, q)
        return q, None
    if fmt in SUB_BITS:
        q = torch.empty(rows, cols * SUB_BITS[fmt] // 8, dtype=torch.uint8, device="cuda")
        engine.quantize(FMT[fmt], x, q)
        return q, None
    if fmt == "nvfp4":
        q = torch.empty(rows, cols // 2, dtype=torch.uint8, device="cuda")
        sf = torch.empty(rows, cols // 16, dtype=torch.uint8, device="cuda")
        engine.quantize(b2g.FMT_NVFP4, x, q, sf)
        return q, sf
    raise ValueError(fmt)


def host_operand(fmt: str, rows: int, cols: int, seed: int, row0: int = 0):
    """(stored, dequantised fp32) rows of the same operand, from the CPU oracle."""
    r = oracle.operand(fmt, rows, cols, seed, DIST[fmt], row0)
    return r[0], r[1]


def host_rows(fmt: str, row_ids, cols: int, seed: int) -> np.ndarray:
    """Dequantised fp32 values of selected rows, from the CPU oracle."""
    out = np.empty((len(row_ids), cols), np.float32)
    for i, r in enumerate(row_ids):
        out[i] = host_operand(fmt, 1, cols, seed, int(r))[1][0]
    return out
