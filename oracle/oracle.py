"""TEST INFRASTRUCTURE ONLY: numpy/ctypes front end of the CPU oracle (liboracle.so).

Used by tests/ as the parity checker and by bench.py's cpu_baseline leg and
``--impl reference`` arm as the timed CPU GEMM.  The product (libb2g, the b2g
package) never imports this module.

The oracle restates, from the mathematics and the public format specifications,
what the reference's hot path would compute if it read its accumulators back:
C = alpha * A . B with A row-major [M][K] and B column-major (stored [N][K]),
cutlass_gemm_mainloop/cutlass_gemm_bench.cu:78-80.  See b2g_oracle.c for the
parity status of each function.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")


def build():
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        L.orc_hash.restype = C.c_uint64
        L.orc_hash.argtypes = [C.c_uint64, C.c_uint64]
        L.orc_uniform.restype = C.c_float
        L.orc_uniform.argtypes = [C.c_uint64, C.c_uint64]
        L.orc_normal.restype = C.c_float
        L.orc_normal.argtypes = [C.c_uint64, C.c_uint64]
        L.orc_fill.argtypes = [_f32p, C.c_int64, C.c_int64, C.c_int64, C.c_uint64, C.c_int]
        L.orc_f32_to_bf16.restype = C.c_uint16
        L.orc_f32_to_bf16.argtypes = [C.c_float]
        L.orc_bf16_to_f32.restype = C.c_float
        L.orc_bf16_to_f32.argtypes = [C.c_uint16]
        L.orc_f32_to_e4m3.restype = C.c_uint8
        L.orc_f32_to_e4m3.argtypes = [C.c_float]
        L.orc_e4m3_to_f32.restype = C.c_float
        L.orc_e4m3_to_f32.argtypes = [C.c_uint8]
        L.orc_f32_to_e2m1.restype = C.c_uint8
        L.orc_f32_to_e2m1.argtypes = [C.c_float]
        L.orc_e2m1_to_f32.restype = C.c_float
        L.orc_e2m1_to_f32.argtypes = [C.c_uint8]
        L.orc_f32_to_e5m2.restype = C.c_uint8
        L.orc_f32_to_e5m2.argtypes = [C.c_float]
        L.orc_e5m2_to_f32.restype = C.c_float
        L.orc_e5m2_to_f32.argtypes = [C.c_uint8]
        L.orc_f32_to_s8.restype = C.c_int8
        L.orc_f32_to_s8.argtypes = [C.c_float]
        L.orc_f32_to_tf32.restype = C.c_float
        L.orc_f32_to_tf32.argtypes = [C.c_float]
        L.orc_quant_elem.argtypes = [_f32p, C.c_int64, C.c_int, C.c_void_p, _f32p]
        L.orc_f32_to_u8.restype = C.c_uint8
        L.orc_f32_to_u8.argtypes = [C.c_float]
        L.orc_f32_to_f16.restype = C.c_uint16
        L.orc_f32_to_f16.argtypes = [C.c_float]
        L.orc_f16_to_f32.restype = C.c_float
        L.orc_f16_to_f32.argtypes = [C.c_uint16]
        for n in ("e2m3", "e3m2"):
            getattr(L, f"orc_f32_to_{n}").restype = C.c_uint8
            getattr(L, f"orc_f32_to_{n}").argtypes = [C.c_float]
            getattr(L, f"orc_{n}_to_f32").restype = C.c_float
            getattr(L, f"orc_{n}_to_f32").argtypes = [C.c_uint8]
        L.orc_quant_sub.argtypes = [_f32p, C.c_int64, C.c_int, _u8p, _f32p]
        L.orc_quant_bf16.argtypes = [_f32p, C.c_int64, _u16p, _f32p]
        L.orc_quant_e4m3.argtypes = [_f32p, C.c_int64, _u8p, _f32p]
        L.orc_quant_nvfp4.argtypes = [_f32p, C.c_int64, C.c_int64, _u8p, _u8p, _f32p]
        L.orc_quant_nvfp4_block.argtypes = [_f32p, C.c_int64, C.c_int64, C.c_int, _u8p, _u8p,
                                            _f32p]
        L.orc_quant_mx.argtypes = [_f32p, C.c_int64, C.c_int64, C.c_int, _u8p, _u8p, _f32p]
        L.orc_quant_mx_block.argtypes = [_f32p, C.c_int64, C.c_int64, C.c_int, C.c_int, _u8p, _u8p,
                                         _f32p]
        L.orc_prune_24.argtypes = [_u16p, C.c_int64, C.c_int64, C.c_int64, C.c_uint64]
        L.orc_compress_24.restype = C.c_int
        L.orc_compress_24.argtypes = [_u16p, C.c_int64, C.c_int64, _u16p, _u32p]
        L.orc_decompress_24.argtypes = [_u16p, _u32p, C.c_int64, C.c_int64, _u16p]
        L.orc_prune_24_u8.argtypes = [_u8p, C.c_int64, C.c_int64, C.c_int64, C.c_uint64]
        L.orc_compress_24_u8.restype = C.c_int
        L.orc_compress_24_u8.argtypes = [_u8p, C.c_int64, C.c_int64, C.c_uint8, _u8p, _u32p]
        L.orc_decompress_24_u8.argtypes = [_u8p, _u32p, C.c_int64, C.c_int64, _u8p]
        L.orc_prune_24_sub.argtypes = [_u8p, C.c_int64, C.c_int64, C.c_int64, C.c_uint64, C.c_int]
        L.orc_compress_24_sub.restype = C.c_int
        L.orc_compress_24_sub.argtypes = [_u8p, C.c_int64, C.c_int64, C.c_int, C.c_uint8, _u8p,
                                          _u32p]
        L.orc_prune_12_f32.argtypes = [_u32p, C.c_int64, C.c_int64, C.c_int64, C.c_uint64]
        L.orc_compress_12_f32.restype = C.c_int
        L.orc_compress_12_f32.argtypes = [_u32p, C.c_int64, C.c_int64, _u32p, _u32p]
        L.orc_decompress_12_f32.argtypes = [_u32p, _u32p, C.c_int64, C.c_int64, _u32p]
        L.orc_gemm_f32.argtypes = [_f32p, _f32p, _f32p, C.c_int64, C.c_int64, C.c_int64,
                                   C.c_int64, C.c_int64, C.c_int64, C.c_float, C.c_int]
        _lib = L
    return _lib


# ------------------------------------------------------------------ generator
def gen(rows: int, cols: int, seed: int, dist: int = 0, row0: int = 0) -> np.ndarray:
    """Rows [row0, row0+rows) of the seeded fp32 matrix of width `cols`."""
    out = np.empty((rows, cols), np.float32)
    lib().orc_fill(out, row0, rows, cols, seed, dist)
    return out


def gen_rows(row_ids, cols: int, seed: int, dist: int = 0) -> np.ndarray:
    out = np.empty((len(row_ids), cols), np.float32)
    for i, r in enumerate(row_ids):
        lib().orc_fill(out[i:i + 1], int(r), 1, cols, seed, dist)
    return out


# ------------------------------------------------------------------ codecs
def quant_bf16(x: np.ndarray):
    x = np.ascontiguousarray(x, np.float32)
    q = np.empty(x.shape, np.uint16)
    d = np.empty(x.shape, np.float32)
    lib().orc_quant_bf16(x, x.size, q, d)
    return q, d


def quant_e4m3(x: np.ndarray):
    x = np.ascontiguousarray(x, np.float32)
    q = np.empty(x.shape, np.uint8)
    d = np.empty(x.shape, np.float32)
    lib().orc_quant_e4m3(x, x.size, q, d)
    return q, d


_ELEM = {"s8": (0, np.int8), "tf32": (1, np.float32), "e5m2": (2, np.uint8), "u8": (3, np.uint8),
         "f16": (4, np.uint16)}
# fp32 scale applied before int8 conversion, so that normal(0,1) data uses the range;
# uint8 also shifts by U8_OFFSET (fp32 multiply, then fp32 add)
S8_PRESCALE = 32.0
U8_OFFSET = 128.0


def quant_elem(x: np.ndarray, fmt: str):
    """Element-wise conversion without scale factors: 's8' / 'u8' (nearest even,
    saturating), 'tf32' (10 mantissa bits, nearest even, fp32 storage), 'e5m2' or
    'f16' (IEEE binary16, nearest even).
    Returns (stored, values the MMA reads as fp32)."""
    x = np.ascontiguousarray(x, np.float32)
    code, dt = _ELEM[fmt]
    q = np.empty(x.shape, dt)
    d = np.empty(x.shape, np.float32)
    lib().orc_quant_elem(x, x.size, code, q.ctypes.data, d)
    return q, d


_SUB = {"e2m1": (0, 4), "e2m3": (1, 6), "e3m2": (2, 6)}


def quant_sub(x: np.ndarray, fmt: str):
    """fp4 / fp6 of kind::f8f6f4 without scale factors ('e2m1', 'e2m3', 'e3m2'),
    packed along each row in groups of 16 (8 or 12 bytes, little-endian).
    Returns (packed rows, values the MMA reads as fp32)."""
    x = np.ascontiguousarray(x, np.float32)
    rows, cols = x.shape
    assert cols % 16 == 0
    code, bits = _SUB[fmt]
    q = np.zeros((rows, cols * bits // 8), np.uint8)
    d = np.empty_like(x)
    lib().orc_quant_sub(x, x.size, code, q, d)
    return q, d


def unpack_sub(q: np.ndarray, bits: int) -> np.ndarray:
    """Codes of packed fp4 / fp6 rows (element i at bits [bits*i, bits*(i+1)) of each
    row's little-endian bit stream), one uint8 each."""
    q = np.ascontiguousarray(q, np.uint8)
    rows = q.shape[0]
    bitv = np.unpackbits(q, axis=1, bitorder="little").reshape(rows, -1, bits)
    return (bitv.astype(np.uint8) << np.arange(bits, dtype=np.uint8)).sum(axis=2).astype(np.uint8)


def gemm_s8_exact(A: np.ndarray, B: np.ndarray, alpha: float) -> np.ndarray:
    """int8 / uint8 GEMM as the engine's kind::i8 path defines C: exact s32 accumulation,
    fp32(acc) rounded to nearest even, times alpha in fp32, then bf16 (nearest
    even).  Returns the bf16 bit patterns."""
    acc = A.astype(np.int64) @ B.astype(np.int64).T
    assert np.abs(acc).max(initial=0) < 2**31
    f = acc.astype(np.float32) * np.float32(alpha)
    q, _ = quant_bf16(f)
    return q


def quant_mx(x: np.ndarray, elem: str, block: int = 32):
    """OCP MX quantisation, one E8M0 scale per `block` (32; 64 for the 2:4-sparse MX
    GEMM) elements: elem 'e4m3' (MXFP8), 'e2m1' (MXFP4, packed), 'e5m2', 'e2m3' or
    'e3m2' (fp6 packed 16 per 12 bytes).
    Returns (stored, sf E8M0 bytes, dequantised fp32)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = x.shape
    assert cols % block == 0
    e, bits = {"e4m3": (0, 8), "e2m1": (1, 4), "e5m2": (2, 8), "e2m3": (3, 6), "e3m2": (4, 6)}[elem]
    q = np.zeros((rows, cols * bits // 8), np.uint8)
    sf = np.empty((rows, cols // block), np.uint8)
    d = np.empty_like(x)
    lib().orc_quant_mx_block(x, rows, cols, e, block, q, sf, d)
    return q, sf, d


def quant_nvfp4(x: np.ndarray, block: int = 16):
    """NVFP4: packed e2m1, one ue4m3 scale e4m3(amax/6) per `block` (16; 32 for the
    4:8-sparse NVFP4 GEMM) elements.  Returns (packed, sf, dequantised fp32)."""
    x = np.ascontiguousarray(x, np.float32)
    rows, cols = x.shape
    q = np.zeros((rows, cols // 2), np.uint8)
    sf = np.empty((rows, cols // block), np.uint8)
    d = np.empty(x.shape, np.float32)
    lib().orc_quant_nvfp4_block(x, rows, cols, block, q, sf, d)
    return q, sf, d


def bf16_to_f32(q: np.ndarray) -> np.ndarray:
    return (q.astype(np.uint32) << 16).view(np.float32)


_F16_TABLE = None


def f16_to_f32(q: np.ndarray) -> np.ndarray:
    """IEEE binary16 codes -> fp32 through the oracle's own decoder (a 65536-entry table)."""
    global _F16_TABLE
    if _F16_TABLE is None:
        _F16_TABLE = np.array([lib().orc_f16_to_f32(i) for i in range(65536)], np.float32)
    return _F16_TABLE[np.asarray(q, np.uint16)]


def e4m3_to_f32(q: np.ndarray) -> np.ndarray:
    table = np.array([lib().orc_e4m3_to_f32(i) for i in range(256)], np.float32)
    return table[q]


def e2m1_to_f32(code: np.ndarray) -> np.ndarray:
    table = np.array([lib().orc_e2m1_to_f32(i) for i in range(16)], np.float32)
    return table[code & 0xF]


# ------------------------------------------------------------------ 2:4
# Element width by stored dtype: 16-bit (bf16 / fp16 codes) or 8-bit (e4m3, e5m2,
# s8, u8 codes).  The non-zero test of the 8-bit compressor: the fp8 formats
# ignore the sign bit (0x80 is -0), the integers do not.
NZ_MASK_8 = {"e4m3": 0x7F, "e5m2": 0x7F, "s8": 0xFF, "u8": 0xFF}
# byte-wise zero tests of the 2:4 compressor: the 8-bit formats, and "mxf4": a byte of
# packed e2m1 (a pair, the 4:8 sparsity of kind::mxf4 / mxf4nvf4), zero when both of
# its elements are, either sign
NZ_MASK_BYTES = {**NZ_MASK_8, "mxf4": 0x77}


def prune_24(q: np.ndarray, seed: int, row0: int = 0, bits: int | None = None) -> np.ndarray:
    """Zero 2 of every 4 consecutive elements of each row (16- or 8-bit codes, or
    packed fp4 / fp6 codes of `bits` bits in uint8 rows), or for 32-bit words (tf32)
    1 of every 2 (structured 1:2)."""
    if bits in (4, 6):
        out = np.ascontiguousarray(q, np.uint8).copy()
        lib().orc_prune_24_sub(out, row0, out.shape[0], out.shape[1] * 8 // bits, seed, bits)
        return out
    if q.dtype.itemsize == 4:
        out = np.ascontiguousarray(q).view(np.uint32).copy()
        lib().orc_prune_12_f32(out, row0, out.shape[0], out.shape[1], seed)
        return out.view(q.dtype)
    if q.dtype.itemsize == 2:
        out = np.ascontiguousarray(q, np.uint16).copy()
        lib().orc_prune_24(out, row0, out.shape[0], out.shape[1], seed)
        return out.view(q.dtype)
    out = np.ascontiguousarray(q).view(np.uint8).copy()
    lib().orc_prune_24_u8(out, row0, out.shape[0], out.shape[1], seed)
    return out.view(q.dtype)


def compress_24(dense: np.ndarray, fmt: str = "bf16"):
    """(compressed [rows][K/2], metadata [rows][K/32] uint32) of a 2:4-sparse matrix of
    16-bit codes (fmt 'bf16' / 'f16') or 8-bit codes (fmt in NZ_MASK_8)."""
    rows, K = dense.shape
    if fmt in _SUB:  # packed fp4 / fp6 codes: K counts elements
        bits = _SUB[fmt][1]
        K = K * 8 // bits
        comp = np.zeros((rows, K // 2 * bits // 8), np.uint8)
        meta = np.empty((rows, K // 32), np.uint32)
        if lib().orc_compress_24_sub(np.ascontiguousarray(dense, np.uint8), rows, K, bits,
                                     0x7 if bits == 4 else 0x1F, comp, meta) != 0:
            raise ValueError("a group of 4 holds more than 2 non-zeros")
        return comp, meta
    if dense.dtype.itemsize == 4:  # tf32, 1:2: metadata [rows][K/16]
        meta = np.empty((rows, K // 16), np.uint32)
        comp = np.empty((rows, K // 2), np.uint32)
        if lib().orc_compress_12_f32(np.ascontiguousarray(dense).view(np.uint32), rows, K, comp,
                                     meta) != 0:
            raise ValueError("a pair holds two non-zeros")
        return comp.view(dense.dtype), meta
    meta = np.empty((rows, K // 32), np.uint32)
    if dense.dtype.itemsize == 2:
        d = np.ascontiguousarray(dense).view(np.uint16)
        comp = np.empty((rows, K // 2), np.uint16)
        rc = lib().orc_compress_24(d, rows, K, comp, meta)
    else:
        d = np.ascontiguousarray(dense).view(np.uint8)
        comp = np.empty((rows, K // 2), np.uint8)
        rc = lib().orc_compress_24_u8(d, rows, K, NZ_MASK_BYTES[fmt], comp, meta)
    if rc != 0:
        raise ValueError("a group of 4 holds more than 2 non-zeros")
    return comp.view(dense.dtype), meta


def decompress_24(comp: np.ndarray, meta: np.ndarray, K: int) -> np.ndarray:
    rows = comp.shape[0]
    if comp.dtype.itemsize == 4:
        out = np.empty((rows, K), np.uint32)
        lib().orc_decompress_12_f32(np.ascontiguousarray(comp).view(np.uint32),
                                    np.ascontiguousarray(meta), rows, K, out)
        return out.view(comp.dtype)
    if comp.dtype.itemsize == 2:
        out = np.empty((rows, K), np.uint16)
        lib().orc_decompress_24(np.ascontiguousarray(comp).view(np.uint16),
                                np.ascontiguousarray(meta), rows, K, out)
    else:
        out = np.empty((rows, K), np.uint8)
        lib().orc_decompress_24_u8(np.ascontiguousarray(comp).view(np.uint8),
                                   np.ascontiguousarray(meta), rows, K, out)
    return out.view(comp.dtype)


# ------------------------------------------------------------------ GEMM
def gemm(A: np.ndarray, B: np.ndarray, alpha: float = 1.0, threads: int | None = None):
    """fp32 C[M][N] = alpha * A[M][K] . B[N][K]^T (B stored as its transpose)."""
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    M, K = A.shape
    N = B.shape[0]
    Cm = np.empty((M, N), np.float32)
    if threads is None:
        threads = os.cpu_count() or 1
    lib().orc_gemm_f32(A, B, Cm, M, N, K, K, K, N, alpha, int(threads))
    return Cm


# ------------------------------------------------------------------ operands of the configs
def operand(fmt: str, rows: int, cols: int, seed: int, dist: int, row0: int = 0,
            prune_seed: int | None = None):
    """Stored operand rows + their dequantised fp32 values, as the engine sees them.

    fmt: 'bf16' | 'f16' | 'e4m3' | 'e5m2' | 's8' | 'u8' | 'tf32' | 'e2m1' | 'e2m3' | 'e3m2'
    | 'nvfp4' | 'mxf8' | 'mxf4' | 'mx_<elem>' (elem e4m3, e5m2, e2m1, e2m3, e3m2)
    | 'mx64_<elem>' (one MX scale per 64 elements).
    Returns (stored, dequant[, sf]).  's8' converts S8_PRESCALE * x, 'u8'
    S8_PRESCALE * x + U8_OFFSET.
    """
    x = gen(rows, cols, seed, dist, row0)
    if fmt == "f16" and prune_seed is not None:
        q, _ = quant_elem(x, "f16")
        q = prune_24(q, prune_seed, row0)
        return q, f16_to_f32(q)
    if fmt == "bf16":
        q, d = quant_bf16(x)
        if prune_seed is not None:
            q = prune_24(q, prune_seed, row0)
            d = bf16_to_f32(q)
        return q, d
    if fmt in NZ_MASK_8:  # the 8-bit formats; 2:4-pruned on the stored codes on request
        if fmt == "e4m3":
            q, d = quant_e4m3(x)
        elif fmt == "s8":
            q, d = quant_elem(x * np.float32(S8_PRESCALE), "s8")
        elif fmt == "u8":
            q, d = quant_elem(x * np.float32(S8_PRESCALE) + np.float32(U8_OFFSET), "u8")
        else:
            q, d = quant_elem(x, fmt)
        if prune_seed is not None:
            qp = prune_24(q, prune_seed, row0)
            d = np.where(qp != q, np.float32(0), d)  # a pruned element reads as 0
            q = qp
        return q, d
    if fmt == "tf32":
        q, d = quant_elem(x, fmt)
        if prune_seed is not None:  # structured 1:2 on the fp32 words
            qp = prune_24(q, prune_seed, row0)
            d = np.where(qp != q, np.float32(0), d)
            q = qp
        return q, d
    if fmt == "f16":
        return quant_elem(x, fmt)
    if fmt in _SUB:
        q, d = quant_sub(x, fmt)
        if prune_seed is not None:  # 2:4 on the packed codes, element by element
            bits = _SUB[fmt][1]
            qp = prune_24(q, prune_seed, row0, bits)
            d = np.where(unpack_sub(qp, bits) != unpack_sub(q, bits), np.float32(0), d)
            q = qp
        return q, d
    if fmt in ("nvfp4", "nvfp4_32"):
        # 'nvfp4_32': one scale per 32 elements, the 4:8-sparse NVFP4 GEMM's block;
        # prune_seed: 4:8 in pairs, 2 of every 4 bytes (pairs of e2m1) zeroed
        q, sf, d = quant_nvfp4(x, 32 if fmt == "nvfp4_32" else 16)
        if prune_seed is not None:
            qp = prune_24(q, prune_seed, row0)
            d = np.where(unpack_sub(qp, 4) != unpack_sub(q, 4), np.float32(0), d)
            q = qp
        return q, d, sf
    if fmt in ("mxf8", "mxf4") or fmt.startswith("mx_") or fmt.startswith("mx64_"):
        # OCP MX: 'mxf8' (e4m3), 'mxf4' (packed e2m1), 'mx_<elem>' on kind::mxf8f6f4;
        # 'mx64_<elem>': one scale per 64 elements (the 2:4-sparse MX GEMM's block)
        block = 64 if fmt.startswith("mx64_") else 32
        elem = {"mxf8": "e4m3", "mxf4": "e2m1"}.get(fmt) or fmt.split("_", 1)[1]
        q, sf, d = quant_mx(x, elem, block)
        if prune_seed is not None:
            # 2:4 pruning of the stored 8-bit codes (the scales stay as quantised), the
            # same positions as the plain 8-bit formats; for packed e2m1, 4:8 in pairs:
            # the same on the bytes, each a pair of elements
            if elem in ("e4m3", "e5m2"):
                qp = prune_24(q, prune_seed, row0)
                d = np.where(qp != q, np.float32(0), d)
            elif elem == "e2m1":
                qp = prune_24(q, prune_seed, row0)
                d = np.where(unpack_sub(qp, 4) != unpack_sub(q, 4), np.float32(0), d)
            else:
                raise ValueError(f"structured pruning of MX {elem} is not built")
            q = qp
        return q, d, sf
    raise ValueError(fmt)


def tolerance_check(got: np.ndarray, ref: np.ndarray, tol: float):
    """Per-element relative check used by every parity test.  Two bounds hold:

        |got - ref| <= tol * (|ref| + rms(ref))      on every entry, and
        |got - ref| <= tol * |ref|                   on every entry with |ref| > rms(ref)

    The first is a relative tolerance `tol` with an absolute floor of tol * rms(ref),
    so that entries of C near zero (cancellation) are judged against the typical
    magnitude of C rather than against themselves; the second is the plain
    per-element relative tolerance on the entries that are not near zero.
    Returns (ok, worst ratio): the larger of the two error / bound maxima.
    """
    got = got.astype(np.float64)
    ref = ref.astype(np.float64)
    rms = float(np.sqrt(np.mean(ref * ref))) if ref.size else 0.0
    err = np.abs(got - ref)
    ratio = err / (tol * (np.abs(ref) + rms) + 1e-30)
    worst = float(ratio.max()) if ratio.size else 0.0
    big = np.abs(ref) > rms
    if big.any():
        worst = max(worst, float((err[big] / (tol * np.abs(ref[big]))).max()))
    return worst <= 1.0, worst


def relative_error(got: np.ndarray, ref: np.ndarray) -> float:
    """Worst plain relative error |got - ref| / |ref| over the entries with
    |ref| > rms(ref) (the second bound of tolerance_check, without tol)."""
    got = got.astype(np.float64)
    ref = ref.astype(np.float64)
    rms = float(np.sqrt(np.mean(ref * ref))) if ref.size else 0.0
    big = np.abs(ref) > rms
    return float((np.abs(got - ref)[big] / np.abs(ref[big])).max()) if big.any() else 0.0
