"""ctypes binding of libb2g.so (the C ABI in include/b2g.h).

The library is built in-tree (``make -C microbench-blackwell_b200``) and loaded
from ``microbench-blackwell_b200/lib/libb2g.so``.  There is no fallback: if the
library is missing, importing the engine raises.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(_HERE), "lib", "libb2g.so")

B2G_OK = 0
B2G_ERR_TIMEOUT = 3
STATUS = {
    0: "ok",
    1: "invalid argument",
    2: "CUDA error",
    3: "kernel wait timed out",
    4: "unsupported",
    5: "no sm_100 device",
    6: "device self-check mismatch",
}

# b2g_format
FMT_BF16 = 0
FMT_E4M3 = 1
FMT_S8 = 2
FMT_E2M1 = 3
FMT_MXF8 = 4
FMT_MXF4 = 5
FMT_NVFP4 = 6
FMT_TF32 = 7
FMT_E5M2 = 8
FMT_E2M3 = 9
FMT_E3M2 = 10
FMT_F16 = 11
FMT_U8 = 12


class GemmDesc(C.Structure):
    _fields_ = [
        ("format", C.c_int32),
        ("sparse", C.c_int32),
        ("M", C.c_int64),
        ("N", C.c_int64),
        ("K", C.c_int64),
        ("lda", C.c_int64),
        ("ldb", C.c_int64),
        ("ldc", C.c_int64),
        ("A", C.c_void_p),
        ("B", C.c_void_p),
        ("C", C.c_void_p),
        ("sfa", C.c_void_p),
        ("sfb", C.c_void_p),
        ("meta", C.c_void_p),
        ("alpha", C.c_float),
        ("cta_group", C.c_int32),
        ("ab_mode", C.c_int32),
        ("tile_n", C.c_int32),
        ("stages", C.c_int32),
        ("max_ctas", C.c_int32),
        ("meta_layout", C.c_int32),
        ("raster_m", C.c_int32),
        ("m_sub", C.c_int32),
        ("split_tail", C.c_int32),
        ("b_format", C.c_int32),
        ("mx_scale", C.c_int32),
        ("instruction", C.c_int32),
    ]


class GemmPlan(C.Structure):
    _fields_ = [(name, C.c_int32) for name in (
        "variant", "kind", "cta_group", "tile_m", "tile_n", "m_sub", "stages", "smem_bytes",
        "tmem_columns", "num_m_tiles", "num_n_tiles", "k_blocks", "raster_m", "tail_start",
        "tail_split", "units", "clusters", "threads", "k_atoms", "instruction")] + [
            ("reserved", C.c_int32 * 2)]


class ProbeDesc(C.Structure):
    _fields_ = [
        (name, C.c_int32)
        for name in (
            "kind", "a_type", "b_type", "a_bits", "b_bits", "sparse", "ab_mode", "cta_group",
            "m", "n", "k", "depth", "scale_type", "mode", "iters", "instruction",
        )
    ]


# (name, restype, argtypes) of every exported entry point of include/b2g.h
_SIGS = [
    ("b2g_abi_version", C.c_int, []),
    ("b2g_status_string", C.c_char_p, [C.c_int]),
    ("b2g_last_error", C.c_char_p, [C.c_void_p]),
    ("b2g_create", C.c_int, [C.c_int, C.POINTER(C.c_void_p)]),
    ("b2g_destroy", C.c_int, [C.c_void_p]),
    ("b2g_device_info", C.c_int, [C.c_void_p] + [C.POINTER(C.c_int)] * 4),
    ("b2g_gemm", C.c_int, [C.c_void_p, C.POINTER(GemmDesc), C.c_void_p]),
    ("b2g_check", C.c_int, [C.c_void_p, C.c_void_p]),
    ("b2g_set_wait_limit", C.c_int, [C.c_void_p, C.c_uint64]),
    ("b2g_selftest_wait", C.c_int, [C.c_void_p, C.c_int, C.POINTER(C.c_uint64), C.c_void_p]),
    ("b2g_compress_24", C.c_int,
     [C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_void_p, C.c_void_p]),
    ("b2g_fill_f32", C.c_int,
     [C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_int64, C.c_uint64, C.c_int, C.c_void_p]),
    ("b2g_quantize", C.c_int,
     [C.c_void_p, C.c_int, C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_void_p, C.c_void_p]),
    ("b2g_tma2d_latency", C.c_int,
     [C.c_void_p, C.c_void_p, C.c_uint64, C.c_uint64, C.c_int, C.c_int, C.c_int, C.c_int64,
      C.c_void_p, C.c_void_p]),
    ("b2g_quantize_mx", C.c_int,
     [C.c_void_p, C.c_int, C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_void_p, C.c_void_p]),
    ("b2g_quantize_mx_block", C.c_int,
     [C.c_void_p, C.c_int, C.c_void_p, C.c_int64, C.c_int64, C.c_int, C.c_void_p, C.c_void_p,
      C.c_void_p]),
    ("b2g_quantize_nvfp4_block", C.c_int,
     [C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]),
    ("b2g_prune_24", C.c_int,
     [C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_int64, C.c_uint64, C.c_void_p]),
    ("b2g_gemm_host", C.c_int, [C.c_void_p, C.POINTER(GemmDesc), C.c_void_p]),
    ("b2g_plan_gemm", C.c_int,
     [C.POINTER(GemmDesc), C.c_int, C.c_int, C.POINTER(GemmPlan), C.c_char_p, C.c_int]),
    ("b2g_stream_bulk1d", C.c_int,
     [C.c_void_p, C.c_void_p, C.c_uint64, C.c_int, C.c_int, C.c_uint32, C.POINTER(C.c_float),
      C.c_void_p]),
    ("b2g_stream_tma2d", C.c_int,
     [C.c_void_p, C.c_void_p, C.c_uint64, C.c_uint64, C.c_int, C.c_int, C.c_int, C.c_int,
      C.POINTER(C.c_float), C.c_void_p]),
    ("b2g_probe_mma", C.c_int,
     [C.c_void_p, C.POINTER(ProbeDesc), C.POINTER(C.c_uint64), C.POINTER(C.c_uint64),
      C.POINTER(C.c_uint64)]),
    ("b2g_gemm_sparse_noalloc", C.c_int,
     [C.POINTER(GemmDesc), C.c_void_p, C.POINTER(C.c_char_p)]),
    ("b2g_prune_24_format", C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int64, C.c_int64,
                                      C.c_int64, C.c_uint64, C.c_void_p]),
    ("b2g_compress_24_format", C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int64, C.c_int64,
                                         C.c_void_p, C.c_void_p, C.c_void_p]),
    ("b2g_sparse_meta_bytes_format", C.c_size_t, [C.c_int, C.c_int64, C.c_int64]),
    ("b2g_sparse_meta_prepare_format", C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int64,
                                                 C.c_int64, C.c_void_p, C.c_void_p]),
    ("b2g_sparse_meta_bytes", C.c_size_t, [C.c_int64, C.c_int64]),
    ("b2g_sparse_meta_prepare", C.c_int,
     [C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_void_p]),
    ("b2g_trace_enable", C.c_int, [C.c_void_p, C.c_int]),
    ("b2g_trace_read", C.c_int, [C.c_void_p, C.POINTER(C.c_uint32), C.c_int]),
    ("b2g_encode_idesc", C.c_uint32, [C.c_int] * 7),
    ("b2g_encode_smem_desc", C.c_uint64, [C.c_uint32, C.c_uint32, C.c_uint32, C.c_int]),
]

EXPORTED = [s[0] for s in _SIGS]

_lib = None


def load() -> C.CDLL:
    """Load libb2g.so once; raise with the build command if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"libb2g.so not found at {LIB_PATH}; build it with "
            "`make -C microbench-blackwell_b200` (or __graft_entry__.build())"
        )
    lib = C.CDLL(LIB_PATH)
    for name, res, args in _SIGS:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib
