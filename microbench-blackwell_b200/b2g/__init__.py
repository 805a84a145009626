"""b2g -- Python host layer of the B200 tensor-core GEMM engine.

Thin wrapper over the C ABI (include/b2g.h, microbench-blackwell_b200/lib/libb2g.so).
PyTorch supplies device memory and streams only; every computation runs in a
CUDA kernel of libb2g.  Nothing here computes on the CPU, and nothing falls
back: a missing library or a non-zero status raises ``B2GError``.

The reference (lookup1980/microbench-blackwell) exposes no library; its
benchmark surface (Makefile variables, RESULT lines, CSV schemas) is kept by
the drop-in mains under microbench-blackwell_b200/drivers/, which call the same
ABI.  This module is what the tests, bench.py and the multi-GPU driver use.
"""
from __future__ import annotations

import ctypes as C

from . import _lib
from ._lib import (FMT_BF16, FMT_E2M1, FMT_E2M3, FMT_E3M2, FMT_E4M3, FMT_E5M2, FMT_F16,
                   FMT_MXF4, FMT_MXF8, FMT_NVFP4, FMT_S8, FMT_TF32, FMT_U8, GemmDesc,
                   ProbeDesc)

__all__ = [
    "B2GError", "Engine", "GemmDesc", "ProbeDesc", "plan_gemm",
    "FMT_BF16", "FMT_E4M3", "FMT_S8", "FMT_E2M1", "FMT_MXF8", "FMT_MXF4", "FMT_NVFP4",
    "FMT_TF32", "FMT_E5M2", "FMT_E2M3", "FMT_E3M2", "FMT_F16", "FMT_U8",
]


class B2GError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"b2g status {status} ({_lib.STATUS.get(status, '?')}): {msg}")
        self.status = status


# bits per element of the packed formats whose tensors hold bytes
_PACKED_BITS = {FMT_E2M1: 4, FMT_E2M3: 6, FMT_E3M2: 6, FMT_MXF4: 4, FMT_NVFP4: 4}


def _ptr(t) -> int:
    return 0 if t is None else int(t.data_ptr())


def _stream(stream) -> int:
    import torch

    if stream is None:
        stream = torch.cuda.current_stream()
    return int(stream.cuda_stream)


class Engine:
    """One handle of libb2g bound to one CUDA device."""

    def __init__(self, device: int = 0):
        self.lib = _lib.load()
        h = C.c_void_p()
        st = self.lib.b2g_create(int(device), C.byref(h))
        if st != _lib.B2G_OK:
            raise B2GError(st, f"b2g_create(device={device}) failed")
        self.h = h
        self.device = int(device)
        sm, clk, ma, mi = C.c_int(), C.c_int(), C.c_int(), C.c_int()
        self.lib.b2g_device_info(self.h, C.byref(sm), C.byref(clk), C.byref(ma), C.byref(mi))
        self.sm_count, self.clock_khz, self.cc = sm.value, clk.value, (ma.value, mi.value)

    def close(self):
        if getattr(self, "h", None):
            self.lib.b2g_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _ok(self, st: int, what: str):
        if st != _lib.B2G_OK:
            msg = self.lib.b2g_last_error(self.h)
            raise B2GError(st, f"{what}: {msg.decode() if msg else ''}")

    # ---------------------------------------------------------------- GEMM
    def gemm(self, A, B, C_out, fmt: int, *, M=None, N=None, K=None, alpha: float = 1.0,
             cta_group: int = 0, tile_n: int = 0, stages: int = 0, max_ctas: int = 0,
             ab_mode: int = 0, sparse: int = 0, meta=None, sfa=None, sfb=None,
             lda=None, ldb=None, ldc=None, meta_layout: int = 0, raster_m: int = 0, m_sub: int = 0,
             split_tail: int = 0, b_format: int = 0, mx_scale: int = 0, instruction: int = 0,
             stream=None):
        """C_out[M][N] (bf16) = alpha * A[M][K] . B[N][K]^T, all row-major tensors.

        A and B are tensors holding the stored format (e4m3 as raw bytes; packed
        e2m1 / fp6 as bytes of packed elements; tf32 as float32).  Leading dimensions
        default to the tensors' row strides, in stored elements.  b_format != 0 gives
        B its own kind::f8f6f4 element type; mx_scale = 1 adds OCP MX scales (sfa,
        sfb) to those element types (kind::mxf8f6f4); instruction = 1 issues the
        weight-stationary tcgen05.mma.ws (.ws.sp when sparse).
        """
        d = self._desc(A, B, C_out, fmt, M=M, N=N, K=K, alpha=alpha, cta_group=cta_group,
                       tile_n=tile_n, stages=stages, max_ctas=max_ctas, ab_mode=ab_mode,
                       sparse=sparse, meta=meta, sfa=sfa, sfb=sfb, lda=lda, ldb=ldb, ldc=ldc,
                       meta_layout=meta_layout, raster_m=raster_m, m_sub=m_sub,
                       split_tail=split_tail, b_format=b_format, mx_scale=mx_scale,
                       instruction=instruction)
        self._ok(self.lib.b2g_gemm(self.h, C.byref(d), _stream(stream)), "b2g_gemm")
        return C_out

    @staticmethod
    def _desc(A, B, C_out, fmt, *, M=None, N=None, K=None, alpha=1.0, cta_group=0, tile_n=0,
              stages=0, max_ctas=0, ab_mode=0, sparse=0, meta=None, sfa=None, sfb=None,
              lda=None, ldb=None, ldc=None, meta_layout=0, raster_m=0, m_sub=0,
              split_tail=0, b_format=0, mx_scale=0, instruction=0):
        d = GemmDesc()
        d.format = fmt
        d.sparse = sparse
        # stored elements per 8 bits of a row (1 for the byte and wider formats,
        # whose tensors hold whole elements)
        sub = {FMT_E2M1: 4, FMT_MXF4: 4, FMT_NVFP4: 4, FMT_E2M3: 6, FMT_E3M2: 6}
        bits, b_bits = sub.get(fmt, 8), sub.get(b_format or fmt, 8)
        elems = lambda nbytes: nbytes * 8 // bits
        d.M = M if M is not None else A.shape[0]
        d.N = N if N is not None else B.shape[0]
        if K is None:
            K = elems(A.shape[1]) * (2 if sparse else 1)
        d.K = K
        d.lda = lda if lda is not None else elems(A.stride(0))
        d.ldb = ldb if ldb is not None else B.stride(0) * 8 // b_bits
        d.b_format = b_format
        d.mx_scale = mx_scale
        d.instruction = instruction
        d.ldc = ldc if ldc is not None else C_out.stride(0)
        d.A, d.B, d.C = _ptr(A), _ptr(B), _ptr(C_out)
        d.sfa, d.sfb, d.meta = _ptr(sfa), _ptr(sfb), _ptr(meta)
        d.alpha = alpha
        d.cta_group, d.ab_mode, d.tile_n, d.stages, d.max_ctas = (
            cta_group, ab_mode, tile_n, stages, max_ctas)
        d.meta_layout = meta_layout
        d.raster_m = raster_m
        d.m_sub = m_sub
        d.split_tail = split_tail
        return d

    def gemm_host(self, A, B, C_out, fmt: int, *, alpha: float = 1.0, stream=None, **kw):
        """b2g_gemm_host: A, B, C_out are HOST tensors (pin them for full copy speed);
        copies in, runs the GEMM, copies C back and synchronises the stream."""
        d = self._desc(A, B, C_out, fmt, alpha=alpha, **kw)
        self._ok(self.lib.b2g_gemm_host(self.h, C.byref(d), _stream(stream)), "b2g_gemm_host")
        return C_out

    def check(self, stream=None):
        """Synchronise the stream and raise if a kernel recorded a device error."""
        self._ok(self.lib.b2g_check(self.h, _stream(stream)), "b2g_check")

    def set_wait_limit(self, ns: int):
        """b2g_set_wait_limit: limit of the kernel-side bounded waits (0 = 2 s)."""
        self._ok(self.lib.b2g_set_wait_limit(self.h, C.c_uint64(int(ns))), "b2g_set_wait_limit")

    def selftest_wait(self, mode: int, stream=None):
        """b2g_selftest_wait: (status, elapsed ns) of a bounded wait on something that
        nothing completes (mode 0 an mbarrier, 1 a global flag); B2G_ERR_TIMEOUT is
        the expected status.  Does not raise on that status."""
        t = C.c_uint64(0)
        st = self.lib.b2g_selftest_wait(self.h, int(mode), C.byref(t), _stream(stream))
        return st, t.value

    # ---------------------------------------------------------------- diagnostics
    TRACE_WORDS = 16

    def trace_enable(self, max_ctas: int):
        self._ok(self.lib.b2g_trace_enable(self.h, int(max_ctas)), "b2g_trace_enable")
        self._trace_ctas = int(max_ctas)

    def trace_read(self):
        n = getattr(self, "_trace_ctas", 0) * self.TRACE_WORDS
        buf = (C.c_uint32 * max(n, 1))()
        self._ok(self.lib.b2g_trace_read(self.h, buf, n), "b2g_trace_read")
        return [list(buf[i * self.TRACE_WORDS:(i + 1) * self.TRACE_WORDS])
                for i in range(n // self.TRACE_WORDS)]

    # ---------------------------------------------------------------- data
    def fill(self, out, seed: int, dist: int = 0, row0: int = 0, stream=None):
        rows, cols = out.shape
        self._ok(self.lib.b2g_fill_f32(self.h, _ptr(out), rows, cols, row0, C.c_uint64(seed),
                                       dist, _stream(stream)), "b2g_fill_f32")
        return out

    def quantize(self, fmt: int, x, out, sf=None, stream=None):
        rows, cols = x.shape
        self._ok(self.lib.b2g_quantize(self.h, fmt, _ptr(x), rows, cols, _ptr(out), _ptr(sf),
                                       _stream(stream)), "b2g_quantize")
        return out

    def quantize_mx(self, elem_fmt: int, x, out, sf, stream=None, block: int = 32):
        """b2g_quantize_mx(_block): OCP MX quantisation to a kind::f8f6f4 element format,
        one E8M0 scale per `block` (32, or 64 for the 2:4-sparse MX GEMM) elements."""
        rows, cols = x.shape
        self._ok(self.lib.b2g_quantize_mx_block(self.h, elem_fmt, _ptr(x), rows, cols, block,
                                                _ptr(out), _ptr(sf), _stream(stream)),
                 "b2g_quantize_mx_block")
        return out

    def quantize_nvfp4(self, x, out, sf, stream=None, block: int = 16):
        """b2g_quantize_nvfp4_block: packed e2m1 and one ue4m3 scale per `block` (16, or
        32 for the 4:8-sparse NVFP4 GEMM) elements."""
        rows, cols = x.shape
        self._ok(self.lib.b2g_quantize_nvfp4_block(self.h, _ptr(x), rows, cols, block, _ptr(out),
                                                   _ptr(sf), _stream(stream)),
                 "b2g_quantize_nvfp4_block")
        return out

    def prune_24(self, m, seed: int, row0: int = 0, stream=None, fmt: int = FMT_BF16):
        """Zero 2 of every 4 elements along each row of the stored codes `m`: 16-bit
        (FMT_BF16, FMT_F16), 8-bit (FMT_E4M3, FMT_E5M2, FMT_S8, FMT_U8, FMT_MXF8) or
        packed fp4 / fp6 (FMT_E2M1, FMT_E2M3, FMT_E3M2: `m` holds bytes) codes; tf32
        (FMT_TF32) is pruned 1:2."""
        rows, cols = m.shape
        cols = cols * 8 // _PACKED_BITS[fmt] if fmt in _PACKED_BITS else cols
        self._ok(self.lib.b2g_prune_24_format(self.h, fmt, _ptr(m), rows, cols, row0,
                                              C.c_uint64(seed), _stream(stream)),
                 "b2g_prune_24_format")
        return m

    def compress_24(self, dense, comp, meta, stream=None, fmt: int = FMT_BF16):
        """2:4 compression of `dense` ([M][K] codes of `fmt`) into comp [M][K/2] and the
        canonical metadata [M][K/32] words (packed fp4 / fp6: K counts elements, not
        the bytes of `dense`'s rows)."""
        M, K = dense.shape
        K = K * 8 // _PACKED_BITS[fmt] if fmt in _PACKED_BITS else K
        self._ok(self.lib.b2g_compress_24_format(self.h, fmt, _ptr(dense), M, K, _ptr(comp),
                                                 _ptr(meta), _stream(stream)),
                 "b2g_compress_24_format")
        return comp, meta

    def sparse_meta_bytes(self, M: int, K: int, fmt: int = FMT_BF16) -> int:
        return int(self.lib.b2g_sparse_meta_bytes_format(fmt, M, K))

    def sparse_meta_prepare(self, meta, M: int, K: int, ready, stream=None, fmt: int = FMT_BF16):
        """Canonical metadata -> the engine's TMEM-ready layout (meta_layout=1)."""
        self._ok(self.lib.b2g_sparse_meta_prepare_format(self.h, fmt, _ptr(meta), M, K, _ptr(ready),
                                                         _stream(stream)),
                 "b2g_sparse_meta_prepare_format")
        return ready

    # ---------------------------------------------------------------- probes
    def stream_bulk1d(self, data, nbytes, ctas_per_sm, num_stages, load_bytes, stream=None) -> float:
        ms = C.c_float(0.0)
        self._ok(self.lib.b2g_stream_bulk1d(self.h, _ptr(data), nbytes, ctas_per_sm, num_stages,
                                            load_bytes, C.byref(ms), _stream(stream)),
                 "b2g_stream_bulk1d")
        return ms.value

    def tma2d_latency(self, data, width, height, box_w, box_h, ctas_per_sm, row0, cycles,
                      stream=None):
        """b2g_tma2d_latency: one box load per CTA; per-CTA cycles into `cycles` (uint32)."""
        self._ok(self.lib.b2g_tma2d_latency(self.h, _ptr(data), width, height, box_w, box_h,
                                            ctas_per_sm, row0, _ptr(cycles), _stream(stream)),
                 "b2g_tma2d_latency")
        return cycles

    def stream_tma2d(self, data, width, height, ctas_per_sm, num_stages, box_w, box_h,
                     stream=None) -> float:
        ms = C.c_float(0.0)
        self._ok(self.lib.b2g_stream_tma2d(self.h, _ptr(data), width, height, ctas_per_sm,
                                           num_stages, box_w, box_h, C.byref(ms),
                                           _stream(stream)), "b2g_stream_tma2d")
        return ms.value

    def probe_mma(self, **kw):
        p = ProbeDesc()
        for k, v in kw.items():
            setattr(p, k, v)
        cyc, tot, med = C.c_uint64(), C.c_uint64(), C.c_uint64()
        self._ok(self.lib.b2g_probe_mma(self.h, C.byref(p), C.byref(cyc), C.byref(tot),
                                        C.byref(med)), "b2g_probe_mma")
        return cyc.value, tot.value, med.value


def plan_gemm(fmt: int, M: int, N: int, K: int, *, sm_count: int = 148, max_clusters: int = 0,
              sparse: int = 0, lda=None, ldb=None, ldc=None, **options) -> dict:
    """b2g_plan_gemm: the launch configuration b2g_gemm would use, computed on the host
    without a device.  Raises B2GError (status, reason) where b2g_gemm would refuse.
    `options` are descriptor fields (cta_group, tile_n, stages, max_ctas, ab_mode,
    m_sub, split_tail, raster_m, meta_layout, b_format, mx_scale, instruction).  The dict
    holds the b2g_gemm_plan fields (variant, kind, tile sizes, stages, smem_bytes, k_blocks,
    k_atoms, split tail, units, clusters, threads, ...)."""
    d = _lib.GemmDesc()
    d.format, d.sparse, d.M, d.N, d.K = fmt, sparse, M, N, K
    d.lda = lda if lda is not None else (K // 2 if sparse else K)
    d.ldb = ldb if ldb is not None else K
    d.ldc = ldc if ldc is not None else N
    for k, v in options.items():
        setattr(d, k, v)
    out = _lib.GemmPlan()
    msg = C.create_string_buffer(512)
    st = _lib.load().b2g_plan_gemm(C.byref(d), sm_count, max_clusters, C.byref(out), msg, 512)
    if st != _lib.B2G_OK:
        raise B2GError(st, f"b2g_plan_gemm: {msg.value.decode()}")
    return {name: getattr(out, name) for name, _ in _lib.GemmPlan._fields_ if name != "reserved"}


def encode_idesc(kind, a_type, b_type, m, n, sparse=0, scale_type=0) -> int:
    return _lib.load().b2g_encode_idesc(kind, a_type, b_type, m, n, sparse, scale_type)


def encode_smem_desc(addr, lbo, sbo, swizzle) -> int:
    return _lib.load().b2g_encode_smem_desc(addr, lbo, sbo, swizzle)
