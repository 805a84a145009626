// b2g_api.cu -- the C ABI of libb2g (declared in include/b2g.h).
//
// Validation, configuration choice, TMA tensor-map construction and dispatch to
// the sm_100a kernels.  No CPU fallback exists: every compute entry point runs a
// CUDA kernel of this library or returns an error status.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <new>

#include "b2g.h"
#include "b2g_desc.h"
#include "b2g_gemm.h"
#include "b2g_ptx.cuh"

using namespace b2g;

typedef CUresult (*PFN_encodeTiled_t)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                      const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                      const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                      CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// b2g_gemm_host splits M into at most kHostChunks row chunks and N into at most
// kHostColChunks column chunks
constexpr int kHostChunks = 4;
constexpr int kHostColChunks = 4;
// widest dense tile (MMA N) that takes two K atoms per ring slot
constexpr int kTwoAtomMaxN = 128;

struct b2g_handle {
  int device;
  int sm_count;
  int clock_khz;
  int cc_major, cc_minor;
  uint32_t* d_err;
  PFN_encodeTiled_t encode_tiled;
  void* ws;                // device workspace of b2g_gemm_host
  size_t ws_bytes;
  void* meta_ws;           // scratch: engine-layout 2:4 metadata of the last sparse call
  size_t meta_ws_bytes;
  void* sf_ws;             // scratch: engine-layout NVFP4 scale factors of the last call
  size_t sf_ws_bytes;
  void* d_probe;           // b2g_probe_mma result words
  void* part_ws;           // split tail: fp32 partial tiles
  size_t part_ws_bytes;
  uint32_t* flag_ws;       // split tail: per-warp stamps (zeroed when allocated)
  size_t flag_ws_bytes;
  uint32_t epoch;          // stamp of the last split-tail launch
  uint64_t wait_ns;        // limit of the kernel-side bounded waits (0: kWaitLimitNs)
  // b2g_gemm_host pipeline: copy-in and copy-out streams, events per row chunk
  cudaStream_t s_in, s_out;
  cudaEvent_t ev_start, ev_out, ev_c, ev_a[kHostChunks], ev_b[kHostColChunks];
  bool pipe_ready;
  uint32_t* trace_host;    // host-mapped progress trace (nullable)
  uint32_t* trace_dev;
  int trace_ctas;
  // co-resident cluster pairs per kernel instance and shared-memory size (the
  // occupancy query of cta_group::2 launches), kept after the first query
  struct OccEntry {
    uint32_t key;
    int smem, clusters;
  } occ[16];
  int n_occ;
  char last_error[512];
};

// Occupancy cache key of a GEMM kernel instance.
static uint32_t occ_key(int kind, int cg, int var, bool ts, int m_sub, int k_atoms, bool ws) {
  return (uint32_t)kind | ((uint32_t)cg << 4) | ((uint32_t)var << 6) | ((uint32_t)ts << 10) |
         ((uint32_t)m_sub << 11) | ((uint32_t)k_atoms << 13) | ((uint32_t)ws << 15);
}

static b2g_status fail(b2g_handle* h, b2g_status s, const char* fmt, ...) {
  if (h) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(h->last_error, sizeof(h->last_error), fmt, ap);
    va_end(ap);
  }
  return s;
}

#define B2G_CUDA(h, expr)                                                                  \
  do {                                                                                     \
    cudaError_t e__ = (expr);                                                              \
    if (e__ != cudaSuccess)                                                                \
      return fail((h), B2G_ERR_CUDA, "%s failed: %s", #expr, cudaGetErrorString(e__));     \
  } while (0)

// Make the handle's device current for the duration of a call.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

extern "C" {

int b2g_abi_version(void) { return B2G_ABI_VERSION; }

const char* b2g_status_string(b2g_status s) {
  switch (s) {
    case B2G_OK: return "ok";
    case B2G_ERR_INVALID: return "invalid argument";
    case B2G_ERR_CUDA: return "CUDA error";
    case B2G_ERR_TIMEOUT: return "kernel wait timed out";
    case B2G_ERR_UNSUPPORTED: return "unsupported";
    case B2G_ERR_NO_DEVICE: return "no sm_100 device";
    case B2G_ERR_MISMATCH: return "device self-check mismatch";
  }
  return "unknown status";
}

const char* b2g_last_error(const b2g_handle* h) { return h ? h->last_error : "null handle"; }

b2g_status b2g_create(int device, b2g_handle** out) {
  if (!out) return B2G_ERR_INVALID;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0 || device < 0 || device >= n)
    return B2G_ERR_NO_DEVICE;
  b2g_handle* h = new (std::nothrow) b2g_handle();
  if (!h) return B2G_ERR_INVALID;
  h->device = device;
  DeviceGuard g(device);
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) {
    delete h;
    return B2G_ERR_NO_DEVICE;
  }
  h->sm_count = prop.multiProcessorCount;
  cudaDeviceGetAttribute(&h->clock_khz, cudaDevAttrClockRate, device);
  h->cc_major = prop.major;
  h->cc_minor = prop.minor;
  if (prop.major != 10) {
    delete h;
    return B2G_ERR_NO_DEVICE;
  }
  if (cudaMalloc(&h->d_err, sizeof(uint32_t)) != cudaSuccess ||
      cudaMemset(h->d_err, 0, sizeof(uint32_t)) != cudaSuccess) {
    delete h;
    return B2G_ERR_CUDA;
  }
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) !=
          cudaSuccess ||
      q != cudaDriverEntryPointSuccess || !fn) {
    cudaFree(h->d_err);
    delete h;
    return B2G_ERR_CUDA;
  }
  h->encode_tiled = reinterpret_cast<PFN_encodeTiled_t>(fn);
  *out = h;
  return B2G_OK;
}

b2g_status b2g_destroy(b2g_handle* h) {
  if (!h) return B2G_OK;
  {
    DeviceGuard g(h->device);
    cudaFree(h->d_err);
    if (h->ws) cudaFree(h->ws);
    if (h->meta_ws) cudaFree(h->meta_ws);
    if (h->sf_ws) cudaFree(h->sf_ws);
    if (h->d_probe) cudaFree(h->d_probe);
    if (h->part_ws) cudaFree(h->part_ws);
    if (h->flag_ws) cudaFree(h->flag_ws);
    if (h->pipe_ready) {
      cudaStreamSynchronize(h->s_in);
      cudaStreamSynchronize(h->s_out);
      cudaStreamDestroy(h->s_in);
      cudaStreamDestroy(h->s_out);
      cudaEventDestroy(h->ev_start);
      cudaEventDestroy(h->ev_out);
      cudaEventDestroy(h->ev_c);
      for (int i = 0; i < kHostChunks; ++i) cudaEventDestroy(h->ev_a[i]);
      for (int j = 0; j < kHostColChunks; ++j) cudaEventDestroy(h->ev_b[j]);
    }
    if (h->trace_host) cudaFreeHost(h->trace_host);
  }
  delete h;
  return B2G_OK;
}

b2g_status b2g_device_info(const b2g_handle* h, int* sm_count, int* clock_khz, int* cc_major,
                           int* cc_minor) {
  if (!h) return B2G_ERR_INVALID;
  if (sm_count) *sm_count = h->sm_count;
  if (clock_khz) *clock_khz = h->clock_khz;
  if (cc_major) *cc_major = h->cc_major;
  if (cc_minor) *cc_minor = h->cc_minor;
  return B2G_OK;
}

b2g_status b2g_check(b2g_handle* h, void* stream) {
  if (!h) return B2G_ERR_INVALID;
  DeviceGuard g(h->device);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  B2G_CUDA(h, cudaStreamSynchronize(s));
  uint32_t w = 0;
  B2G_CUDA(h, cudaMemcpyAsync(&w, h->d_err, sizeof(w), cudaMemcpyDeviceToHost, s));
  B2G_CUDA(h, cudaStreamSynchronize(s));
  if (w) {
    B2G_CUDA(h, cudaMemsetAsync(h->d_err, 0, sizeof(uint32_t), s));
    B2G_CUDA(h, cudaStreamSynchronize(s));
    if (w & ERRW_BAD_SPARSITY)
      return fail(h, B2G_ERR_INVALID, "2:4 compressor: a group of 4 holds more than 2 non-zeros");
    return fail(h, B2G_ERR_TIMEOUT, "kernel wait timed out (error word 0x%x)", w);
  }
  return B2G_OK;
}

b2g_status b2g_set_wait_limit(b2g_handle* h, uint64_t ns) {
  if (!h) return B2G_ERR_INVALID;
  if (ns != 0 && (ns < 1000 || ns > kWaitLimitNs))
    return fail(h, B2G_ERR_INVALID, "b2g_set_wait_limit: 0 (default) or 1000 .. %llu ns",
                (unsigned long long)kWaitLimitNs);
  h->wait_ns = ns;
  return B2G_OK;
}

b2g_status b2g_selftest_wait(b2g_handle* h, int mode, uint64_t* elapsed_ns, void* stream) {
  if (!h) return B2G_ERR_INVALID;
  if (mode != 0 && mode != 1) return fail(h, B2G_ERR_INVALID, "b2g_selftest_wait: mode 0 or 1");
  DeviceGuard g(h->device);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (!h->d_probe) B2G_CUDA(h, cudaMalloc(&h->d_probe, 4 * sizeof(unsigned long long)));
  unsigned long long* words = static_cast<unsigned long long*>(h->d_probe);
  // words[0]: elapsed time; words[1]: the flag nothing sets (zero)
  B2G_CUDA(h, cudaMemsetAsync(words, 0, 4 * sizeof(unsigned long long), s));
  B2G_CUDA(h, wait_selftest_launch(mode, h->wait_ns, reinterpret_cast<const uint32_t*>(words + 1),
                                   h->d_err, words, s));
  unsigned long long t = 0;
  B2G_CUDA(h, cudaMemcpyAsync(&t, words, sizeof(t), cudaMemcpyDeviceToHost, s));
  B2G_CUDA(h, cudaStreamSynchronize(s));
  if (elapsed_ns) *elapsed_ns = t;
  return b2g_check(h, stream);
}

b2g_status b2g_trace_enable(b2g_handle* h, int max_ctas) {
  if (!h || max_ctas < 0) return B2G_ERR_INVALID;
  DeviceGuard g(h->device);
  if (h->trace_host) {
    B2G_CUDA(h, cudaDeviceSynchronize());
    cudaFreeHost(h->trace_host);
    h->trace_host = h->trace_dev = nullptr;
    h->trace_ctas = 0;
  }
  if (max_ctas == 0) return B2G_OK;
  const size_t bytes = (size_t)max_ctas * kTraceWords * sizeof(uint32_t);
  void* p = nullptr;
  B2G_CUDA(h, cudaHostAlloc(&p, bytes, cudaHostAllocMapped));
  memset(p, 0, bytes);
  void* dp = nullptr;
  B2G_CUDA(h, cudaHostGetDevicePointer(&dp, p, 0));
  h->trace_host = (uint32_t*)p;
  h->trace_dev = (uint32_t*)dp;
  h->trace_ctas = max_ctas;
  return B2G_OK;
}

b2g_status b2g_trace_read(const b2g_handle* h, uint32_t* out, int nwords) {
  if (!h || !out || nwords < 0) return B2G_ERR_INVALID;
  const int have = h->trace_ctas * kTraceWords;
  for (int i = 0; i < nwords; ++i)
    out[i] = i < have ? ((volatile const uint32_t*)h->trace_host)[i] : 0u;
  return B2G_OK;
}

uint32_t b2g_encode_idesc(int kind, int a_type, int b_type, int m, int n, int sparse,
                          int scale_type) {
  return encode_idesc(kind, a_type, b_type, m, n, sparse, scale_type);
}

uint64_t b2g_encode_smem_desc(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                              int swizzle) {
  return encode_smem_desc(smem_addr, lbo_bytes, sbo_bytes, swizzle);
}

// ------------------------------------------------------------------ GEMM
static b2g_status make_tmap_2d(b2g_handle* h, CUtensorMap* tm, CUtensorMapDataType dt,
                               const void* base, uint64_t inner, uint64_t outer,
                               uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                               CUtensorMapSwizzle swz) {
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  CUresult r = h->encode_tiled(tm, dt, 2, const_cast<void*>(base), dims, strides, box, es,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(h, B2G_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) dims=%llu x %llu", (int)r,
                (unsigned long long)inner, (unsigned long long)outer);
  return B2G_OK;
}

// The launch configuration of one GEMM, decided on the host from the descriptor's
// shapes and options alone (no device, no pointers): b2g_gemm launches exactly
// this, and b2g_gemm_plan returns its public part.
struct Plan {
  b2g_gemm_plan pub;
  int kind, a_type, elem_bits, var;
  bool sparse, ts;
  // fp4 / fp6 of kind::f8f6f4: packed in memory, unpacked by the TMA into the
  // MMA's 16-byte chunks (16 elements per chunk), so 128 elements per 128-byte
  // shared-memory row like fp8
  bool unpack;
  // B's element type (A's unless b_format names another kind::f8f6f4 type)
  int b_type, b_elem_bits;
  bool b_unpack;
  CUtensorMapDataType b_dt;
  CUtensorMapDataType dt;
  int64_t a_cols;   // stored A elements per row
  size_t smem;
  int b_rows;       // B rows of one CTA's tile
  bool ws;          // weight-stationary MMA form (tcgen05.mma.ws{.sp})
};

static b2g_status say_plan(char* msg, size_t len, b2g_status st, const char* fmt, ...) {
  if (msg && len) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(msg, len, fmt, ap);
    va_end(ap);
  }
  return st;
}

// Element types of kind::f8f6f4: type code, bits in memory, whether the TMA unpacks
// them (fp4 sixteen per 8 bytes, fp6 sixteen per 12 bytes) and the tensor-map type.
static bool f8f6f4_type(int fmt, int* code, int* bits, bool* unpack, CUtensorMapDataType* dt) {
  switch (fmt) {
    case B2G_FMT_E4M3: *code = 0; *bits = 8; *unpack = false; *dt = CU_TENSOR_MAP_DATA_TYPE_UINT8; return true;
    case B2G_FMT_E5M2: *code = 1; *bits = 8; *unpack = false; *dt = CU_TENSOR_MAP_DATA_TYPE_UINT8; return true;
    case B2G_FMT_E2M3: *code = 3; *bits = 6; *unpack = true; *dt = CU_TENSOR_MAP_DATA_TYPE_16U6_ALIGN16B; return true;
    case B2G_FMT_E3M2: *code = 4; *bits = 6; *unpack = true; *dt = CU_TENSOR_MAP_DATA_TYPE_16U6_ALIGN16B; return true;
    case B2G_FMT_E2M1: *code = 5; *bits = 4; *unpack = true; *dt = CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B; return true;
    default: return false;
  }
}

static b2g_status plan_gemm(const b2g_gemm_desc* d, int sm_count, int max_clusters, Plan* p,
                            char* msg, size_t len) {
  memset(p, 0, sizeof(*p));
  if (sm_count <= 0) return say_plan(msg, len, B2G_ERR_INVALID, "sm_count must be positive");
  if (d->M <= 0 || d->N <= 0 || d->K <= 0)
    return say_plan(msg, len, B2G_ERR_INVALID, "M, N, K must be positive");
  if (d->M > INT32_MAX / 2 || d->N > INT32_MAX / 2 || d->K > INT32_MAX / 2)
    return say_plan(msg, len, B2G_ERR_INVALID, "dimension too large");
  if (d->ab_mode != 0 && d->ab_mode != 1)
    return say_plan(msg, len, B2G_ERR_INVALID, "ab_mode must be 0 or 1");
  const bool sparse = d->sparse != 0, ts = d->ab_mode == 1;
  p->sparse = sparse;
  p->ts = ts;
  p->var = sparse ? GEMM_SPARSE : GEMM_DENSE;
  switch (d->format) {
    case B2G_FMT_BF16:
      p->kind = KIND_F16; p->a_type = 1; p->elem_bits = 16; p->dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
      break;
    case B2G_FMT_E4M3:
    case B2G_FMT_E5M2:
    case B2G_FMT_E2M1:  // scale-free, on kind::f8f6f4 (fp4 / fp6 unpacked by the TMA)
    case B2G_FMT_E2M3:
    case B2G_FMT_E3M2:
      p->kind = KIND_F8F6F4;
      f8f6f4_type(d->format, &p->a_type, &p->elem_bits, &p->unpack, &p->dt);
      break;
    case B2G_FMT_S8:  // kind::i8, signed type code 1, s32 accumulator
    case B2G_FMT_U8:  // unsigned type code 0
      p->kind = KIND_I8; p->a_type = d->format == B2G_FMT_S8 ? 1 : 0; p->elem_bits = 8;
      p->dt = CU_TENSOR_MAP_DATA_TYPE_UINT8;
      break;
    case B2G_FMT_F16:  // kind::f16 type code 0 (A and B both fp16: the kind takes no mix)
      p->kind = KIND_F16; p->a_type = 0; p->elem_bits = 16; p->dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
      break;
    case B2G_FMT_TF32:  // kind::tf32 type code 2, fp32 storage
      p->kind = KIND_TF32; p->a_type = 2; p->elem_bits = 32; p->dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
      break;
    case B2G_FMT_NVFP4:
      // packed e2m1, tensor maps in bytes; MXF4 type code of E2M1 is 1
      p->kind = KIND_MXF4NVF4; p->a_type = 1; p->elem_bits = 4; p->dt = CU_TENSOR_MAP_DATA_TYPE_UINT8;
      p->var = GEMM_NVFP4;
      break;
    case B2G_FMT_MXF8:  // e4m3 operands, one E8M0 scale per 32 K
      p->kind = KIND_MXF8F6F4; p->a_type = 0; p->elem_bits = 8; p->dt = CU_TENSOR_MAP_DATA_TYPE_UINT8;
      p->var = GEMM_MXF8;
      break;
    case B2G_FMT_MXF4:  // packed e2m1, one E8M0 scale per 32 K
      p->kind = KIND_MXF4; p->a_type = 1; p->elem_bits = 4; p->dt = CU_TENSOR_MAP_DATA_TYPE_UINT8;
      p->var = GEMM_MXF4;
      break;
    default:
      return say_plan(msg, len, B2G_ERR_UNSUPPORTED, "format %d not built yet", d->format);
  }
  if (d->mx_scale) {
    // OCP MX scales on a kind::f8f6f4 element format: the block-scaled kind::mxf8f6f4
    // variant (B2G_FMT_MXF8 is e4m3 with this on)
    if (p->kind != KIND_F8F6F4 && d->format != B2G_FMT_MXF8)
      return say_plan(msg, len, B2G_ERR_UNSUPPORTED,
                      "mx_scale is built for the kind::f8f6f4 element formats");
    p->kind = KIND_MXF8F6F4;
    p->var = GEMM_MXF8;
  }
  if (sparse && p->var == GEMM_NVFP4) {
    // 4:8-sparse A in pairs on kind::mxf4nvf4 block16: the MXFP4 pair layout, one
    // ue4m3 scale per 32 dense K (the MMA's four scales over its 128)
    p->var = GEMM_NVFP4_SP;
    if (d->K % 64)
      return say_plan(msg, len, B2G_ERR_INVALID, "sparse NVFP4: K %% 64 == 0 needed");
  }
  if (sparse && p->var == GEMM_MXF4) {
    // 4:8-sparse A in pairs on kind::mxf4: 2:4 on the bytes of packed e2m1 (a byte
    // is a pair), metadata words of 64 elements, one E8M0 scale per 64 dense K
    p->var = GEMM_MXF4_SP;
    if (d->K % 64)
      return say_plan(msg, len, B2G_ERR_INVALID, "sparse MXFP4: K %% 64 == 0 needed");
  }
  if (sparse && p->var == GEMM_MXF8) {
    // 2:4-sparse A on kind::mxf8f6f4 (tcgen05.mma.sp ... block_scale): the 8-bit
    // element types, unpacked fp4 / fp6 not built
    if (p->elem_bits != 8 || p->unpack)
      return say_plan(msg, len, B2G_ERR_UNSUPPORTED,
                      "2:4-sparse A with MX scales is built for e4m3 and e5m2");
    p->var = GEMM_MXF8_SP;
    if (d->K % 64)
      return say_plan(msg, len, B2G_ERR_INVALID,
                      "2:4-sparse MX: K %% 64 == 0 needed (one scale per 64 dense K)");
  }
  p->b_type = p->a_type;
  p->b_elem_bits = p->elem_bits;
  p->b_unpack = p->unpack;
  p->b_dt = p->dt;
  const bool mixed = d->b_format != 0 && d->b_format != d->format;
  if (mixed) {
    int ac, ab;
    bool au;
    CUtensorMapDataType adt;
    // (sparse A mixes too, on kind::f8f6f4 without MX scales)
    if ((sparse && p->var != GEMM_SPARSE) || !f8f6f4_type(d->format, &ac, &ab, &au, &adt) ||
        !f8f6f4_type(d->b_format, &p->b_type, &p->b_elem_bits, &p->b_unpack, &p->b_dt))
      return say_plan(msg, len, B2G_ERR_UNSUPPORTED,
                      "A and B formats differ: only kind::f8f6f4 element types mix");
  }
  const int var = p->var, elem_bits = p->elem_bits, b_bits = p->b_elem_bits;
  if (sparse && d->format != B2G_FMT_BF16 && d->format != B2G_FMT_F16 &&
      d->format != B2G_FMT_E4M3 && d->format != B2G_FMT_E5M2 && d->format != B2G_FMT_S8 &&
      d->format != B2G_FMT_U8 && d->format != B2G_FMT_TF32 && d->format != B2G_FMT_MXF8 &&
      d->format != B2G_FMT_E2M1 && d->format != B2G_FMT_E2M3 && d->format != B2G_FMT_E3M2 &&
      d->format != B2G_FMT_MXF4 && d->format != B2G_FMT_NVFP4)
    return say_plan(msg, len, B2G_ERR_UNSUPPORTED,
                    "structured-sparse GEMM is built for bf16, fp16, e4m3, e5m2, e2m1, e2m3, e3m2, "
                    "s8, u8 (2:4), MX e4m3 / e5m2 (2:4), MXFP4 and NVFP4 (4:8 in pairs) and tf32 "
                    "(1:2)");
  // sparse fp4 / fp6: the compressed A row (K / 2 elements) in whole 128-element boxes
  if (sparse && p->unpack && d->K % 256)
    return say_plan(msg, len, B2G_ERR_INVALID, "sparse fp4 / fp6 (f8f6f4): K %% 256 == 0 needed");
  // the s32 accumulator of kind::i8 must not wrap: |a*b| <= 128*128 (s8) or 255*255 (u8)
  if (p->kind == KIND_I8 && d->K > (d->format == B2G_FMT_S8 ? 131071 : 33025))
    return say_plan(msg, len, B2G_ERR_INVALID,
                    "i8: K above %d could overflow the s32 accumulator",
                    d->format == B2G_FMT_S8 ? 131071 : 33025);
  // the unpacking tensor maps take K in whole 128-element boxes and row strides
  // in multiples of 32 bytes
  if (((p->unpack || p->b_unpack) && d->K % 128) || (p->unpack && d->lda % 128) ||
      (p->b_unpack && d->ldb % 128))
    return say_plan(msg, len, B2G_ERR_INVALID,
                    "fp4 / fp6 (f8f6f4): K, lda and ldb must be multiples of 128");
  if (ts && (sparse || mixed || d->mx_scale ||
             (d->format != B2G_FMT_BF16 && d->format != B2G_FMT_E4M3)))
    return say_plan(msg, len, B2G_ERR_UNSUPPORTED, "TS operands are built for dense bf16 / e4m3");
  auto row_bytes = [&](int64_t n) { return n * elem_bits / 8; };
  p->a_cols = sparse ? d->K / 2 : d->K;
  if (sparse && d->K % 32) return say_plan(msg, len, B2G_ERR_INVALID, "sparse: K %% 32 == 0 needed");
  if (sparse && d->meta_layout != 0 && d->meta_layout != 1)
    return say_plan(msg, len, B2G_ERR_INVALID, "meta_layout must be 0 or 1");
  if (gemm_block_scaled(var) && d->K % 32)
    return say_plan(msg, len, B2G_ERR_INVALID, "block-scaled formats: K %% 32 == 0 needed");
  if (d->lda < p->a_cols || d->ldb < d->K || d->ldc < d->N)
    return say_plan(msg, len, B2G_ERR_INVALID, "leading dimension smaller than the matrix extent");
  if (row_bytes(d->lda) % 16 || d->ldb * b_bits / 8 % 16 || (d->lda * elem_bits) % 8 ||
      (d->ldb * b_bits) % 8)
    return say_plan(msg, len, B2G_ERR_INVALID, "lda/ldb must be multiples of 16 bytes (TMA stride rule)");

  // tcgen05.mma.ws{.sp}: the weight-stationary form exists for cta_group::1 and the
  // kinds without block scaling, with N 64 / 128 / 256 (umma_tput.cu and
  // tcgen05_sparse_mma.cu issue it for those kinds only)
  if (d->instruction != 0 && d->instruction != 1)
    return say_plan(msg, len, B2G_ERR_INVALID, "instruction must be 0 (mma) or 1 (mma.ws)");
  const bool ws = d->instruction == 1;
  p->ws = ws;
  if (ws && (gemm_block_scaled(var) || ts || d->cta_group == 2 || d->m_sub == 2))
    return say_plan(msg, len, B2G_ERR_UNSUPPORTED,
                    ".ws is built for SS operands, cta_group 1, one A sub-tile and the kinds "
                    "without block scaling");
  int cg = d->cta_group;
  if (cg == 0) cg = ws ? 1 : (d->M >= 256) ? 2 : 1;
  if (cg != 1 && cg != 2) return say_plan(msg, len, B2G_ERR_INVALID, "cta_group must be 0, 1 or 2");
  int bn = d->tile_n;
  if (bn == 0 && ws) bn = (d->N >= 256 && !sparse) ? 256 : (d->N > 64 ? 128 : 64);
  // 4:8-sparse MXFP4 / NVFP4: 192-column tiles (with two A sub-tiles, the default on
  // long K, the accumulators, metadata ring and scale factors fill TMEM exactly);
  // measured at 16384³: 7382 (NVFP4) and 7781 (MXFP4) TFLOP/s against 6451-6727 and
  // 6675-7126 with one sub-tile
  if (bn == 0 && (var == GEMM_NVFP4_SP || var == GEMM_MXF4_SP)) bn = 192;
  if (ws && bn != 64 && bn != 128 && bn != 256)
    return say_plan(msg, len, B2G_ERR_INVALID, ".ws: tile_n must be 64, 128 or 256");
  if (bn == 0) {
    bn = (sparse || gemm_block_scaled(var) || ts) ? 224
                                                  : (d->N >= 256) ? 256 : (d->N > 64 ? 128 : 64);
    if (bn == 256) {
      // Dense, wide N: 256 or 192 columns, whichever needs fewer column-steps of
      // MMA over whole waves of the persistent grid, counting 32 columns of
      // per-tile overhead (bf16 4096^3 on 74 pairs: 4 waves of 256 = 1152 against
      // 5 waves of 192 = 1120, measured 1378 against 1398 TFLOP/s; at 8192^3 the
      // 256 tile wins, 4032 against 4256).
      int64_t cl = sm_count / cg;
      if (max_clusters > 0 && max_clusters < cl) cl = max_clusters;
      if (d->max_ctas > 0 && d->max_ctas / cg < cl) cl = d->max_ctas / cg;
      if (cl < 1) cl = 1;
      const int64_t m_tiles = (d->M + 128 * cg - 1) / (128 * cg);
      auto cost = [&](int64_t n) {
        const int64_t waves = (m_tiles * ((d->N + n - 1) / n) + cl - 1) / cl;
        return waves * (n + 32);
      };
      if (cost(192) < cost(256)) bn = 192;
    }
  }
  if (bn < 32 * cg || bn > 256 || bn % (16 * cg) != 0 || bn % 32 != 0)
    return say_plan(msg, len, B2G_ERR_INVALID, "tile_n %d invalid for cta_group %d", bn, cg);
  if (d->m_sub < 0 || d->m_sub > 2) return say_plan(msg, len, B2G_ERR_INVALID, "m_sub must be 0, 1 or 2");
  // dense m_sub = 2 (512-row pair tiles, one accumulator): SS operands of the f16 and
  // f8f6f4 kinds, tile_n up to 256 (2 x 256 accumulator columns fill TMEM)
  const bool dense2 = var == GEMM_DENSE && !ts && !ws &&
                      (p->kind == KIND_F16 || p->kind == KIND_F8F6F4);
  if (d->m_sub == 2 && var == GEMM_DENSE && !dense2)
    return say_plan(msg, len, B2G_ERR_UNSUPPORTED,
                    "dense m_sub = 2 is built for SS f16 / f8f6f4 operands");
  // (sparse MX: one sub-tile unless asked; two leave TMEM for tile_n <= 192 only)
  int64_t cl2 = sm_count / cg;
  if (max_clusters > 0 && max_clusters < cl2) cl2 = max_clusters;
  if (d->max_ctas > 0 && d->max_ctas / cg < cl2) cl2 = d->max_ctas / cg;
  if (cl2 < 1) cl2 = 1;
  const int m_sub = d->m_sub ? d->m_sub
                    : (ws || var == GEMM_MXF8_SP || (var == GEMM_DENSE && !dense2)) ? 1
                             : gemm_default_m_sub(var, d->M, d->N, d->K, cg, bn,
                                                  var == GEMM_DENSE ? (int)cl2 : sm_count / cg);
  const int tmem = gemm_tmem_columns(bn, var, ts, m_sub, p->kind);
  if (tmem > 512)
    return say_plan(msg, len, B2G_ERR_INVALID,
                    "tile_n %d with m_sub %d needs %d TMEM columns, above 512 (the accumulators, "
                    "sparse metadata and scale factors)",
                    bn, m_sub, tmem);
  p->b_rows = bn / cg;
  int stages = d->stages;
  const int max_smem = 227 * 1024;
  // Two 128-byte K atoms per ring slot for dense SS tiles of up to kTwoAtomMaxN
  // columns, if the ring still holds at least 4 of the larger slots: their MMAs are
  // short, and the slot's fixed costs (barrier wait, fence, commit, expect_tx) then
  // fall on twice the MMAs.  Measured at 8192^3 bf16: 2-CTA 128-column tiles 872 ->
  // 1076 TFLOP/s (4 stages); one CTA of 128 x 128 (3 stages) lost 23 % instead.
  int ka = 1;
  if (var == GEMM_DENSE && !ts && !ws && m_sub == 1 && bn <= kTwoAtomMaxN) {
    int fit = 8;
    while (fit > 2 && gemm_smem_bytes(fit, p->b_rows, var, m_sub, 2, p->kind) > (size_t)max_smem) --fit;
    if (fit >= 4 && (stages == 0 || stages <= fit)) ka = 2;
  }
  if (stages == 0) {
    stages = 8;
    while (stages > 2 && gemm_smem_bytes(stages, p->b_rows, var, m_sub, ka, p->kind) > (size_t)max_smem)
      --stages;
  }
  if (stages < 2 || stages > 8) return say_plan(msg, len, B2G_ERR_INVALID, "stages must be in [2, 8]");
  p->smem = gemm_smem_bytes(stages, p->b_rows, var, m_sub, ka, p->kind);
  if (p->smem > (size_t)max_smem)
    return say_plan(msg, len, B2G_ERR_INVALID, "stages=%d does not fit shared memory (%zu bytes)",
                    stages, p->smem);
  if (d->raster_m < 0 || d->raster_m > 4096)
    return say_plan(msg, len, B2G_ERR_INVALID, "raster_m out of range");
  if (d->split_tail < 0 || d->split_tail > 4)
    return say_plan(msg, len, B2G_ERR_INVALID, "split_tail must be 0 (auto), 1 (off) or 2..4");

  // K extent of one ring slot: one 128-byte A atom (sparse: 64 compressed = 128
  // dense elements; unpacked fp4 / fp6: 128 elements in 16-byte chunks)
  const int elems_per_atom = p->unpack ? 128 : 128 * 8 / elem_bits;
  const int64_t k_per_slot = (sparse ? 2 : ka) * elems_per_atom;
  const int64_t k_blocks = (d->K + k_per_slot - 1) / k_per_slot;
  const int num_m_tiles = (int)((d->M + 128 * m_sub * cg - 1) / (128 * m_sub * cg));
  const int num_n_tiles = (int)((d->N + bn - 1) / bn);
  const int tiles = num_m_tiles * num_n_tiles;

  int clusters = sm_count / cg;
  if (max_clusters > 0 && max_clusters < clusters) clusters = max_clusters;
  if (d->max_ctas > 0 && d->max_ctas / cg < clusters) clusters = d->max_ctas / cg > 0 ? d->max_ctas / cg : 1;
  // Split tail: the tiles of the last, partial wave are cut into S K ranges on
  // otherwise idle clusters.  Every cluster of the persistent grid is resident
  // and takes at most one tail unit, so the finishing split's wait for the
  // others always ends (it is also bounded).  One accumulator buffer (m_sub = 2)
  // keeps whole tiles.
  int S = 1;
  const int rem = tiles % clusters;  // tiles of the last wave (all of them if tiles < clusters)
  // (an i8 tile is never split: its partial sums would be added in fp32, not s32)
  if (m_sub == 1 && d->split_tail != 1 && rem > 0 && p->kind != KIND_I8) {
    S = clusters / rem;
    if (S > 4) S = 4;
    if (d->split_tail >= 2 && d->split_tail < S) S = d->split_tail;
    if (S > k_blocks / 2) S = (int)(k_blocks / 2);
  }
  const int tail_start = S >= 2 ? tiles - rem : tiles;
  if (S < 2) S = 1;
  const int units = S > 1 ? tail_start + (tiles - tail_start) * S : tiles;
  if (clusters > units) clusters = units;

  b2g_gemm_plan& o = p->pub;
  o.variant = var;
  o.kind = p->kind;
  o.cta_group = cg;
  o.tile_m = 128 * m_sub * cg;
  o.tile_n = bn;
  o.m_sub = m_sub;
  o.stages = stages;
  o.smem_bytes = (int32_t)p->smem;
  o.tmem_columns = tmem;
  o.num_m_tiles = num_m_tiles;
  o.num_n_tiles = num_n_tiles;
  o.k_blocks = (int32_t)k_blocks;
  // Raster groups of tile rows sweep all of B once per group.  A wave of 74
  // clusters in groups of 8 tile rows touches the fewest distinct A and B bytes
  // at the BASELINE shapes (about 35 MB for e4m3 8192^3, against 45 MB with 4
  // rows), which is what sets the DRAM traffic; under the power cap the group
  // height does not change the throughput.
  o.raster_m = d->raster_m ? d->raster_m : 8;
  o.tail_start = tail_start;
  o.tail_split = S;
  o.units = units;
  o.clusters = clusters;
  o.threads = gemm_kernel_threads(m_sub);
  o.k_atoms = ka;
  o.instruction = ws ? 1 : 0;
  return B2G_OK;
}

b2g_status b2g_plan_gemm(const b2g_gemm_desc* d, int sm_count, int max_clusters,
                         b2g_gemm_plan* out, char* msg, int msg_len) {
  if (!d || !out) return B2G_ERR_INVALID;
  if (msg && msg_len > 0) msg[0] = 0;
  Plan p;
  const b2g_status st =
      plan_gemm(d, sm_count, max_clusters, &p, msg, msg_len > 0 ? (size_t)msg_len : 0);
  if (st == B2G_OK) *out = p.pub;
  return st;
}

b2g_status b2g_gemm(b2g_handle* h, const b2g_gemm_desc* d, void* stream) {
  if (!h || !d) return B2G_ERR_INVALID;
  h->last_error[0] = 0;
  Plan p;
  b2g_status st = plan_gemm(d, h->sm_count, 0, &p, h->last_error, sizeof(h->last_error));
  if (st != B2G_OK) return st;
  if (!d->A || !d->B || !d->C) return fail(h, B2G_ERR_INVALID, "null operand pointer");
  if ((reinterpret_cast<uintptr_t>(d->A) | reinterpret_cast<uintptr_t>(d->B)) & 15)
    return fail(h, B2G_ERR_INVALID, "A and B must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(d->C) & 1) return fail(h, B2G_ERR_INVALID, "C misaligned");
  if (p.sparse && (!d->meta || (reinterpret_cast<uintptr_t>(d->meta) & 15)))
    return fail(h, B2G_ERR_INVALID, "sparse: 16-byte aligned metadata needed");
  if (gemm_block_scaled(p.var) && (!d->sfa || !d->sfb))
    return fail(h, B2G_ERR_INVALID, "block-scaled formats: both scale-factor arrays needed");

  DeviceGuard g(h->device);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int cg = p.pub.cta_group, bn = p.pub.tile_n, m_sub = p.pub.m_sub, var = p.var;
  if (cg == 2) {  // co-resident cluster pairs under this shared-memory footprint
    int mc = 0;
    const uint32_t key = occ_key(p.kind, cg, var, p.ts, m_sub, p.pub.k_atoms, p.ws);
    int hit = -1;
    for (int i = 0; i < h->n_occ; ++i)
      if (h->occ[i].key == key && h->occ[i].smem == (int)p.smem) hit = i;
    if (hit >= 0) {
      mc = h->occ[hit].clusters;
    } else {
      B2G_CUDA(h, gemm_max_active_clusters(p.kind, cg, var, p.ts, m_sub, p.pub.k_atoms, p.ws,
                                           (int)p.smem, &mc));
      const int slot = h->n_occ < 16 ? h->n_occ++ : (int)(key % 16u);
      h->occ[slot] = {key, (int)p.smem, mc};
    }
    if (mc > 0 && mc < p.pub.clusters) {
      st = plan_gemm(d, h->sm_count, mc, &p, h->last_error, sizeof(h->last_error));
      if (st != B2G_OK) return st;
    }
  }
  const int elem_bits = p.elem_bits;
  auto row_bytes = [&](int64_t n) { return n * elem_bits / 8; };
  const int64_t k_blocks = p.pub.k_blocks;

  // tensor maps count elements, except for e2m1 that stays packed in shared memory
  // (NVFP4, MXF4), which they count in bytes; the unpacking maps (fp4 / fp6 of
  // f8f6f4) count elements, 128 per 128-byte shared-memory row
  const bool bytes_map = elem_bits == 4 && !p.unpack;
  const int tm_elems_per_atom = (bytes_map || p.unpack) ? 128 : 128 * 8 / elem_bits;
  const int64_t tm_a_cols = bytes_map ? p.a_cols / 2 : p.a_cols;
  const int64_t tm_k = bytes_map ? d->K / 2 : d->K;
  // B: its own element type when A and B mix kind::f8f6f4 types (never a bytes map)
  const int tm_b_elems_per_atom = p.b_elem_bits == elem_bits ? tm_elems_per_atom : 128;
  if ((p.unpack && (reinterpret_cast<uintptr_t>(d->A) & 31)) ||
      (p.b_unpack && (reinterpret_cast<uintptr_t>(d->B) & 31)))
    return fail(h, B2G_ERR_INVALID, "fp4 / fp6 (f8f6f4): A and B must be 32-byte aligned");
  GemmMaps maps;
  memset(&maps, 0, sizeof(maps));
  st = make_tmap_2d(h, &maps.a, p.dt, d->A, (uint64_t)tm_a_cols, (uint64_t)d->M,
                    (uint64_t)row_bytes(d->lda), (uint32_t)tm_elems_per_atom, 128,
                    CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != B2G_OK) return st;
  st = make_tmap_2d(h, &maps.b, p.b_dt, d->B, (uint64_t)tm_k, (uint64_t)d->N,
                    (uint64_t)(d->ldb * p.b_elem_bits / 8), (uint32_t)tm_b_elems_per_atom,
                    (uint32_t)p.b_rows, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != B2G_OK) return st;
  if (p.sparse) {  // (2:4 metadata: map e)
    // metadata layout of the element width in shared memory (fp4 / fp6 unpacked: 8)
    const bool pairs = var == GEMM_MXF4_SP || var == GEMM_NVFP4_SP;
    const int meta_bits = (p.unpack || pairs) ? 8 : elem_bits;
    // metadata describes bytes for sparse MXFP4 / NVFP4 (a pair of e2m1 per byte)
    const int64_t meta_k = pairs ? d->K / 2 : d->K;
    const void* ready = d->meta;
    if (d->meta_layout == 0) {
      const size_t need = meta_ready_bytes(d->M, meta_k, meta_bits);
      if (h->meta_ws_bytes < need) {
        B2G_CUDA(h, cudaStreamSynchronize(s));
        if (h->meta_ws) cudaFree(h->meta_ws);
        h->meta_ws = nullptr;
        h->meta_ws_bytes = 0;
        B2G_CUDA(h, cudaMalloc(&h->meta_ws, need));
        h->meta_ws_bytes = need;
      }
      B2G_CUDA(h, launch_meta_ready((const uint32_t*)d->meta, d->M, meta_k, (uint32_t*)h->meta_ws,
                                    h->sm_count, s, meta_bits));
      ready = h->meta_ws;
    }
    // one box per ring slot and 128-row block: 2 KB (16-bit A) or 4 KB (8-bit), in
    // kSideLine-byte lines
    const uint32_t box_lines = (meta_bits == 8 ? 4096 : 2048) / kSideLine;
    const uint64_t lines_total = (uint64_t)((d->M + 127) / 128) * (uint64_t)k_blocks * box_lines;
    st = make_tmap_2d(h, &maps.e, CU_TENSOR_MAP_DATA_TYPE_UINT8, ready, kSideLine, lines_total,
                      kSideLine, kSideLine, box_lines, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st != B2G_OK) return st;
  }
  if (gemm_block_scaled(var)) {
    // scale factors -> engine blocks in the handle's scratch (SFA per 128 rows,
    // SFB per tile_n rows padded to 256), `groups` 4-byte groups per ring slot
    // the same (groups, block_rows, padded_rows) as the launches below: the sizes must agree
    const int groups = gemm_sf_groups(var);
    // one scale per 16 (NVFP4), 64 (2:4-sparse MX: one per sparse MMA) or 32 K
    const int64_t sf_cols = var == GEMM_NVFP4                                ? d->K / 16
                            : (var == GEMM_MXF8_SP || var == GEMM_MXF4_SP) ? d->K / 64
                                                                           : d->K / 32;
    // (NVFP4_SP: one ue4m3 per 32 dense K, the last case)
    const size_t na = sf_ready_bytes(d->M, sf_cols, groups, 128, 128);
    const size_t nb = sf_ready_bytes(d->N, sf_cols, groups, bn, 256);
    const size_t need = na + nb;
    if (h->sf_ws_bytes < need) {
      B2G_CUDA(h, cudaStreamSynchronize(s));
      if (h->sf_ws) cudaFree(h->sf_ws);
      h->sf_ws = nullptr;
      h->sf_ws_bytes = 0;
      B2G_CUDA(h, cudaMalloc(&h->sf_ws, need));
      h->sf_ws_bytes = need;
    }
    uint8_t* ra = static_cast<uint8_t*>(h->sf_ws);
    uint8_t* rb = ra + na;
    B2G_CUDA(h, launch_sf_ready((const uint8_t*)d->sfa, d->M, sf_cols, groups, 128, 128, ra,
                                h->sm_count, s));
    B2G_CUDA(h, launch_sf_ready((const uint8_t*)d->sfb, d->N, sf_cols, groups, bn, 256, rb,
                                h->sm_count, s));
    // one ring slot: 512 x groups bytes of SFA, 1024 x groups of SFB, in kSideLine
    // lines; maps e, f (or f, g after a sparse A's metadata)
    CUtensorMap* map_sfa = p.sparse ? &maps.f : &maps.e;
    CUtensorMap* map_sfb = p.sparse ? &maps.g : &maps.f;
    st = make_tmap_2d(h, map_sfa, CU_TENSOR_MAP_DATA_TYPE_UINT8, ra, kSideLine, na / kSideLine,
                      kSideLine, kSideLine, (uint32_t)(512 * groups / kSideLine),
                      CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st != B2G_OK) return st;
    st = make_tmap_2d(h, map_sfb, CU_TENSOR_MAP_DATA_TYPE_UINT8, rb, kSideLine, nb / kSideLine,
                      kSideLine, kSideLine, (uint32_t)(1024 * groups / kSideLine),
                      CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st != B2G_OK) return st;
  }

  GemmArgs a;
  memset(&a, 0, sizeof(a));
  a.M = (int)d->M;
  a.N = (int)d->N;
  a.num_m_tiles = p.pub.num_m_tiles;
  a.num_n_tiles = p.pub.num_n_tiles;
  a.k_blocks = (int)k_blocks;
  a.tile_n = bn;
  a.stages = p.pub.stages;
  a.group_m = p.pub.raster_m;
  // the kernel's K units per ring slot: 128 for every 8-bit shared-memory layout
  a.elem_bits = p.unpack ? 8 : elem_bits;
  a.tx_a_bits = p.unpack ? elem_bits : 0;
  a.tx_b_bits = p.b_unpack ? p.b_elem_bits : 0;
  // scale type: ue4m3 (NVFP4) or E8M0 (MX formats)
  a.idesc = encode_idesc(p.kind, p.a_type, p.b_type, 128 * cg, bn, p.sparse ? 1 : 0,
                         var == GEMM_MXF8 || var == GEMM_MXF4 || var == GEMM_MXF8_SP ||
                                 var == GEMM_MXF4_SP
                             ? 1
                             : 0);
  a.alpha = d->alpha;
  a.C = reinterpret_cast<__nv_bfloat16*>(d->C);
  a.ldc = d->ldc;
  a.c_vec_ok = ((reinterpret_cast<uintptr_t>(d->C) & 15) == 0 && (d->ldc % 8) == 0) ? 1 : 0;
  a.err = h->d_err;
  a.trace = h->trace_dev;
  a.wait_ns = h->wait_ns;
  a.tail_start = p.pub.tail_start;
  a.tail_split = p.pub.tail_split;
  if (p.pub.tail_split >= 2) {
    const int tiles = p.pub.num_m_tiles * p.pub.num_n_tiles, S = p.pub.tail_split;
    const int rem = tiles - p.pub.tail_start;
    const size_t part_need = (size_t)rem * (S - 1) * (size_t)(128 * cg) * (size_t)bn * sizeof(float);
    const size_t flag_need = (size_t)rem * (S - 1) * cg * 4 * sizeof(uint32_t);
    if (h->part_ws_bytes < part_need || h->flag_ws_bytes < flag_need) {
      B2G_CUDA(h, cudaStreamSynchronize(s));
      if (h->part_ws_bytes < part_need) {
        if (h->part_ws) cudaFree(h->part_ws);
        h->part_ws = nullptr;
        h->part_ws_bytes = 0;
        B2G_CUDA(h, cudaMalloc(&h->part_ws, part_need));
        h->part_ws_bytes = part_need;
      }
      if (h->flag_ws_bytes < flag_need) {
        if (h->flag_ws) cudaFree(h->flag_ws);
        h->flag_ws = nullptr;
        h->flag_ws_bytes = 0;
        B2G_CUDA(h, cudaMalloc(&h->flag_ws, flag_need));
        B2G_CUDA(h, cudaMemset(h->flag_ws, 0, flag_need));
        h->flag_ws_bytes = flag_need;
      }
    }
    if (++h->epoch == 0) ++h->epoch;  // 0 is the value of fresh flags
    a.part = static_cast<float*>(h->part_ws);
    a.flags = h->flag_ws;
    a.epoch = h->epoch;
  }
  const int clusters = p.pub.clusters;
  if (h->trace_dev && clusters * cg > h->trace_ctas) a.trace = nullptr;  // buffer too small
  B2G_CUDA(h, gemm_launch(p.kind, cg, var, p.ts, m_sub, p.pub.k_atoms, p.ws, maps, a,
                          clusters * cg, p.smem, s));
  return B2G_OK;
}

size_t b2g_sparse_meta_bytes(int64_t M, int64_t K) {
  return (M > 0 && K > 0) ? meta_ready_bytes(M, K) : 0;
}

// Stored bits of one A element of the 2:4-sparse GEMM's formats (0: not sparse-capable).
static int sparse_elem_bits(int format) {
  switch (format) {
    case B2G_FMT_BF16:
    case B2G_FMT_F16: return 16;
    case B2G_FMT_E4M3:
    case B2G_FMT_E5M2:
    case B2G_FMT_MXF8:  // MX e4m3 codes: the 8-bit forms (scales are not touched)
    case B2G_FMT_S8:
    case B2G_FMT_U8: return 8;
    case B2G_FMT_E2M1: return 4;  // packed fp4 / fp6 of kind::f8f6f4 (2:4 on elements)
    case B2G_FMT_E2M3:
    case B2G_FMT_E3M2: return 6;
    case B2G_FMT_TF32: return 32;  // structured 1:2 (pairs read as four 16-bit halves)
    default: return 0;
  }
}

// Element width whose TMEM metadata layout a sparse format uses: the fp4 / fp6
// codes are unpacked to one byte each in shared memory, so theirs is the 8-bit one.
static int sparse_meta_bits(int format) {
  const int bits = sparse_elem_bits(format);
  return (bits == 4 || bits == 6) ? 8 : bits;
}

size_t b2g_sparse_meta_bytes_format(int format, int64_t M, int64_t K) {
  if (format == B2G_FMT_MXF4 || format == B2G_FMT_NVFP4)  // pairs of packed e2m1: the 8-bit
                                                           // layout over K / 2 bytes
    return (M > 0 && K > 0) ? meta_ready_bytes(M, K / 2, 8) : 0;
  const int bits = sparse_meta_bits(format);
  return (bits && M > 0 && K > 0) ? meta_ready_bytes(M, K, bits) : 0;
}

b2g_status b2g_sparse_meta_prepare(b2g_handle* h, const void* d_meta, int64_t M, int64_t K,
                                   void* d_ready, void* stream) {
  return b2g_sparse_meta_prepare_format(h, B2G_FMT_BF16, d_meta, M, K, d_ready, stream);
}

b2g_status b2g_sparse_meta_prepare_format(b2g_handle* h, int format, const void* d_meta, int64_t M,
                                          int64_t K, void* d_ready, void* stream) {
  if (!h) return B2G_ERR_INVALID;
  if (format == B2G_FMT_MXF4 || format == B2G_FMT_NVFP4) {  // pairs of packed e2m1:
                                                             // canonical [M][K/64] words
    if (!d_meta || !d_ready || M <= 0 || K <= 0 || K % 64 ||
        (reinterpret_cast<uintptr_t>(d_meta) & 3) || (reinterpret_cast<uintptr_t>(d_ready) & 15))
      return fail(h, B2G_ERR_INVALID,
                  "b2g_sparse_meta_prepare (MXFP4): K %% 64 == 0 and aligned buffers needed");
    DeviceGuard g(h->device);
    B2G_CUDA(h, launch_meta_ready((const uint32_t*)d_meta, M, K / 2, (uint32_t*)d_ready,
                                  h->sm_count, reinterpret_cast<cudaStream_t>(stream), 8));
    return B2G_OK;
  }
  const int bits = sparse_meta_bits(format);
  if (!bits) return fail(h, B2G_ERR_UNSUPPORTED, "b2g_sparse_meta_prepare: format %d", format);
  // one canonical metadata word covers 32 dense K (16 for tf32, whose pairs are
  // described as groups of four 16-bit halves)
  const int64_t k_word = bits == 32 ? 16 : 32;
  if (!d_meta || !d_ready || M <= 0 || K <= 0 || K % k_word ||
      (reinterpret_cast<uintptr_t>(d_meta) & 3) || (reinterpret_cast<uintptr_t>(d_ready) & 15))
    return fail(h, B2G_ERR_INVALID,
                "b2g_sparse_meta_prepare: K %% %d == 0 and aligned buffers needed", (int)k_word);
  DeviceGuard g(h->device);
  B2G_CUDA(h, launch_meta_ready((const uint32_t*)d_meta, M, K, (uint32_t*)d_ready, h->sm_count,
                                reinterpret_cast<cudaStream_t>(stream), bits));
  return B2G_OK;
}

// ------------------------------------------------------------------ host-buffer GEMM
static size_t align_up_sz(size_t x, size_t a) { return (x + a - 1) / a * a; }

static b2g_status host_pipe_init(b2g_handle* h) {
  if (h->pipe_ready) return B2G_OK;
  B2G_CUDA(h, cudaStreamCreateWithFlags(&h->s_in, cudaStreamNonBlocking));
  B2G_CUDA(h, cudaStreamCreateWithFlags(&h->s_out, cudaStreamNonBlocking));
  B2G_CUDA(h, cudaEventCreateWithFlags(&h->ev_start, cudaEventDisableTiming));
  B2G_CUDA(h, cudaEventCreateWithFlags(&h->ev_out, cudaEventDisableTiming));
  B2G_CUDA(h, cudaEventCreateWithFlags(&h->ev_c, cudaEventDisableTiming));
  for (int i = 0; i < kHostChunks; ++i)
    B2G_CUDA(h, cudaEventCreateWithFlags(&h->ev_a[i], cudaEventDisableTiming));
  for (int j = 0; j < kHostColChunks; ++j)
    B2G_CUDA(h, cudaEventCreateWithFlags(&h->ev_b[j], cudaEventDisableTiming));
  h->pipe_ready = true;
  return B2G_OK;
}

// End to end on host buffers, pipelined over blocks of C: B is cut into up to
// kHostColChunks column chunks (with their scale factors) and A into up to
// kHostChunks row chunks of whole 512-row multiples (with their metadata or scale
// factors).  The copy-in stream carries the chunks with the B
// chunks spread among the A chunks; block (i, j) of C is computed on the
// caller's stream as soon as A_i and B_j are in, and copied out (2D) on a
// copy-out stream as soon as it is done.  The copy engines run both directions at once and the first
// block leaves after a few MB have arrived, so the PCIe time is about the larger
// of the two directions.  Every block computes whole tiles in the same K order as
// one b2g_gemm over the whole problem (unless split_tail asks for splits), so C
// is the same.
b2g_status b2g_gemm_host(b2g_handle* h, const b2g_gemm_desc* d, void* stream) {
  if (!h || !d) return B2G_ERR_INVALID;
  if (!d->A || !d->B || !d->C || d->M <= 0 || d->N <= 0 || d->K <= 0)
    return fail(h, B2G_ERR_INVALID, "b2g_gemm_host: null pointer or empty problem");
  // stored bits per element of A and of B
  auto bits_of = [](int f) -> size_t {
    switch (f) {
      case B2G_FMT_TF32: return 32;
      case B2G_FMT_BF16:
      case B2G_FMT_F16: return 16;
      case B2G_FMT_NVFP4:
      case B2G_FMT_E2M1:
      case B2G_FMT_MXF4: return 4;
      case B2G_FMT_E2M3:
      case B2G_FMT_E3M2: return 6;
      default: return 8;
    }
  };
  const size_t a_row = (size_t)d->lda * bits_of(d->format) / 8;  // bytes per stored row
  const size_t b_row = (size_t)d->ldb * bits_of(d->b_format ? d->b_format : d->format) / 8;
  const size_t c_row = (size_t)d->ldc * 2;
  // scale bytes per row: per 16 K (NVFP4), 64 K (2:4-sparse MX) or 32 K
  const bool sparse_mx = d->sparse && (d->mx_scale || d->format == B2G_FMT_MXF8 ||
                                       d->format == B2G_FMT_MXF4);
  const size_t sf_row = (size_t)(d->format == B2G_FMT_NVFP4 ? (d->sparse ? d->K / 32 : d->K / 16)
                                 : sparse_mx                ? d->K / 64
                                                            : d->K / 32);
  // engine-layout metadata of one 128-row block (meta_layout 1): every K slot's block
  // (sparse MXFP4: the metadata describes the K / 2 bytes of packed e2m1 pairs)
  const bool pairs = d->sparse && (d->format == B2G_FMT_MXF4 || d->format == B2G_FMT_NVFP4);
  const int meta_bits = pairs ? 8
                        : (d->sparse && sparse_meta_bits(d->format)) ? sparse_meta_bits(d->format)
                                                                       : 16;
  const int64_t meta_k = pairs ? d->K / 2 : d->K;
  const size_t meta_rowblock = meta_ready_bytes(128, meta_k, meta_bits);
  const bool meta_ready_layout = d->meta_layout == 1;
  // canonical metadata bytes per row: [K/32] words, [K/16] for tf32's pairs, [K/64]
  // for MXFP4's byte pairs
  const size_t meta_row = (size_t)(d->K / (d->format == B2G_FMT_TF32 ? 16 : pairs ? 64 : 32)) * 4;
  const size_t a_bytes = (size_t)d->M * a_row;
  const size_t b_bytes = (size_t)d->N * b_row;
  const size_t c_bytes = (size_t)d->M * c_row;
  const size_t sfa_bytes = d->sfa ? (size_t)d->M * sf_row : 0;
  const size_t sfb_bytes = d->sfb ? (size_t)d->N * sf_row : 0;
  const size_t meta_bytes = !d->meta ? 0
                            : meta_ready_layout ? meta_ready_bytes(d->M, meta_k, meta_bits)
                                                : (size_t)d->M * meta_row;
  const size_t o_a = 0, o_b = align_up_sz(o_a + a_bytes, 256), o_c = align_up_sz(o_b + b_bytes, 256),
               o_sa = align_up_sz(o_c + c_bytes, 256), o_sb = align_up_sz(o_sa + sfa_bytes, 256),
               o_m = align_up_sz(o_sb + sfb_bytes, 256), total = align_up_sz(o_m + meta_bytes, 256);
  DeviceGuard g(h->device);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (h->ws_bytes < total) {
    B2G_CUDA(h, cudaStreamSynchronize(s));
    if (h->ws) cudaFree(h->ws);
    h->ws = nullptr;
    h->ws_bytes = 0;
    B2G_CUDA(h, cudaMalloc(&h->ws, total));
    h->ws_bytes = total;
  }
  b2g_status st = host_pipe_init(h);
  if (st != B2G_OK) return st;
  uint8_t* w = static_cast<uint8_t*>(h->ws);
  const uint8_t* hA = static_cast<const uint8_t*>(d->A);
  const uint8_t* hB = static_cast<const uint8_t*>(d->B);
  const uint8_t* hSA = static_cast<const uint8_t*>(d->sfa);
  const uint8_t* hSB = static_cast<const uint8_t*>(d->sfb);
  const uint8_t* hM = static_cast<const uint8_t*>(d->meta);
  uint8_t* hC = static_cast<uint8_t*>(d->C);

  // row chunks: multiples of 512 rows; column chunks: multiples of 256 columns
  // (whole tile rows and columns for every tile shape)
  int64_t rch = (d->M + kHostChunks - 1) / kHostChunks;
  rch = (rch + 511) / 512 * 512;
  const int na = (int)((d->M + rch - 1) / rch);
  int64_t cch = (d->N + kHostColChunks - 1) / kHostColChunks;
  cch = (cch + 255) / 256 * 256;
  const int nb = (int)((d->N + cch - 1) / cch);
  auto rows_of = [&](int i) { return (d->M - i * rch < rch) ? d->M - i * rch : rch; };
  auto cols_of = [&](int j) { return (d->N - j * cch < cch) ? d->N - j * cch : cch; };

  // the side streams start after the work already queued on the caller's stream
  B2G_CUDA(h, cudaEventRecord(h->ev_start, s));
  B2G_CUDA(h, cudaStreamWaitEvent(h->s_in, h->ev_start, 0));
  B2G_CUDA(h, cudaStreamWaitEvent(h->s_out, h->ev_start, 0));
  auto copy_b = [&](int j) -> b2g_status {
    const int64_t c0 = j * cch, cols = cols_of(j);
    B2G_CUDA(h, cudaMemcpyAsync(w + o_b + c0 * b_row, hB + c0 * b_row, cols * b_row,
                                cudaMemcpyHostToDevice, h->s_in));
    if (sfb_bytes)
      B2G_CUDA(h, cudaMemcpyAsync(w + o_sb + c0 * sf_row, hSB + c0 * sf_row, cols * sf_row,
                                  cudaMemcpyHostToDevice, h->s_in));
    B2G_CUDA(h, cudaEventRecord(h->ev_b[j], h->s_in));
    return B2G_OK;
  };
  auto meta_span = [&](int i, size_t* off, size_t* len) {
    const int64_t r0 = i * rch, rows = rows_of(i);
    if (meta_ready_layout) {  // [128-row block][K slot][metadata block]
      *off = (size_t)(r0 / 128) * meta_rowblock;
      *len = (size_t)((rows + 127) / 128) * meta_rowblock;
    } else {
      *off = (size_t)r0 * meta_row;
      *len = (size_t)rows * meta_row;
    }
  };
  auto copy_a = [&](int i) -> b2g_status {
    const int64_t r0 = i * rch, rows = rows_of(i);
    B2G_CUDA(h, cudaMemcpyAsync(w + o_a + r0 * a_row, hA + r0 * a_row, rows * a_row,
                                cudaMemcpyHostToDevice, h->s_in));
    if (sfa_bytes)
      B2G_CUDA(h, cudaMemcpyAsync(w + o_sa + r0 * sf_row, hSA + r0 * sf_row, rows * sf_row,
                                  cudaMemcpyHostToDevice, h->s_in));
    if (meta_bytes) {
      size_t off, len;
      meta_span(i, &off, &len);
      B2G_CUDA(h, cudaMemcpyAsync(w + o_m + off, hM + off, len, cudaMemcpyHostToDevice, h->s_in));
    }
    B2G_CUDA(h, cudaEventRecord(h->ev_a[i], h->s_in));
    return B2G_OK;
  };
  // Input order: the B chunks spread evenly among the A chunks (B_0 first), so
  // that the blocks of C become ready at a steady rate; each arrival unlocks the
  // blocks it forms with the chunks of the other operand already in.
  int order[kHostChunks + kHostColChunks];  // >= 0: A chunk, < 0: B chunk -1 - j
  int n_in = 0;
  for (int i = 0, j = 0; i < na || j < nb;) {
    if (j < nb && (i == na || (int64_t)j * na <= (int64_t)i * nb)) order[n_in++] = -1 - j++;
    else order[n_in++] = i++;
  }
  for (int q = 0; q < n_in; ++q)
    if ((st = order[q] >= 0 ? copy_a(order[q]) : copy_b(-1 - order[q])) != B2G_OK) return st;

  int a_in = 0, b_in = 0;  // chunks arrived so far, in order
  for (int q = 0; q < n_in; ++q) {
    const bool is_a = order[q] >= 0;
    B2G_CUDA(h, cudaStreamWaitEvent(s, is_a ? h->ev_a[order[q]] : h->ev_b[-1 - order[q]], 0));
    const int i_lo = is_a ? order[q] : 0, i_hi = is_a ? order[q] + 1 : a_in;
    const int j_lo = is_a ? 0 : -1 - order[q], j_hi = is_a ? b_in : -order[q];
    if (is_a) ++a_in; else ++b_in;
    for (int j = j_lo; j < j_hi; ++j)
    for (int i = i_lo; i < i_hi; ++i) {
      const int64_t c0 = j * cch, cols = cols_of(j);
      const int64_t r0 = i * rch, rows = rows_of(i);
      b2g_gemm_desc dd = *d;
      dd.M = rows;
      dd.N = cols;
      dd.A = w + o_a + r0 * a_row;
      dd.B = w + o_b + c0 * b_row;
      dd.C = w + o_c + r0 * c_row + c0 * 2;
      dd.sfa = sfa_bytes ? w + o_sa + r0 * sf_row : nullptr;
      dd.sfb = sfb_bytes ? w + o_sb + c0 * sf_row : nullptr;
      if (meta_bytes) {
        size_t off, len;
        meta_span(i, &off, &len);
        dd.meta = w + o_m + off;
      }
      if (dd.split_tail == 0) dd.split_tail = 1;
      if (dd.cta_group == 0) dd.cta_group = d->M >= 256 ? 2 : 1;
      st = b2g_gemm(h, &dd, stream);
      if (st != B2G_OK) return st;
      B2G_CUDA(h, cudaEventRecord(h->ev_c, s));
      B2G_CUDA(h, cudaStreamWaitEvent(h->s_out, h->ev_c, 0));
      B2G_CUDA(h, cudaMemcpy2DAsync(hC + r0 * c_row + c0 * 2, c_row, w + o_c + r0 * c_row + c0 * 2,
                                    c_row, (size_t)cols * 2, (size_t)rows,
                                    cudaMemcpyDeviceToHost, h->s_out));
    }
  }
  B2G_CUDA(h, cudaEventRecord(h->ev_out, h->s_out));
  B2G_CUDA(h, cudaStreamWaitEvent(s, h->ev_out, 0));
  return b2g_check(h, stream);
}

// ------------------------------------------------------------------ data generation
b2g_status b2g_fill_f32(b2g_handle* h, float* d_out, int64_t rows, int64_t cols, int64_t row0,
                        uint64_t seed, int dist, void* stream) {
  if (!h || !d_out || rows < 0 || cols < 0 || row0 < 0 || (dist != 0 && dist != 1))
    return fail(h, B2G_ERR_INVALID, "b2g_fill_f32: bad arguments");
  if (rows * cols == 0) return B2G_OK;
  DeviceGuard g(h->device);
  B2G_CUDA(h, launch_fill_f32(d_out, rows, cols, row0, seed, dist, h->sm_count,
                              reinterpret_cast<cudaStream_t>(stream)));
  return B2G_OK;
}

b2g_status b2g_quantize(b2g_handle* h, int format, const float* d_in, int64_t rows, int64_t cols,
                        void* d_out, void* d_sf, void* stream) {
  if (!h || !d_in || !d_out || rows < 0 || cols < 0)
    return fail(h, B2G_ERR_INVALID, "b2g_quantize: bad arguments");
  if (rows * cols == 0) return B2G_OK;
  DeviceGuard g(h->device);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (format) {
    case B2G_FMT_BF16:
      B2G_CUDA(h, launch_quant_bf16(d_in, rows * cols, (uint16_t*)d_out, h->sm_count, s));
      return B2G_OK;
    case B2G_FMT_E4M3:
      if (reinterpret_cast<uintptr_t>(d_in) & 7)
        return fail(h, B2G_ERR_INVALID, "e4m3 quantiser needs 8-byte aligned input");
      B2G_CUDA(h, launch_quant_e4m3(d_in, rows * cols, (uint8_t*)d_out, h->sm_count, s));
      return B2G_OK;
    case B2G_FMT_E2M1:
    case B2G_FMT_E2M3:
    case B2G_FMT_E3M2:
      if (cols % 16 || (reinterpret_cast<uintptr_t>(d_in) & 15) ||
          (reinterpret_cast<uintptr_t>(d_out) & 7))
        return fail(h, B2G_ERR_INVALID, "fp4 / fp6 quantiser: cols %% 16 and aligned buffers needed");
      B2G_CUDA(h, launch_quant_sub(format == B2G_FMT_E2M1 ? 0 : (format == B2G_FMT_E2M3 ? 1 : 2),
                                   d_in, rows * cols, (uint8_t*)d_out, h->sm_count, s));
      return B2G_OK;
    case B2G_FMT_S8:
    case B2G_FMT_TF32:
    case B2G_FMT_E5M2:
    case B2G_FMT_U8:
    case B2G_FMT_F16:
      B2G_CUDA(h, launch_quant_elem(format == B2G_FMT_S8     ? 0
                                    : format == B2G_FMT_TF32 ? 1
                                    : format == B2G_FMT_E5M2 ? 2
                                    : format == B2G_FMT_U8   ? 3
                                                             : 4,
                                    d_in, rows * cols, d_out, h->sm_count, s));
      return B2G_OK;
    case B2G_FMT_MXF8:
    case B2G_FMT_MXF4:
      if (!d_sf || cols % 32 || (reinterpret_cast<uintptr_t>(d_in) & 15) ||
          (reinterpret_cast<uintptr_t>(d_out) & 15))
        return fail(h, B2G_ERR_INVALID, "MX quantiser: cols %% 32, 16-byte aligned buffers and sf needed");
      B2G_CUDA(h, launch_quant_mx(d_in, rows, cols, format == B2G_FMT_MXF8 ? 0 : 1,
                                  (uint8_t*)d_out, (uint8_t*)d_sf, h->sm_count, s));
      return B2G_OK;
    case B2G_FMT_NVFP4:
      if (!d_sf || cols % 16 || (reinterpret_cast<uintptr_t>(d_in) & 15) ||
          (reinterpret_cast<uintptr_t>(d_out) & 7))
        return fail(h, B2G_ERR_INVALID, "nvfp4 quantiser: cols %% 16, aligned buffers and sf needed");
      B2G_CUDA(h, launch_quant_nvfp4(d_in, rows, cols, (uint8_t*)d_out, (uint8_t*)d_sf,
                                     h->sm_count, s));
      return B2G_OK;
    default:
      return fail(h, B2G_ERR_UNSUPPORTED, "b2g_quantize: format %d", format);
  }
}

b2g_status b2g_quantize_mx(b2g_handle* h, int elem_format, const float* d_in, int64_t rows,
                           int64_t cols, void* d_out, void* d_sf, void* stream) {
  return b2g_quantize_mx_block(h, elem_format, d_in, rows, cols, 32, d_out, d_sf, stream);
}

b2g_status b2g_quantize_mx_block(b2g_handle* h, int elem_format, const float* d_in, int64_t rows,
                                 int64_t cols, int block, void* d_out, void* d_sf, void* stream) {
  if (!h) return B2G_ERR_INVALID;
  if (block != 32 && block != 64)
    return fail(h, B2G_ERR_INVALID, "b2g_quantize_mx: block must be 32 or 64");
  if (!d_in || !d_out || !d_sf || rows < 0 || cols < 0 || cols % block ||
      (reinterpret_cast<uintptr_t>(d_in) & 15) || (reinterpret_cast<uintptr_t>(d_out) & 15))
    return fail(h, B2G_ERR_INVALID,
                "b2g_quantize_mx: cols %% block, 16-byte aligned buffers and sf needed");
  int elem;
  switch (elem_format) {
    case B2G_FMT_E4M3: elem = 0; break;
    case B2G_FMT_E2M1: elem = 1; break;
    case B2G_FMT_E5M2: elem = 2; break;
    case B2G_FMT_E2M3: elem = 3; break;
    case B2G_FMT_E3M2: elem = 4; break;
    default: return fail(h, B2G_ERR_UNSUPPORTED, "b2g_quantize_mx: format %d", elem_format);
  }
  if (rows * cols == 0) return B2G_OK;
  DeviceGuard g(h->device);
  B2G_CUDA(h, launch_quant_mx(d_in, rows, cols, elem, (uint8_t*)d_out, (uint8_t*)d_sf,
                              h->sm_count, reinterpret_cast<cudaStream_t>(stream), block));
  return B2G_OK;
}

b2g_status b2g_quantize_nvfp4_block(b2g_handle* h, const float* d_in, int64_t rows, int64_t cols,
                                    int block, void* d_out, void* d_sf, void* stream) {
  if (!h) return B2G_ERR_INVALID;
  if (block != 16 && block != 32)
    return fail(h, B2G_ERR_INVALID, "b2g_quantize_nvfp4_block: block must be 16 or 32");
  if (!d_in || !d_out || !d_sf || rows < 0 || cols < 0 || cols % block ||
      (reinterpret_cast<uintptr_t>(d_in) & 15) || (reinterpret_cast<uintptr_t>(d_out) & 7))
    return fail(h, B2G_ERR_INVALID,
                "b2g_quantize_nvfp4_block: cols %% block, aligned buffers and sf needed");
  if (rows * cols == 0) return B2G_OK;
  DeviceGuard g(h->device);
  B2G_CUDA(h, launch_quant_nvfp4(d_in, rows, cols, (uint8_t*)d_out, (uint8_t*)d_sf, h->sm_count,
                                 reinterpret_cast<cudaStream_t>(stream), block));
  return B2G_OK;
}

b2g_status b2g_prune_24(b2g_handle* h, void* d_bf16, int64_t rows, int64_t cols, int64_t row0,
                        uint64_t seed, void* stream) {
  if (!h || !d_bf16 || rows < 0 || cols < 0 || row0 < 0 || cols % 4 ||
      (reinterpret_cast<uintptr_t>(d_bf16) & 7))
    return fail(h, B2G_ERR_INVALID, "b2g_prune_24: cols %% 4 == 0 and 8-byte alignment needed");
  if (rows * cols == 0) return B2G_OK;
  DeviceGuard g(h->device);
  B2G_CUDA(h, launch_prune_24((uint16_t*)d_bf16, rows, cols, row0, seed, h->sm_count,
                              reinterpret_cast<cudaStream_t>(stream)));
  return B2G_OK;
}

b2g_status b2g_compress_24(b2g_handle* h, const void* d_dense, int64_t M, int64_t K, void* d_comp,
                           void* d_meta, void* stream) {
  if (!h || !d_dense || !d_comp || !d_meta || M < 0 || K < 0 || K % 32 ||
      ((reinterpret_cast<uintptr_t>(d_dense) | reinterpret_cast<uintptr_t>(d_comp)) & 15) ||
      (reinterpret_cast<uintptr_t>(d_meta) & 3))
    return fail(h, B2G_ERR_INVALID, "b2g_compress_24: K %% 32 == 0 and 16-byte alignment needed");
  if (M * K == 0) return B2G_OK;
  DeviceGuard g(h->device);
  B2G_CUDA(h, launch_compress_24((const uint16_t*)d_dense, M, K, (uint16_t*)d_comp,
                                 (uint32_t*)d_meta, h->d_err, h->sm_count,
                                 reinterpret_cast<cudaStream_t>(stream)));
  return B2G_OK;
}

b2g_status b2g_compress_24_format(b2g_handle* h, int format, const void* d_dense, int64_t M,
                                  int64_t K, void* d_comp, void* d_meta, void* stream) {
  if (!h) return B2G_ERR_INVALID;
  if (format == B2G_FMT_MXF4 || format == B2G_FMT_NVFP4) {
    // 4:8 in pairs of packed e2m1 (kind::mxf4 / mxf4nvf4 .sp): 2:4 on the bytes, a byte
    // being a pair, zero when both of its elements are (either sign); K counts elements
    if (!d_dense || !d_comp || !d_meta || M < 0 || K < 0 || K % 64 ||
        ((reinterpret_cast<uintptr_t>(d_dense) | reinterpret_cast<uintptr_t>(d_comp)) & 15) ||
        (reinterpret_cast<uintptr_t>(d_meta) & 3))
      return fail(h, B2G_ERR_INVALID,
                  "b2g_compress_24_format (MXFP4): K %% 64 == 0 and 16-byte alignment needed");
    if (M * K == 0) return B2G_OK;
    DeviceGuard g(h->device);
    B2G_CUDA(h, launch_compress_24_u8((const uint8_t*)d_dense, M, K / 2, 0x77u, (uint8_t*)d_comp,
                                      (uint32_t*)d_meta, h->d_err, h->sm_count,
                                      reinterpret_cast<cudaStream_t>(stream)));
    return B2G_OK;
  }
  const int bits = sparse_elem_bits(format);
  if (!bits) return fail(h, B2G_ERR_UNSUPPORTED, "b2g_compress_24_format: format %d", format);
  if (bits == 16) return b2g_compress_24(h, d_dense, M, K, d_comp, d_meta, stream);
  if (bits == 4 || bits == 6) {  // packed fp4 / fp6 codes in, packed kept codes out
    if (!d_dense || !d_comp || !d_meta || M < 0 || K < 0 || K % 32 ||
        ((reinterpret_cast<uintptr_t>(d_dense) | reinterpret_cast<uintptr_t>(d_comp)) & 15) ||
        (reinterpret_cast<uintptr_t>(d_meta) & 3))
      return fail(h, B2G_ERR_INVALID,
                  "b2g_compress_24_format (fp4 / fp6): K %% 32 == 0 and 16-byte alignment needed");
    if (M * K == 0) return B2G_OK;
    DeviceGuard g(h->device);
    // the sign bit is left out of the zero test (-0 counts as zero)
    B2G_CUDA(h, launch_compress_24_sub((const uint8_t*)d_dense, M, K, bits, bits == 4 ? 0x7u : 0x1Fu,
                                       (uint8_t*)d_comp, (uint32_t*)d_meta, h->d_err, h->sm_count,
                                       reinterpret_cast<cudaStream_t>(stream)));
    return B2G_OK;
  }
  if (bits == 32) {  // tf32 1:2: metadata [M][K/16] words
    if (!d_dense || !d_comp || !d_meta || M < 0 || K < 0 || K % 16 ||
        ((reinterpret_cast<uintptr_t>(d_dense) | reinterpret_cast<uintptr_t>(d_comp)) & 15) ||
        (reinterpret_cast<uintptr_t>(d_meta) & 3))
      return fail(h, B2G_ERR_INVALID,
                  "b2g_compress_24_format (tf32): K %% 16 == 0 and 16-byte alignment needed");
    if (M * K == 0) return B2G_OK;
    DeviceGuard g(h->device);
    B2G_CUDA(h, launch_compress_12_f32((const uint32_t*)d_dense, M, K, (uint32_t*)d_comp,
                                       (uint32_t*)d_meta, h->d_err, h->sm_count,
                                       reinterpret_cast<cudaStream_t>(stream)));
    return B2G_OK;
  }
  if (!d_dense || !d_comp || !d_meta || M < 0 || K < 0 || K % 32 ||
      ((reinterpret_cast<uintptr_t>(d_dense) | reinterpret_cast<uintptr_t>(d_comp)) & 15) ||
      (reinterpret_cast<uintptr_t>(d_meta) & 3))
    return fail(h, B2G_ERR_INVALID, "b2g_compress_24_format: K %% 32 == 0 and 16-byte alignment needed");
  if (M * K == 0) return B2G_OK;
  DeviceGuard g(h->device);
  // non-zero test: the fp8 formats ignore the sign bit (0x80 is -0), the integers do not
  const uint32_t nz_mask =
      (format == B2G_FMT_E4M3 || format == B2G_FMT_E5M2 || format == B2G_FMT_MXF8) ? 0x7Fu : 0xFFu;
  B2G_CUDA(h, launch_compress_24_u8((const uint8_t*)d_dense, M, K, nz_mask, (uint8_t*)d_comp,
                                    (uint32_t*)d_meta, h->d_err, h->sm_count,
                                    reinterpret_cast<cudaStream_t>(stream)));
  return B2G_OK;
}

b2g_status b2g_prune_24_format(b2g_handle* h, int format, void* d, int64_t rows, int64_t cols,
                               int64_t row0, uint64_t seed, void* stream) {
  if (!h) return B2G_ERR_INVALID;
  if (format == B2G_FMT_MXF4 || format == B2G_FMT_NVFP4) {  // 4:8 in pairs: 2 of every 4
                                                             // bytes (pairs) zeroed
    if (!d || rows < 0 || cols < 0 || row0 < 0 || cols % 8 || (reinterpret_cast<uintptr_t>(d) & 3))
      return fail(h, B2G_ERR_INVALID,
                  "b2g_prune_24_format (MXFP4): cols %% 8 == 0 and 4-byte alignment needed");
    if (rows * cols == 0) return B2G_OK;
    DeviceGuard g(h->device);
    B2G_CUDA(h, launch_prune_24_u8((uint8_t*)d, rows, cols / 2, row0, seed, h->sm_count,
                                   reinterpret_cast<cudaStream_t>(stream)));
    return B2G_OK;
  }
  const int bits = sparse_elem_bits(format);
  if (!bits) return fail(h, B2G_ERR_UNSUPPORTED, "b2g_prune_24_format: format %d", format);
  if (bits == 16) return b2g_prune_24(h, d, rows, cols, row0, seed, stream);
  if (bits == 4 || bits == 6) {  // packed fp4 / fp6 codes, whole 16-element groups
    if (!d || rows < 0 || cols < 0 || row0 < 0 || cols % 16 || (reinterpret_cast<uintptr_t>(d) & 3))
      return fail(h, B2G_ERR_INVALID,
                  "b2g_prune_24_format (fp4 / fp6): cols %% 16 == 0 and 4-byte alignment needed");
    if (rows * cols == 0) return B2G_OK;
    DeviceGuard g(h->device);
    B2G_CUDA(h, launch_prune_24_sub((uint8_t*)d, rows, cols, row0, bits, seed, h->sm_count,
                                    reinterpret_cast<cudaStream_t>(stream)));
    return B2G_OK;
  }
  if (bits == 32) {  // tf32 1:2
    if (!d || rows < 0 || cols < 0 || row0 < 0 || cols % 2 || (reinterpret_cast<uintptr_t>(d) & 7))
      return fail(h, B2G_ERR_INVALID,
                  "b2g_prune_24_format (tf32): cols %% 2 == 0 and 8-byte alignment needed");
    if (rows * cols == 0) return B2G_OK;
    DeviceGuard g(h->device);
    B2G_CUDA(h, launch_prune_12_f32((uint32_t*)d, rows, cols, row0, seed, h->sm_count,
                                    reinterpret_cast<cudaStream_t>(stream)));
    return B2G_OK;
  }
  if (!d || rows < 0 || cols < 0 || row0 < 0 || cols % 4 || (reinterpret_cast<uintptr_t>(d) & 3))
    return fail(h, B2G_ERR_INVALID, "b2g_prune_24_format: cols %% 4 == 0 and 4-byte alignment needed");
  if (rows * cols == 0) return B2G_OK;
  DeviceGuard g(h->device);
  B2G_CUDA(h, launch_prune_24_u8((uint8_t*)d, rows, cols, row0, seed, h->sm_count,
                                 reinterpret_cast<cudaStream_t>(stream)));
  return B2G_OK;
}

// ------------------------------------------------------------------ probes (later)
b2g_status b2g_stream_tma2d(b2g_handle* h, const float* d_data, uint64_t width, uint64_t height,
                            int ctas_per_sm, int num_stages, int box_w, int box_h,
                            float* elapsed_ms, void* stream) {
  if (!h || !d_data) return B2G_ERR_INVALID;
  if (width == 0 || height == 0 || (width * 4) % 16 || (reinterpret_cast<uintptr_t>(d_data) & 15))
    return fail(h, B2G_ERR_INVALID, "b2g_stream_tma2d: rows must be multiples of 16 bytes");
  if (box_w < 4 || box_w > 256 || box_w % 4 || (uint64_t)box_w > width || box_h < 1 ||
      box_h > 256 || num_stages < 1 || num_stages > 16 || ctas_per_sm < 1 || ctas_per_sm > 32)
    return fail(h, B2G_ERR_INVALID,
                "b2g_stream_tma2d: box 4..256 (x4) by 1..256, stages 1..16, ctas_per_sm 1..32");
  const size_t box_bytes = (size_t)box_w * (size_t)box_h * 4;
  const size_t smem = box_bytes * (size_t)num_stages + 1024;
  if (smem > 227 * 1024)
    return fail(h, B2G_ERR_INVALID, "b2g_stream_tma2d: %d stages of %zu bytes exceed shared memory",
                num_stages, box_bytes);
  DeviceGuard g(h->device);
  CUtensorMap tm;
  b2g_status st = make_tmap_2d(h, &tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, d_data, width, height,
                               width * 4, (uint32_t)box_w, (uint32_t)box_h,
                               CU_TENSOR_MAP_SWIZZLE_NONE);
  if (st != B2G_OK) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  B2G_CUDA(h, tma2d_stream_prepare((int)smem));  // set-up outside the timed interval
  cudaEvent_t e0, e1;
  B2G_CUDA(h, cudaEventCreate(&e0));
  B2G_CUDA(h, cudaEventCreate(&e1));
  B2G_CUDA(h, cudaEventRecord(e0, s));
  cudaError_t le = tma2d_stream_launch(tm, height, box_w, box_h, num_stages,
                                       h->sm_count * ctas_per_sm, (int)smem, h->d_err, s);
  B2G_CUDA(h, cudaEventRecord(e1, s));
  B2G_CUDA(h, cudaEventSynchronize(e1));
  float ms = 0.0f;
  cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  B2G_CUDA(h, le);
  if (elapsed_ms) *elapsed_ms = ms;
  return b2g_check(h, stream);
}

b2g_status b2g_tma2d_latency(b2g_handle* h, const float* d_data, uint64_t width, uint64_t height,
                             int box_w, int box_h, int ctas_per_sm, int64_t row0,
                             uint32_t* d_cycles, void* stream) {
  if (!h || !d_data || !d_cycles) return B2G_ERR_INVALID;
  if (width == 0 || height == 0 || (width * 4) % 16 || (reinterpret_cast<uintptr_t>(d_data) & 15))
    return fail(h, B2G_ERR_INVALID, "b2g_tma2d_latency: rows must be multiples of 16 bytes");
  if (box_w < 4 || box_w > 256 || box_w % 4 || (uint64_t)box_w > width || box_h < 1 ||
      box_h > 256 || ctas_per_sm < 1 || ctas_per_sm > 32 || row0 < 0)
    return fail(h, B2G_ERR_INVALID, "b2g_tma2d_latency: box 4..256 (x4) by 1..256, ctas_per_sm 1..32");
  const int grid = h->sm_count * ctas_per_sm;
  if ((uint64_t)row0 + (uint64_t)grid * (uint64_t)box_h > height || row0 + (int64_t)grid * box_h > INT32_MAX)
    return fail(h, B2G_ERR_INVALID, "b2g_tma2d_latency: rows row0 .. row0 + CTAs x box_h outside the data");
  DeviceGuard g(h->device);
  CUtensorMap tm;
  b2g_status st = make_tmap_2d(h, &tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, d_data, width, height,
                               width * 4, (uint32_t)box_w, (uint32_t)box_h,
                               CU_TENSOR_MAP_SWIZZLE_NONE);
  if (st != B2G_OK) return st;
  // all the shared memory a block may take, whatever the box, so that the carveout
  // is the same for every configuration (as the reference pins it)
  int smem = 0;
  B2G_CUDA(h, tma2d_latency_smem(h->device, &smem));
  if ((size_t)box_w * (size_t)box_h * 4 + 1024 > (size_t)smem)
    return fail(h, B2G_ERR_INVALID, "b2g_tma2d_latency: a %d x %d box exceeds shared memory", box_w,
                box_h);
  B2G_CUDA(h, tma2d_latency_launch(tm, row0, box_w, box_h, grid, smem, d_cycles, h->d_err,
                                   reinterpret_cast<cudaStream_t>(stream)));
  return b2g_check(h, stream);
}

b2g_status b2g_stream_bulk1d(b2g_handle* h, const void* d_data, uint64_t bytes, int ctas_per_sm,
                             int num_stages, uint32_t load_bytes, float* elapsed_ms,
                             void* stream) {
  if (!h || !d_data) return B2G_ERR_INVALID;
  if (load_bytes < 16 || load_bytes % 16 || (reinterpret_cast<uintptr_t>(d_data) & 15) ||
      bytes == 0 || bytes % load_bytes)
    return fail(h, B2G_ERR_INVALID,
                "b2g_stream_bulk1d: 16-byte aligned data, load_bytes a multiple of 16 dividing bytes");
  if (num_stages < 1 || num_stages > 16 || ctas_per_sm < 1 || ctas_per_sm > 32)
    return fail(h, B2G_ERR_INVALID, "b2g_stream_bulk1d: stages 1..16, ctas_per_sm 1..32");
  const size_t smem = (size_t)load_bytes * (size_t)num_stages;
  if (smem > 227 * 1024)
    return fail(h, B2G_ERR_INVALID, "b2g_stream_bulk1d: %d stages of %u bytes exceed shared memory",
                num_stages, load_bytes);
  DeviceGuard g(h->device);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  B2G_CUDA(h, bulk1d_stream_prepare((int)smem));  // set-up outside the timed interval
  cudaEvent_t e0, e1;
  B2G_CUDA(h, cudaEventCreate(&e0));
  B2G_CUDA(h, cudaEventCreate(&e1));
  B2G_CUDA(h, cudaEventRecord(e0, s));
  cudaError_t le = bulk1d_stream_launch(d_data, bytes / load_bytes, load_bytes, num_stages,
                                        h->sm_count * ctas_per_sm, (int)smem, h->d_err, s);
  B2G_CUDA(h, cudaEventRecord(e1, s));
  B2G_CUDA(h, cudaEventSynchronize(e1));
  float ms = 0.0f;
  cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  B2G_CUDA(h, le);
  if (elapsed_ms) *elapsed_ms = ms;
  return b2g_check(h, stream);
}

// Shapes the probe accepts: the tcgen05 shape tables restricted to the points the
// reference's own sweeps run (umma_throughput/benchmark.py:26-43,
// tcgen05_sparse_mma/benchmark.py:215-218), so that no launch carries an
// instruction shape outside what the hardware documents.
// Element type codes each kind takes (the instruction descriptor's A / B type
// fields): a code outside its kind's set makes the MMA an illegal instruction on the
// device, so the host refuses it first.
static bool probe_type_ok(int kind, int code) {
  switch (kind) {
    case KIND_TF32: return code == 2;
    case KIND_F16: return code == 0 || code == 1;
    case KIND_F8F6F4:
    case KIND_MXF8F6F4: return code == 0 || code == 1 || code == 3 || code == 4 || code == 5;
    case KIND_I8: return code == 0 || code == 1;
    case KIND_MXF4:
    case KIND_MXF4NVF4: return code == 1;  // e2m1 (the kinds' own code)
    default: return false;
  }
}

static const char* probe_shape_error(const b2g_probe_desc* p) {
  const bool bs = p->kind >= 4;
  if (p->kind < 0 || p->kind > 6) return "kind must be 0..6";
  if (!probe_type_ok(p->kind, p->a_type) || !probe_type_ok(p->kind, p->b_type))
    return "A / B type code outside the kind's element types (f8f6f4 / mxf8f6f4: 0, 1, 3, 4, 5; "
           "f16: 0, 1; i8: 0, 1; tf32: 2; mxf4 / mxf4nvf4: 1)";
  if (p->kind == KIND_F16 && p->a_type != p->b_type) return "kind::f16 takes one type for A and B";
  if (p->scale_type != 0 && p->scale_type != 1) return "scale_type must be 0 (ue4m3) or 1 (ue8m0)";
  if ((p->kind == KIND_MXF8F6F4 || p->kind == KIND_MXF4) && p->scale_type != 1)
    return "mxf8f6f4 and mxf4 take ue8m0 scales (scale_type 1)";
  if (p->sparse != 0 && p->sparse != 1) return "sparse must be 0 or 1";
  if (p->ab_mode != 0 && p->ab_mode != 1) return "ab_mode must be 0 (SS) or 1 (TS)";
  if (p->cta_group != 1 && p->cta_group != 2) return "cta_group must be 1 or 2";
  if (p->instruction != 0 && p->instruction != 1) return "instruction must be 0 (mma) or 1 (ws)";
  if (p->n < 64 || p->n > 256 || p->n % 16) return "N must be a multiple of 16 in [64, 256]";
  if (p->depth < 1 || p->depth > 4096) return "depth must be in [1, 4096]";
  if (p->instruction == 1) {
    if (p->cta_group != 1) return ".ws is cta_group::1 only";
    if (bs) return ".ws is not block-scaled";
    if (p->m != 32 && p->m != 64 && p->m != 128) return ".ws needs M in {32, 64, 128}";
    if (p->n != 64 && p->n != 128 && p->n != 256) return ".ws needs N in {64, 128, 256}";
    return nullptr;
  }
  if (p->sparse) {
    if (p->m != 128 * p->cta_group) return "sparse needs M = 128 (cta_group 1) or 256 (cta_group 2)";
    return nullptr;
  }
  if (p->cta_group == 1) {
    if (bs ? p->m != 128 : (p->m != 64 && p->m != 128)) return "cta_group 1 needs M in {64, 128} (128 block-scaled)";
  } else if (p->m != 128 && p->m != 256) {
    return "cta_group 2 needs M in {128, 256}";
  }
  return nullptr;
}

b2g_status b2g_probe_mma(b2g_handle* h, const b2g_probe_desc* p, uint64_t* cycles,
                         uint64_t* total_mmas, uint64_t* median_cycles) {
  if (!h || !p) return B2G_ERR_INVALID;
  const char* why = probe_shape_error(p);
  if (why) return fail(h, B2G_ERR_INVALID, "b2g_probe_mma: %s", why);
  if (p->mode != 0 && p->mode != 1) return fail(h, B2G_ERR_INVALID, "mode must be 0 or 1");
  DeviceGuard g(h->device);
  if (!h->d_probe) B2G_CUDA(h, cudaMalloc(&h->d_probe, 4 * sizeof(unsigned long long)));
  int kid = p->kind;
  if (kid == KIND_MXF4NVF4 && p->scale_type == 0) kid = 7;  // ue4m3 scales: block16 (NVFP4)
  ProbeArgs a;
  memset(&a, 0, sizeof(a));
  a.idesc = encode_idesc(p->kind, p->a_type, p->b_type, p->m, p->n, p->sparse, p->scale_type);
  a.a_rows = p->m / p->cta_group;
  a.b_rows = p->n;
  a.depth = p->depth;
  a.iters = p->mode == 0 ? (p->iters > 0 ? p->iters : 1000) : 100;
  a.mode = p->mode;
  a.d_col = 0;
  a.a_col = (uint32_t)((p->n + 15) / 16 * 16);  // 16 columns of TS A
  a.sf_col = a.a_col + 16;                      // SFA 4 + SFB 8 columns
  a.meta_col = a.sf_col + 16;                   // sparse metadata, 4 columns
  uint32_t cols = 32;
  while (cols < a.meta_col + 4) cols <<= 1;
  a.tmem_cols = cols;
  a.sf_word = p->scale_type ? 0x7F7F7F7Fu : 0x38383838u;  // 1.0 as ue8m0 / ue4m3
  a.result = reinterpret_cast<unsigned long long*>(h->d_probe);
  a.err = h->d_err;
  const size_t smem = (size_t)(a.a_rows + a.b_rows) * 128 + 1024;
  B2G_CUDA(h, cudaMemset(h->d_probe, 0, 4 * sizeof(unsigned long long)));
  B2G_CUDA(h, probe_launch(kid, p->sparse, p->instruction, p->cta_group, p->ab_mode, a, smem, 0));
  b2g_status st = b2g_check(h, nullptr);
  if (st != B2G_OK) return st;
  unsigned long long r[4];
  B2G_CUDA(h, cudaMemcpy(r, h->d_probe, sizeof(r), cudaMemcpyDeviceToHost));
  if (cycles) *cycles = r[0];
  if (total_mmas) *total_mmas = r[1];
  if (median_cycles) *median_cycles = r[2];
  return B2G_OK;
}

}  // extern "C"
