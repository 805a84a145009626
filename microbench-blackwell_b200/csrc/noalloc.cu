// noalloc.cu -- b2g_gemm_sparse_noalloc: the 2:4 sparse GEMM for callers that
// cannot allocate device memory.
//
// b2g_gemm needs a handle, and a handle owns device memory: b2g_create allocates
// its error word, and the sparse path allocates the scratch buffer that holds
// the metadata in the engine's TMEM-ready layout.  Some callers cannot call
// cudaMalloc at all.  Examples: a plugin hosted by a framework whose caching
// allocator owns every byte of device memory (a private cudaMalloc there
// bypasses its accounting and can fail once the pool has reserved the GPU);
// code in a latency-critical serving loop, where cudaMalloc and cudaFree may
// synchronise the device; and code that runs with device memory fully
// pre-reserved for a fixed budget.  This entry point takes no handle and
// allocates nothing.  Its scratch -- one error word and the reordered metadata
// -- lives in the file-scope static array below, which every GPU that loads the
// library holds until the process exits.
//
// Limits and sharing:
//   * the metadata scratch holds at most kNoAllocMetaMax = 16 MiB.  The engine
//     layout takes ceil(M / 128) * ceil(K / 128) * 2048 bytes, so the limit is
//     ceil(M / 128) * ceil(K / 128) <= 8192 (for example M = 8192, K = 16384);
//     larger problems are rejected with B2G_ERR_INVALID and a message;
//   * every call uses the same array.  Calls that overlap on the GPU (two
//     streams, two host threads) race on it and corrupt each other's result.
//     Serialise them.  The error word is cleared at the start of every call; the
//     metadata region is rewritten in full for the call's M x K;
//   * the first call on a device looks up the array's device address
//     (cudaGetSymbolAddress) with that device current, and the address is kept
//     for that device's context; a call that finds a different context (after
//     cudaDeviceReset, for example) looks it up again.  Make the first call on a
//     device before any stream capture;
//   * the call synchronises `stream` before it returns, to report kernel-side
//     wait timeouts through its status.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "b2g.h"
#include "b2g_desc.h"
#include "b2g_gemm.h"

using namespace b2g;

namespace {

constexpr size_t kNoAllocHeader = 256;           // error word, padded to one 256-byte line
constexpr size_t kNoAllocMetaMax = 16u << 20;    // engine-layout metadata, bytes
constexpr int kMaxDevices = 64;

typedef CUresult (*PFN_encodeTiled_noalloc)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                            const cuuint64_t*, const cuuint64_t*,
                                            const cuuint32_t*, const cuuint32_t*,
                                            CUtensorMapInterleave, CUtensorMapSwizzle,
                                            CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

typedef CUresult (*PFN_ctxGetCurrent_noalloc)(CUcontext*);
typedef CUresult (*PFN_ctxGetId_noalloc)(CUcontext, unsigned long long*);

std::mutex g_setup_mu;
uint8_t* g_scratch_dev[kMaxDevices];            // device address of the array, per device
unsigned long long g_scratch_ctx[kMaxDevices];  // unique id of the context it belongs to
PFN_encodeTiled_noalloc g_encode = nullptr;
PFN_ctxGetCurrent_noalloc g_ctx_current = nullptr;
PFN_ctxGetId_noalloc g_ctx_id = nullptr;
thread_local char g_msg[256];

b2g_status say(const char** err_msg, b2g_status s, const char* text) {
  snprintf(g_msg, sizeof(g_msg), "b2g_gemm_sparse_noalloc: %s", text);
  if (err_msg) *err_msg = g_msg;
  return s;
}

}  // namespace

// The scratch itself: [0, 256) error word, [256, 256 + 16 MiB) metadata.
static __device__ __align__(256) uint8_t g_b2g_noalloc_scratch[kNoAllocHeader + kNoAllocMetaMax];

static void* driver_entry(const char* name) {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &fn, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess)
    return nullptr;
  return fn;
}

// Once per device and context, with that device current: the array's device
// address.  In host code the symbol is only a host-side stand-in and must never
// be passed to a kernel.
static b2g_status noalloc_setup(int dev, uint8_t** scratch, const char** err_msg) {
  std::lock_guard<std::mutex> lk(g_setup_mu);
  if (!g_encode) {
    g_encode = reinterpret_cast<PFN_encodeTiled_noalloc>(driver_entry("cuTensorMapEncodeTiled"));
    g_ctx_current = reinterpret_cast<PFN_ctxGetCurrent_noalloc>(driver_entry("cuCtxGetCurrent"));
    g_ctx_id = reinterpret_cast<PFN_ctxGetId_noalloc>(driver_entry("cuCtxGetId"));
    if (!g_encode || !g_ctx_current || !g_ctx_id) {
      g_encode = nullptr;
      return say(err_msg, B2G_ERR_CUDA, "CUDA driver entry points not found");
    }
  }
  // the runtime made the device's primary context current (cudaGetDevice /
  // cudaDeviceGetAttribute ran before this); its unique id tells whether the
  // cached address still belongs to a live context
  CUcontext ctx = nullptr;
  unsigned long long ctx_id = 0;
  if (g_ctx_current(&ctx) != CUDA_SUCCESS || !ctx || g_ctx_id(ctx, &ctx_id) != CUDA_SUCCESS)
    return say(err_msg, B2G_ERR_CUDA, "no current CUDA context");
  if (!g_scratch_dev[dev] || g_scratch_ctx[dev] != ctx_id) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_b2g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      char buf[160];
      snprintf(buf, sizeof(buf), "cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return say(err_msg, B2G_ERR_CUDA, buf);
    }
    g_scratch_dev[dev] = static_cast<uint8_t*>(p);
    g_scratch_ctx[dev] = ctx_id;
  }
  *scratch = g_scratch_dev[dev];
  return B2G_OK;
}

static bool tmap_2d(CUtensorMap* tm, CUtensorMapDataType dt, const void* base, uint64_t inner,
                    uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                    CUtensorMapSwizzle swz) {
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  return g_encode(tm, dt, 2, const_cast<void*>(base), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

extern "C" b2g_status b2g_gemm_sparse_noalloc(const b2g_gemm_desc* d, void* stream,
                                              const char** err_msg) {
  if (err_msg) *err_msg = nullptr;
  if (!d) return say(err_msg, B2G_ERR_INVALID, "null descriptor");
  if (d->format != B2G_FMT_BF16 || d->sparse != 1 || d->meta_layout != 0 || d->ab_mode != 0)
    return say(err_msg, B2G_ERR_INVALID,
               "needs format bf16, sparse = 1, meta_layout = 0 (canonical metadata), ab_mode = 0");
  if (d->M <= 0 || d->N <= 0 || d->K <= 0 || d->K % 32 || d->M > INT32_MAX / 2 ||
      d->N > INT32_MAX / 2 || d->K > INT32_MAX / 2)
    return say(err_msg, B2G_ERR_INVALID, "M, N, K must be positive, K a multiple of 32");
  if (!d->A || !d->B || !d->C || !d->meta)
    return say(err_msg, B2G_ERR_INVALID, "null A, B, C or metadata pointer");
  const size_t meta_bytes = meta_ready_bytes(d->M, d->K);
  if (meta_bytes > kNoAllocMetaMax) {
    char buf[200];
    snprintf(buf, sizeof(buf),
             "the metadata takes ceil(M/128) * ceil(K/128) * 2048 = %zu bytes, above the "
             "16 MiB static scratch (ceil(M/128) * ceil(K/128) must be at most 8192)",
             meta_bytes);
    return say(err_msg, B2G_ERR_INVALID, buf);
  }
  if (d->lda < d->K / 2 || d->ldb < d->K || d->ldc < d->N || (d->lda * 2) % 16 ||
      (d->ldb * 2) % 16 ||
      ((reinterpret_cast<uintptr_t>(d->A) | reinterpret_cast<uintptr_t>(d->B)) & 15) ||
      (reinterpret_cast<uintptr_t>(d->meta) & 3) || (reinterpret_cast<uintptr_t>(d->C) & 1))
    return say(err_msg, B2G_ERR_INVALID, "leading dimensions or alignment (16-byte rows) invalid");

  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return say(err_msg, B2G_ERR_NO_DEVICE, "no current CUDA device");
  int major = 0, sms = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (major != 10 || sms <= 0) return say(err_msg, B2G_ERR_NO_DEVICE, "current device is not sm_100");
  uint8_t* scratch = nullptr;
  b2g_status st = noalloc_setup(dev, &scratch, err_msg);
  if (st != B2G_OK) return st;
  uint32_t* err_word = reinterpret_cast<uint32_t*>(scratch);
  uint32_t* ready = reinterpret_cast<uint32_t*>(scratch + kNoAllocHeader);

  // configuration: the planner b2g_gemm uses (b2g_plan_gemm), with whole tiles,
  // since a split tail needs workspace
  b2g_gemm_desc pd = *d;
  pd.split_tail = 1;
  pd.instruction = 0;  // the ordinary tcgen05.mma form
  b2g_gemm_plan plan;
  char plan_msg[200];
  if (b2g_plan_gemm(&pd, sms, 0, &plan, plan_msg, sizeof(plan_msg)) != B2G_OK)
    return say(err_msg, B2G_ERR_INVALID, plan_msg);
  if (plan.cta_group == 2) {  // co-resident cluster pairs under this shared-memory footprint
    int mc = 0;
    if (gemm_max_active_clusters(KIND_F16, 2, GEMM_SPARSE, false, plan.m_sub, 1, false,
                                 plan.smem_bytes, &mc) == cudaSuccess &&
        mc > 0 && mc < plan.clusters &&
        b2g_plan_gemm(&pd, sms, mc, &plan, plan_msg, sizeof(plan_msg)) != B2G_OK)
      return say(err_msg, B2G_ERR_INVALID, plan_msg);
  }
  const int cg = plan.cta_group, bn = plan.tile_n, m_sub = plan.m_sub;
  const int b_rows = bn / cg;
  const size_t smem = (size_t)plan.smem_bytes;

  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(err_word, 0, sizeof(uint32_t), s) != cudaSuccess)
    return say(err_msg, B2G_ERR_CUDA, "clearing the error word failed");
  if (launch_meta_ready(static_cast<const uint32_t*>(d->meta), d->M, d->K, ready, sms, s) !=
      cudaSuccess)
    return say(err_msg, B2G_ERR_CUDA, "metadata reorder launch failed");

  const int64_t k_blocks = plan.k_blocks;
  GemmMaps maps;
  memset(&maps, 0, sizeof(maps));
  if (!tmap_2d(&maps.a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, d->A, (uint64_t)(d->K / 2), (uint64_t)d->M,
               (uint64_t)(d->lda * 2), 64, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !tmap_2d(&maps.b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, d->B, (uint64_t)d->K, (uint64_t)d->N,
               (uint64_t)(d->ldb * 2), 64, (uint32_t)b_rows, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !tmap_2d(&maps.e, CU_TENSOR_MAP_DATA_TYPE_UINT8, ready, kSideLine,
               (uint64_t)((d->M + 127) / 128) * (uint64_t)k_blocks * (2048 / kSideLine),
               kSideLine, kSideLine, 2048 / kSideLine, CU_TENSOR_MAP_SWIZZLE_NONE))
    return say(err_msg, B2G_ERR_CUDA, "cuTensorMapEncodeTiled failed");

  GemmArgs a;
  memset(&a, 0, sizeof(a));
  a.M = (int)d->M;
  a.N = (int)d->N;
  a.num_m_tiles = plan.num_m_tiles;
  a.num_n_tiles = plan.num_n_tiles;
  a.k_blocks = (int)k_blocks;
  a.tile_n = bn;
  a.stages = plan.stages;
  a.group_m = plan.raster_m;
  a.elem_bits = 16;
  a.idesc = encode_idesc(KIND_F16, 1, 1, 128 * cg, bn, 1, 0);
  a.alpha = d->alpha;
  a.C = reinterpret_cast<__nv_bfloat16*>(d->C);
  a.ldc = d->ldc;
  a.c_vec_ok = ((reinterpret_cast<uintptr_t>(d->C) & 15) == 0 && (d->ldc % 8) == 0) ? 1 : 0;
  a.err = err_word;
  a.trace = nullptr;

  a.tail_start = plan.tail_start;  // whole tiles: tail_split 1
  a.tail_split = plan.tail_split;
  if (gemm_launch(KIND_F16, cg, GEMM_SPARSE, false, m_sub, 1, false, maps, a, plan.clusters * cg,
                  smem, s) != cudaSuccess)
    return say(err_msg, B2G_ERR_CUDA, "GEMM launch failed");

  // Synchronous: report kernel-side wait timeouts through the return code.
  uint32_t w = 0;
  if (cudaMemcpyAsync(&w, err_word, sizeof(w), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return say(err_msg, B2G_ERR_CUDA, cudaGetErrorString(cudaGetLastError()));
  if (w) return say(err_msg, B2G_ERR_TIMEOUT, "a kernel-side wait timed out");
  return B2G_OK;
}
